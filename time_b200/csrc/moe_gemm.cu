// moe_gemm.cu -- grouped, 128x128 block-scaled FP8 expert GEMM for sm_100a.
//
// Replaces the reference's per-top-k-slot "launch_fp8_dequantize + cbwSgemm"
// expert loop (src/terra/engine.t:1321-1346; intended semantics
// src/futhark/kernels.fut:343-368) with one persistent kernel per projection:
//
//   gate/up  (CBW_GEMM_GATED_SWIGLU): h = silu(W_gate x) * (W_up x), quantised
//            to e4m3 with one fp32 scale per 128 output columns (the input
//            format of the down projection);
//   down     (CBW_GEMM_DOWN_BF16):    y = W_down h, written as bf16.
//
// Design (one CTA per SM, persistent over a device-built tile list):
//   * Operands are "swap-AB": the UMMA M side (128 lanes of TMEM) is 128
//     weight rows -- exactly one 128x128 scale block -- and the N side is up
//     to N_MAX tokens of one expert, so ragged expert groups pad only to 16
//     tokens.  Tiles of one (expert, weight-row block) are adjacent in the
//     list, so concurrently running CTAs share each weight tile through L2.
//   * warp 0: TMA producer (weights box 128x128 B, tokens in 32-row boxes)
//     into a 3-deep operand ring that the MMA commit alone releases, and the
//     K block's token scales (bulk copy) into a separate 8-deep scale ring that
//     the promotion warps release -- so operand loads never wait for promotion.
//   * warp 1: allocates TMEM (512 columns) and issues tcgen05.mma kind::f8f6f4
//     (4 x K=32 per 128-wide K block) into one of two TMEM partial buffers;
//     a fresh partial per K block, since the fp32 block scales differ per K
//     block and tcgen05's own block scaling only takes power-of-two scales.
//   * warp 2: folds the K block's weight scale into the token scales in place
//     (c[n] = a_scale[n] * w_scale) once per CTA per K block.
//   * warps 4..19 (warpgroups 1-4, 112 registers each after setmaxnreg; the
//     role warpgroup drops to 32): "promotion": tcgen05.ld the partial (16
//     columns per load, four per K block), acc += partial * c with packed fp32x2 FMAs in
//     registers, release the TMEM buffer and the scale entry; at the
//     end of a tile run the fused epilogue (SwiGLU + requant, or bf16) through
//     a transposing shared-memory stage so global stores are row-contiguous.
//   * Every mbarrier wait is bounded (~2 s); on timeout the CTA raises an
//     abort flag, drains its own TMA/MMA work, frees TMEM and reports through
//     the error word instead of hanging the GPU.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cooperative_groups.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "sm100.cuh"
#include "cublas_wrappers.h"

namespace {

using namespace tb;

constexpr int kBlockK = 128;            // K bytes (e4m3 elements) per stage
constexpr int kTileM = 128;             // weight rows per UMMA (TMEM lanes)
constexpr int kFirstPromoWarp = 4;      // warpgroup 0: TMA, MMA, scale folding, idle
constexpr int kNumPromoWarps = 16;      // warpgroups 1..4
constexpr int kNumThreads = (kFirstPromoWarp + kNumPromoWarps) * 32;   // 640
// Register split (setmaxnreg): launched at 96 per thread (640 x 96 = 61440),
// warpgroup 0 gives back to 32, the four promotion warpgroups take 112:
// 128 x 32 + 512 x 112 = 61440, and per SM sub-partition 1 x 32 x 32 +
// 4 x 32 x 112 = 15360 <= 16384.
constexpr int kRoleRegs = 32;
constexpr int kPromoRegs = 112;
static_assert(128 * kRoleRegs + 512 * kPromoRegs <= kNumThreads * 96, "register split exceeds the launch");
constexpr int kMaxGroups = 512;
constexpr int kTmemCols = 512;
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;
constexpr uint64_t kDrainTimeoutNs = 200000000ull;

// kSmall: the decode form.  A tile holds at most 32 tokens, so an operand
// stage shrinks to the weights plus 4 KB and the ring holds 4 (gated) or 9
// (down) stages instead of 3 -- with a few tokens per expert the GEMM is a
// weight stream.  Its rate is then set by the per-K-block promotion chain
// (TMEM loads, fold, release), so the four promotion column groups, which
// all cover the tile's 32 columns here, share the K blocks: group j folds the
// tile's K blocks kb = j (mod 4); TMEM holds eight 64-column partial buffers
// (gate at +0, up at +32); at the end of a tile the groups' sums are added in
// group order 0, 1, 2, 3 through shared memory.  The sum order differs from
// the full form's, so one caller should use one form for comparable results.
template <bool kGated, bool kSmall = false, bool kX2 = false>
struct GemmCfg {
    static constexpr int kPlanes = kX2 ? 2 : 1;            // activation e4m3 planes: hi (+ lo residual)
    static constexpr int kNMax = kGated ? 128 : 256;       // token columns of the promotion layout
    static constexpr int kTileTok = kSmall ? 32 : kNMax;   // tokens per tile
    static constexpr int kStages = kX2 ? (kSmall ? (kGated ? 3 : 6) : 2)
                                       : (kSmall ? (kGated ? 4 : 9) : 3);   // operand ring
    static constexpr int kSStages = 8;                      // token-scale ring
    static constexpr int kATiles = kGated ? 2 : 1;          // gate + up
    static constexpr int kABytes = kATiles * kTileM * kBlockK;
    static constexpr int kBBytes = kPlanes * kTileTok * kBlockK;   // [plane][tokens][128 B]
    static constexpr int kStageBytes = kABytes + kBBytes;   // 48 KB; small: 36 KB gated, 20 KB down (one plane)
    static constexpr int kTBufs = kSmall ? 8 : 2;           // TMEM partial buffers
    static constexpr int kTBufColsSm = 64;                  // small form: columns per buffer
    static constexpr int kNumCombined = kGated ? 2 : 1;
    static constexpr int kScaleFloats = kNumCombined * kNMax;   // one scale-ring entry
    static constexpr int kRawSlot = kNumCombined - 1;       // where the bulk copy lands in an entry
    static constexpr int kBufCols = kSmall ? kTBufColsSm : 256;   // TMEM columns per partial buffer
    static constexpr int kUpOff = kSmall ? 32 : 128;        // the up partial's columns within a buffer
    static constexpr int kPromoGroups = kSmall ? 4 : 1;     // column groups sharing a tile's K blocks
    static constexpr int kColsPerWarp = kNMax / 4;          // 32 (gated) / 64 (down)
    static constexpr int kOutStageBytes = kGated ? kTileTok * 128 * 4 : kTileTok * 128 * 2;
    // small form: the column groups' sums, [64 (gated) / 32 columns][128 rows] fp32
    static constexpr int kRedBytes = kSmall ? (kGated ? 64 : 32) * 128 * 4 : 0;
    // shared-memory carve-up (offsets from the 1024-aligned base)
    static constexpr int kOffStages = 0;
    static constexpr int kOffOut = kOffStages + kStages * kStageBytes;
    static constexpr int kOffRed = kOffOut + kOutStageBytes;
    static constexpr int kOffScale = kOffRed + kRedBytes;
    static constexpr int kOffTables = kOffScale + kSStages * kScaleFloats * 4;
    static constexpr int kOffBars = kOffTables + (4 * kMaxGroups + 2) * 4;   // prefix, chunks, start, count
    // full/empty per operand stage; sfull/sempty/cready per scale entry;
    // tfull/tempty per TMEM buffer; one epilogue group barrier
    static constexpr int kNumBars = 2 * kStages + 3 * kSStages + 2 * kTBufs + 1;
    static constexpr int kOffMisc = kOffBars + kNumBars * 8;
    static constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack
    static_assert(kOffBars % 8 == 0, "mbarrier alignment");
    static_assert(kStageBytes % 1024 == 0, "128-byte-swizzled stages start on 1024-byte boundaries");
    static_assert(kStages <= 32 && kSStages <= 32, "armed masks hold one bit per stage");
    static_assert(kTBufs * kBufCols <= kTmemCols, "TMEM partial buffers");
    static_assert(!kSmall || (kSStages == 8 && kTBufs == 8), "small form: ring positions from the K-block count");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
    static_assert(!kX2 || kGated || kSmall, "two-plane activations: the full down form runs on CTA pairs");
};

struct GemmParams {
    const float* a_scale;   // [K/128][a_ld]
    int a_ld;
    const float* w_scale;   // [G][w_rows/128][K/128]
    const int32_t* count;   // [G]
    const int32_t* start;   // [G]
    void* out;
    float* out_scale;
    int out_ld;
    size_t out_plane;       // two-plane mode, gated: bytes from the hi plane of out to its lo plane
    int G;
    int K;
    int N;                  // output columns per group
    int w_rows;             // weight rows per group (2N gated, N down)
    int* error_word;
    // token-major down form only: [rows] address of each output row (nullptr:
    // the row goes to out), e.g. the token owner's return buffer in another
    // GPU's memory; every epilogue thread fences at system scope at its end
    void* const* row_out = nullptr;
};

struct TileCoord {
    int g, nb, row0, nrows, ntile;
};

__device__ __forceinline__ TileCoord decode_tile(int tile, const int* prefix, const int* chunks,
                                                 const int* starts, const int* counts, int G,
                                                 int n_max) {
    int lo = 0, hi = G - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    TileCoord c;
    c.g = lo;
    int local = tile - prefix[lo];
    int C = chunks[lo];
    c.nb = local / C;
    int chunk = local - c.nb * C;
    c.row0 = starts[lo] + chunk * n_max;
    c.nrows = min(n_max, counts[lo] - chunk * n_max);
    c.ntile = (c.nrows + 15) & ~15;
    return c;
}

// Wait that ignores the abort flag (used only to drain own async work).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kDrainTimeoutNs) break;
    }
}

template <bool kGated, bool kSmall, bool kX2>
__global__ void __launch_bounds__(kNumThreads, 1)
grouped_fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_a64,
                        const __grid_constant__ CUtensorMap tmap_a128,
                        const GemmParams p) {
    using C = GemmCfg<kGated, kSmall, kX2>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

    float* scale_ring = reinterpret_cast<float*>(smem + C::kOffScale);
    int* t_prefix = reinterpret_cast<int*>(smem + C::kOffTables);           // [G+1]
    int* t_chunks = t_prefix + (kMaxGroups + 1);                            // [G]
    int* t_start = t_chunks + kMaxGroups;                                   // [G]
    int* counts_smem = t_start + kMaxGroups;                                // [G]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
    uint64_t* full_bar = bars;
    uint64_t* empty_bar = bars + C::kStages;
    uint64_t* sfull_bar = bars + 2 * C::kStages;
    uint64_t* sempty_bar = sfull_bar + C::kSStages;
    uint64_t* cready_bar = sempty_bar + C::kSStages;
    uint64_t* tfull_bar = cready_bar + C::kSStages;
    uint64_t* tempty_bar = tfull_bar + C::kTBufs;
    uint64_t* epi_bar = tempty_bar + C::kTBufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = p.G;
    const int KB = p.K / kBlockK;

    // ---------------------------------------------------------------- setup
    if (warp == 0 && lane == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int s = 0; s < C::kSStages; ++s) {
            mbar_init(&sfull_bar[s], 1);
            mbar_init(&sempty_bar[s], kNumPromoWarps / C::kPromoGroups);
            mbar_init(&cready_bar[s], 1);
        }
        for (int b = 0; b < C::kTBufs; ++b) {
            mbar_init(&tfull_bar[b], 1);
            mbar_init(&tempty_bar[b], kNumPromoWarps / C::kPromoGroups);
        }
        mbar_init(epi_bar, kNumPromoWarps);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmap_w);
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_a64);
        prefetch_tmap(&tmap_a128);
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    if (warp == 2) {
        // tiles per group: ceil(count / tile tokens) token chunks x (N / 128) row blocks
        const int nbt = p.N / 128;
        int per_lane = (G + 31) / 32;
        int g0 = lane * per_lane;
        int local = 0;
        for (int i = 0; i < per_lane; ++i) {
            int g = g0 + i;
            if (g < G) {
                int cnt = p.count[g];
                int ch = (cnt + C::kTileTok - 1) / C::kTileTok;
                t_chunks[g] = ch;
                t_start[g] = p.start[g];
                counts_smem[g] = cnt;
                local += ch * nbt;
            }
        }
        int incl = local;
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < per_lane; ++i) {
            int g = g0 + i;
            if (g < G) {
                t_prefix[g] = run;
                run += t_chunks[g] * nbt;
            }
        }
        if (lane == 31) t_prefix[G] = incl;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total_tiles = t_prefix[G];

    if (warp < kFirstPromoWarp) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(kRoleRegs));
      if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int s = 0, ss = 0;
            uint32_t phase = 0, sphase = 0;
            uint32_t armed_mask = 0, armed_phase = 0;     // operand ring: last arm per stage and its phase
            uint32_t sarmed_mask = 0, sarmed_phase = 0;   // scale ring
            bool ok = true;
            for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
                TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, C::kTileTok);
                // token rows in as few loads as the box sizes allow (each TMA instruction
                // costs the SM's copy engine far more than its bytes): one box of 32, 64 or
                // 128 rows, or 128-row boxes for down tiles of more than 128 rows
                const int box = tc.ntile <= 32 ? 32 : (tc.ntile <= 64 ? 64 : 128);
                const int b_loads = (tc.ntile + box - 1) / box;
                const CUtensorMap* tmap_b = box == 32 ? &tmap_a : (box == 64 ? &tmap_a64 : &tmap_a128);
                const uint32_t bytes = C::kABytes + b_loads * box * kBlockK * C::kPlanes;
                const int wrow = tc.g * p.w_rows + tc.nb * kTileM;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait_bounded(&empty_bar[s], phase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    uint8_t* st = smem + C::kOffStages + s * C::kStageBytes;
                    mbar_arrive_expect_tx(&full_bar[s], bytes);
                    if (kGated)   // gate and up rows in one load: {K, rows, gate/up}
                        tma_load_3d(&tmap_w, &full_bar[s], st, kb * kBlockK, wrow, 0);
                    else
                        tma_load_2d(&tmap_w, &full_bar[s], st, kb * kBlockK, wrow);
                    for (int r = 0; r < b_loads; ++r) {
                        uint8_t* dst = st + C::kABytes + r * box * kBlockK * C::kPlanes;
                        if constexpr (kX2)   // {K, rows, plane}: [hi | lo][box rows][128 B]
                            tma_load_3d(tmap_b, &full_bar[s], dst, kb * kBlockK, tc.row0 + box * r, 0);
                        else
                            tma_load_2d(tmap_b, &full_bar[s], dst, kb * kBlockK, tc.row0 + box * r);
                    }
                    armed_mask |= 1u << s;
                    armed_phase = (armed_phase & ~(1u << s)) | (phase << s);
                    if (++s == C::kStages) { s = 0; phase ^= 1; }

                    if (!mbar_wait_bounded(&sempty_bar[ss], sphase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    mbar_arrive_expect_tx(&sfull_bar[ss], tc.ntile * 4);
                    bulk_load(scale_ring + ss * C::kScaleFloats + C::kRawSlot * C::kNMax,
                              p.a_scale + (size_t)kb * p.a_ld + tc.row0, tc.ntile * 4, &sfull_bar[ss]);
                    sarmed_mask |= 1u << ss;
                    sarmed_phase = (sarmed_phase & ~(1u << ss)) | (sphase << ss);
                    if (++ss == C::kSStages) { ss = 0; sphase ^= 1; }
                }
            }
            if (!ok) {
                // let every copy this thread issued land before the CTA can exit
                for (int i = 0; i < C::kStages; ++i)
                    if (armed_mask & (1u << i)) mbar_drain(&full_bar[i], (armed_phase >> i) & 1u);
                for (int i = 0; i < C::kSStages; ++i)
                    if (sarmed_mask & (1u << i)) mbar_drain(&sfull_bar[i], (sarmed_phase >> i) & 1u);
            }
        }
      } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int s = 0, b = 0;
            uint32_t phase = 0, tphase = 0;
            bool ok = true;
            bool issued = false;
            for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
                TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, C::kTileTok);
                const uint32_t idesc = idesc_e4m3_f32(kTileM, tc.ntile);
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait_bounded(&full_bar[s], phase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    if (!mbar_wait_bounded(&tempty_bar[b], tphase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + C::kOffStages + s * C::kStageBytes);
                    const uint32_t b_addr = a_addr + C::kABytes;
                    const uint32_t d = tmem_base + b * C::kBufCols;
                    // two-plane mode: the lo plane's products add into the same partial
                    // (one K block = W (hi + lo), one scale), at the box's plane offset
                    const uint32_t plane_bytes =
                        (tc.ntile <= 32 ? 32 : (tc.ntile <= 64 ? 64 : 128)) * kBlockK;
#pragma unroll
                    for (int pl = 0; pl < C::kPlanes; ++pl) {
#pragma unroll
                        for (int k = 0; k < kBlockK / 32; ++k) {
                            const uint64_t bdesc = umma_desc_sw128(b_addr + pl * plane_bytes + k * 32);
                            const uint32_t acc = (k > 0 || pl > 0) ? 1u : 0u;
                            umma_f8(d, umma_desc_sw128(a_addr + k * 32), bdesc, idesc, acc);
                            if (kGated)
                                umma_f8(d + C::kUpOff, umma_desc_sw128(a_addr + kTileM * kBlockK + k * 32), bdesc, idesc,
                                        acc);
                        }
                    }
                    umma_commit(&empty_bar[s]);
                    umma_commit(&tfull_bar[b]);
                    issued = true;
                    if (++s == C::kStages) { s = 0; phase ^= 1; }
                    if (++b == C::kTBufs) { b = 0; tphase ^= 1; }
                }
            }
            if (!ok && issued) {
                // the last commit lands after every MMA this thread issued
                int lb = (b + C::kTBufs - 1) % C::kTBufs;
                uint32_t lph = (b == 0) ? (tphase ^ 1) : tphase;
                mbar_drain(&tfull_bar[lb], lph);
            }
        }
      } else if (warp == 2) {
        // ------------------------------------------------------------ scale folding
        int ss = 0;
        uint32_t sphase = 0;
        bool ok = true;
        const int wsb = p.w_rows / kTileM;
        for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
            TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, C::kTileTok);
            const float* wsg = p.w_scale + ((size_t)tc.g * wsb + tc.nb) * KB;
            const float* wsu = p.w_scale + ((size_t)tc.g * wsb + (p.N / kTileM) + tc.nb) * KB;
            for (int kb = 0; kb < KB; ++kb) {
                const float sg = __ldg(wsg + kb);
                const float su = kGated ? __ldg(wsu + kb) : 0.0f;
                if (!mbar_wait_bounded(&sfull_bar[ss], sphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                float* e = scale_ring + ss * C::kScaleFloats;
                for (int c = lane; c < tc.ntile; c += 32) {
                    const float a = e[C::kRawSlot * C::kNMax + c];
                    e[c] = a * sg;
                    if (kGated) e[C::kNMax + c] = a * su;
                }
                // the entry is overwritten by the async proxy (bulk copy) next
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&cready_bar[ss]);
                if (++ss == C::kSStages) { ss = 0; sphase ^= 1; }
            }
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(kPromoRegs));
        // ------------------------------------------------------------ promotion + epilogue
        const int pw = warp - kFirstPromoWarp;        // 0..15
        const int quarter = warp & 3;                  // TMEM lane quarter this warp may access
        const int colgrp = pw >> 2;                    // 0..3
        const int col0 = kSmall ? 0 : colgrp * C::kColsPerWarp;   // small form: every group covers the tile
        const int row_in_tile = quarter * 32 + lane;   // weight row within the 128-row block
        const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        int ss = 0, b = 0;
        uint32_t sphase = 0, tphase = 0, ephase = 0;
        bool ok = true;
        int kbase = 0;   // small form: K blocks of this CTA's earlier tiles

        // 32-column pieces per K block: gated = gate cols [col0, +32) and the
        // matching up cols (TMEM +128); down = cols [col0, +32) and [col0+32, +32).
        constexpr int kPieces = 2;
        constexpr int kAcc2 = C::kColsPerWarp * C::kNumCombined / 2;   // 32 float2 either way
        // bounded group barrier of the 16 promotion warps (epilogue staging)
        auto group_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(epi_bar);
            const bool r = mbar_wait_bounded(epi_bar, ephase, abort_flag, kWaitTimeoutNs);
            ephase ^= 1;
            return r;
        };

        for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
            TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, C::kTileTok);
            bool live[kPieces];
#pragma unroll
            for (int q = 0; q < kPieces; ++q) live[q] = (kGated ? col0 : col0 + 32 * q) < tc.ntile;
            float2 acc2[kAcc2];
#pragma unroll
            for (int i = 0; i < kAcc2; ++i) acc2[i] = make_float2(0.0f, 0.0f);

            for (int kb = 0; kb < KB; ++kb) {
                if constexpr (kSmall) {
                    // group kb % 4 owns K block kb of every tile (so a row's partial sums
                    // never depend on where its tile ran); ring positions and parities
                    // follow the CTA's K-block count, as the producer and MMA issue them
                    if ((kb & 3) != colgrp) continue;
                    const int g = kbase + kb;
                    ss = g & 7;
                    sphase = (g >> 3) & 1;
                    b = g & 7;
                    tphase = (g >> 3) & 1;
                }
                if (!mbar_wait_bounded(&cready_bar[ss], sphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                if (!mbar_wait_bounded(&tfull_bar[b], tphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                tc_fence_after();
                const float* e = scale_ring + ss * C::kScaleFloats;
                const uint32_t tbuf = lane_addr + b * C::kBufCols;
                // four 16-column chunks c = (piece q, half h); the TMEM load of
                // chunk c+1 is in flight while chunk c is folded
                auto ld_chunk = [&](int c, uint32_t (&pv)[16]) {
                    const int q = c >> 1, h = c & 1;
                    const int tcol = kGated ? (q * C::kUpOff + col0) : (col0 + 32 * q);
                    tmem_ld16(tbuf + tcol + 16 * h, pv);
                };
                auto fold_chunk = [&](int c, const uint32_t (&pv)[16]) {
                    const int q = c >> 1, h = c & 1;
                    const float* cs = (kGated ? (e + q * C::kNMax + col0) : (e + col0 + 32 * q)) + 16 * h;
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        const float4 c4 = *reinterpret_cast<const float4*>(cs + j);
                        float2& a0 = acc2[q * 16 + 8 * h + j / 2];
                        float2& a1 = acc2[q * 16 + 8 * h + j / 2 + 1];
                        a0 = ffma2(make_float2(__uint_as_float(pv[j]), __uint_as_float(pv[j + 1])),
                                   make_float2(c4.x, c4.y), a0);
                        a1 = ffma2(make_float2(__uint_as_float(pv[j + 2]), __uint_as_float(pv[j + 3])),
                                   make_float2(c4.z, c4.w), a1);
                    }
                };
                const int nch = live[1] ? 4 : (live[0] ? 2 : 0);
                if (!kGated) {
                    // down: one 16-register set (two sets spill next to its 64 accumulators)
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (c >= nch) break;
                        uint32_t pv[16];
                        ld_chunk(c, pv);
                        tmem_wait_ld();
                        fold_chunk(c, pv);
                    }
                } else if (nch) {
                    uint32_t pa[16], pb[16];
                    ld_chunk(0, pa);
                    tmem_wait_ld();
                    ld_chunk(1, pb);
                    fold_chunk(0, pa);
                    tmem_wait_ld();
                    if (nch > 2) ld_chunk(2, pa);
                    fold_chunk(1, pb);
                    if (nch > 2) {
                        tmem_wait_ld();
                        ld_chunk(3, pb);
                        fold_chunk(2, pa);
                        tmem_wait_ld();
                        fold_chunk(3, pb);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tempty_bar[b]);
                    mbar_arrive(&sempty_bar[ss]);
                }
                if constexpr (!kSmall) {
                    if (++ss == C::kSStages) { ss = 0; sphase ^= 1; }
                    if (++b == C::kTBufs) { b = 0; tphase ^= 1; }
                }
            }
            if (!ok || *abort_flag) { ok = false; break; }
            if constexpr (kSmall) {
                kbase += KB;
                // the groups' sums, added in group order: red = acc0, += acc1, += acc2; group 3 keeps the total
                float* red = reinterpret_cast<float*>(smem + C::kOffRed);   // [column][128 rows]
                constexpr int kRedPairs = kGated ? 32 : 16;
                // acc2[q * 16 + k] holds piece q's columns 2k, 2k + 1
                auto red_col = [](int i) { return kGated ? (i >> 4) * 32 + 2 * (i & 15) : 2 * i; };
                auto add_red = [&]() {
#pragma unroll
                    for (int i = 0; i < kRedPairs; ++i) {
                        const int c = red_col(i);
                        acc2[i].x += red[c * 128 + row_in_tile];
                        acc2[i].y += red[(c + 1) * 128 + row_in_tile];
                    }
                };
                auto store_red = [&]() {
#pragma unroll
                    for (int i = 0; i < kRedPairs; ++i) {
                        const int c = red_col(i);
                        red[c * 128 + row_in_tile] = acc2[i].x;
                        red[(c + 1) * 128 + row_in_tile] = acc2[i].y;
                    }
                };
                if (colgrp == 0) store_red();
                if (!group_sync()) { ok = false; break; }
                if (colgrp == 1) { add_red(); store_red(); }
                if (!group_sync()) { ok = false; break; }
                if (colgrp == 2) { add_red(); store_red(); }
                if (!group_sync()) { ok = false; break; }
                if (colgrp == 3) add_red();
                if (!ok) break;
            }

            // ---------------------------------------------------------- epilogue
            // acc2[i] holds columns 2i, 2i+1 of this warp's 64 accumulators:
            // gated: [0, 32) gate cols col0.., [32, 64) the matching up cols;
            // down: cols col0 .. col0+63.
            if (kGated) {
                float* stage = reinterpret_cast<float*>(smem + C::kOffOut);   // [N_MAX][128] fp32
#pragma unroll
                for (int c = 0; c < C::kColsPerWarp; ++c) {
                    const float g = (c & 1) ? acc2[c >> 1].y : acc2[c >> 1].x;
                    const float u = (c & 1) ? acc2[16 + (c >> 1)].y : acc2[16 + (c >> 1)].x;
                    const float h = (g / (1.0f + expf(-g))) * u;
                    // the small form's stage holds only the tile's columns, written by group 3 (the total)
                    if (!kSmall || (colgrp == 3 && col0 + c < tc.ntile)) stage[(col0 + c) * 128 + row_in_tile] = h;
                }
                if (!group_sync()) { ok = false; break; }
                uint8_t* outq = reinterpret_cast<uint8_t*>(p.out);
                for (int c = pw; c < tc.ntile; c += kNumPromoWarps) {
                    const size_t row = static_cast<size_t>(tc.row0 + c);
                    uint32_t packed = 0, packed_lo = 0;
                    float scale = 0.0f;
                    if (c < tc.nrows) {
                        const float4 v = *reinterpret_cast<const float4*>(stage + c * 128 + lane * 4);
                        float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                        if (amax > 0.0f) {
                            const float inv = 448.0f / amax;
                            if constexpr (kX2) {
                                const uint32_t s0 = cvt_e4m3x2_split(__fmul_rn(v.x, inv), __fmul_rn(v.y, inv));
                                const uint32_t s1 = cvt_e4m3x2_split(__fmul_rn(v.z, inv), __fmul_rn(v.w, inv));
                                packed = (s0 & 0xFFFFu) | (s1 << 16);
                                packed_lo = (s0 >> 16) | (s1 & 0xFFFF0000u);
                            } else {
                                const uint32_t lo = cvt_e4m3x2(v.x * inv, v.y * inv);
                                const uint32_t hi = cvt_e4m3x2(v.z * inv, v.w * inv);
                                packed = lo | (hi << 16);
                            }
                            scale = amax / 448.0f;
                        }
                    }
                    *reinterpret_cast<uint32_t*>(outq + row * p.N + tc.nb * 128 + lane * 4) = packed;
                    if constexpr (kX2)
                        *reinterpret_cast<uint32_t*>(outq + p.out_plane + row * p.N + tc.nb * 128 + lane * 4) = packed_lo;
                    if (lane == 0) p.out_scale[(size_t)tc.nb * p.out_ld + row] = scale;
                }
                if (!group_sync()) { ok = false; break; }
            } else {
                __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem + C::kOffOut);  // [N_MAX][128]
#pragma unroll
                for (int c = 0; c < C::kColsPerWarp; ++c) {
                    const float v = (c & 1) ? acc2[c >> 1].y : acc2[c >> 1].x;
                    if (!kSmall || (colgrp == 3 && col0 + c < tc.ntile))
                        stage[(col0 + c) * 128 + row_in_tile] = __float2bfloat16_rn(v);
                }
                if (!group_sync()) { ok = false; break; }
                __nv_bfloat16* outy = reinterpret_cast<__nv_bfloat16*>(p.out);
                for (int c = pw; c < tc.nrows; c += kNumPromoWarps) {
                    const uint2 v = *reinterpret_cast<const uint2*>(stage + c * 128 + lane * 4);
                    *reinterpret_cast<uint2*>(outy + static_cast<size_t>(tc.row0 + c) * p.N + tc.nb * 128 + lane * 4) = v;
                }
                if (!group_sync()) { ok = false; break; }
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
    if (threadIdx.x == 0 && *abort_flag && p.error_word) atomicExch(p.error_word, 1);
}

// ------------------------------------------------------------------ token-major full form
// The default full form.  The roles of the one-SM form are kept, but the UMMA
// operands are not swapped: M = 128 token rows of one expert (TMEM lanes) and
// N = 256 weight rows -- the tile's 128 gate rows and their 128 up rows
// (gated), or two 128-row blocks of W_down (down) -- so one tcgen05.mma is
// 128 x 256 x 32.  An N = 128 or N = 64 instruction costs the tensor core about
// as long as an N = 256 one (a fixed per-instruction floor, measured: 64 % and
// 32 % of the fp8 peak against 96 % for N = 256 at M = 128), so the gated K
// block issues 4 instructions per plane instead of 8, and the padding of a
// ragged token chunk to 128 rows costs less than the instruction count saved.
// A thread of the promotion warps owns one token row, so its per-K-block scale
// is a scalar (token scale x weight-block scale, folded once per CTA by the
// scale warp) and the fused epilogue stores each thread's 32 (gated, e4m3) or
// 64 (down, bf16) output columns straight from registers: the 1x128 amax of a
// token is the max over the four column-group warps of its lane quarter,
// exchanged through 2 KB of shared memory.  Without the transposing stage the
// operand ring holds four 48 KB stages (one plane) or three 64 KB stages (two
// planes).  The products, their K order and every rounding step are those of
// the one-SM form, so both give bit-identical outputs.
template <bool kGated, bool kX2>
struct TmCfg {
    static constexpr int kPlanes = kX2 ? 2 : 1;
    static constexpr int kTok = 128;                          // token rows per tile (UMMA M)
    static constexpr int kWRows = 256;                        // weight rows per tile (UMMA N)
    static constexpr int kWBytes = kWRows * kBlockK;          // 32 KB
    static constexpr int kABytes = kPlanes * kTok * kBlockK;  // 16 / 32 KB: [plane][rows][128 B]
    static constexpr int kStageBytes = kWBytes + kABytes;
    static constexpr int kStages = kX2 ? 3 : 4;
    static constexpr int kSStages = 8;
    static constexpr int kScaleFloats = 2 * kTok;             // folded [first weight block][second] per token
    static constexpr int kTBufs = 2;                          // 2 x 256 TMEM columns
    static constexpr int kBufCols = 256;
    static constexpr int kOffStages = 0;
    static constexpr int kOffScale = kOffStages + kStages * kStageBytes;
    static constexpr int kOffAmax = kOffScale + kSStages * kScaleFloats * 4;   // [tile parity][4 groups][128] fp32
    static constexpr int kOffTables = kOffAmax + 2 * 4 * kTok * 4;
    static constexpr int kOffBars = kOffTables + (4 * kMaxGroups + 2) * 4;
    static constexpr int kNumBars = 2 * kStages + 3 * kSStages + 2 * kTBufs + 1;
    static constexpr int kOffMisc = kOffBars + kNumBars * 8;
    static constexpr int kSmemBytes = kOffMisc + 64 + 1024;
    static_assert(kOffBars % 8 == 0, "mbarrier alignment");
    static_assert(kStageBytes % 1024 == 0 && kWBytes % 1024 == 0, "128-byte-swizzled tiles on 1024-byte boundaries");
    static_assert(kTBufs * kBufCols <= kTmemCols, "TMEM partial buffers");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <bool kGated, bool kX2>
__global__ void __launch_bounds__(kNumThreads, 1)
grouped_fp8_gemm_tm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                           const __grid_constant__ CUtensorMap tmap_a,
                           const __grid_constant__ CUtensorMap tmap_a64,
                           const __grid_constant__ CUtensorMap tmap_a128,
                           const GemmParams p) {
    using C = TmCfg<kGated, kX2>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

    float* scale_ring = reinterpret_cast<float*>(smem + C::kOffScale);
    float* amax_x = reinterpret_cast<float*>(smem + C::kOffAmax);
    int* t_prefix = reinterpret_cast<int*>(smem + C::kOffTables);
    int* t_chunks = t_prefix + (kMaxGroups + 1);
    int* t_start = t_chunks + kMaxGroups;
    int* counts_smem = t_start + kMaxGroups;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
    uint64_t* full_bar = bars;
    uint64_t* empty_bar = bars + C::kStages;
    uint64_t* sfull_bar = bars + 2 * C::kStages;
    uint64_t* sempty_bar = sfull_bar + C::kSStages;
    uint64_t* cready_bar = sempty_bar + C::kSStages;
    uint64_t* tfull_bar = cready_bar + C::kSStages;
    uint64_t* tempty_bar = tfull_bar + C::kTBufs;
    uint64_t* epi_bar = tempty_bar + C::kTBufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kOffMisc + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = p.G;
    const int KB = p.K / kBlockK;
    const int nbt = kGated ? p.N / kTileM : p.N / C::kWRows;   // output column blocks per group

    // ---------------------------------------------------------------- setup
    if (warp == 0 && lane == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int s = 0; s < C::kSStages; ++s) {
            mbar_init(&sfull_bar[s], 1);
            mbar_init(&sempty_bar[s], kNumPromoWarps);
            mbar_init(&cready_bar[s], 1);
        }
        for (int b = 0; b < C::kTBufs; ++b) {
            mbar_init(&tfull_bar[b], 1);
            mbar_init(&tempty_bar[b], kNumPromoWarps);
        }
        mbar_init(epi_bar, kNumPromoWarps);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmap_w);
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_a64);
        prefetch_tmap(&tmap_a128);
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    if (warp == 2) {
        // tiles per group: ceil(count / 128) token chunks x nbt column blocks
        int per_lane = (G + 31) / 32;
        int g0 = lane * per_lane;
        int local = 0;
        for (int i = 0; i < per_lane; ++i) {
            int g = g0 + i;
            if (g < G) {
                int cnt = p.count[g];
                int ch = (cnt + C::kTok - 1) / C::kTok;
                t_chunks[g] = ch;
                t_start[g] = p.start[g];
                counts_smem[g] = cnt;
                local += ch * nbt;
            }
        }
        int incl = local;
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < per_lane; ++i) {
            int g = g0 + i;
            if (g < G) {
                t_prefix[g] = run;
                run += t_chunks[g] * nbt;
            }
        }
        if (lane == 31) t_prefix[G] = incl;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total_tiles = t_prefix[G];

    if (warp < kFirstPromoWarp) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(kRoleRegs));
      if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int s = 0, ss = 0;
            uint32_t phase = 0, sphase = 0;
            uint32_t armed_mask = 0, armed_phase = 0;
            uint32_t sarmed_mask = 0, sarmed_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
                TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, C::kTok);
                // one token box of 32, 64 or 128 rows (the MMA reads 128 rows; rows past
                // the chunk hold stale bytes whose output rows are never stored)
                const int box = tc.ntile <= 32 ? 32 : (tc.ntile <= 64 ? 64 : 128);
                const CUtensorMap* tmap_b = box == 32 ? &tmap_a : (box == 64 ? &tmap_a64 : &tmap_a128);
                const uint32_t bytes = C::kWBytes + box * kBlockK * C::kPlanes;
                const int wrow = tc.g * p.w_rows + tc.nb * (kGated ? kTileM : C::kWRows);
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait_bounded(&empty_bar[s], phase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    uint8_t* st = smem + C::kOffStages + s * C::kStageBytes;
                    mbar_arrive_expect_tx(&full_bar[s], bytes);
                    if (kGated)   // {K, rows, gate/up}: [128 gate rows][128 up rows]
                        tma_load_3d(&tmap_w, &full_bar[s], st, kb * kBlockK, wrow, 0);
                    else          // 256 rows
                        tma_load_2d(&tmap_w, &full_bar[s], st, kb * kBlockK, wrow);
                    if constexpr (kX2)   // {K, rows, plane}: [hi | lo][box rows][128 B]
                        tma_load_3d(tmap_b, &full_bar[s], st + C::kWBytes, kb * kBlockK, tc.row0, 0);
                    else
                        tma_load_2d(tmap_b, &full_bar[s], st + C::kWBytes, kb * kBlockK, tc.row0);
                    armed_mask |= 1u << s;
                    armed_phase = (armed_phase & ~(1u << s)) | (phase << s);
                    if (++s == C::kStages) { s = 0; phase ^= 1; }

                    if (!mbar_wait_bounded(&sempty_bar[ss], sphase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    mbar_arrive_expect_tx(&sfull_bar[ss], tc.ntile * 4);
                    bulk_load(scale_ring + ss * C::kScaleFloats + C::kTok,
                              p.a_scale + (size_t)kb * p.a_ld + tc.row0, tc.ntile * 4, &sfull_bar[ss]);
                    sarmed_mask |= 1u << ss;
                    sarmed_phase = (sarmed_phase & ~(1u << ss)) | (sphase << ss);
                    if (++ss == C::kSStages) { ss = 0; sphase ^= 1; }
                }
            }
            if (!ok) {
                for (int i = 0; i < C::kStages; ++i)
                    if (armed_mask & (1u << i)) mbar_drain(&full_bar[i], (armed_phase >> i) & 1u);
                for (int i = 0; i < C::kSStages; ++i)
                    if (sarmed_mask & (1u << i)) mbar_drain(&sfull_bar[i], (sarmed_phase >> i) & 1u);
            }
        }
      } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int s = 0, b = 0;
            uint32_t phase = 0, tphase = 0;
            bool ok = true;
            bool issued = false;
            const uint32_t idesc = idesc_e4m3_f32(C::kTok, C::kWRows);
            for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
                TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, C::kTok);
                const uint32_t plane_bytes = (tc.ntile <= 32 ? 32 : (tc.ntile <= 64 ? 64 : 128)) * kBlockK;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait_bounded(&full_bar[s], phase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    if (!mbar_wait_bounded(&tempty_bar[b], tphase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t w_addr = smem_u32(smem + C::kOffStages + s * C::kStageBytes);
                    const uint32_t a_addr = w_addr + C::kWBytes;
                    const uint32_t d = tmem_base + b * C::kBufCols;
#pragma unroll
                    for (int pl = 0; pl < C::kPlanes; ++pl) {
#pragma unroll
                        for (int k = 0; k < kBlockK / 32; ++k)
                            umma_f8(d, umma_desc_sw128(a_addr + pl * plane_bytes + k * 32),
                                    umma_desc_sw128(w_addr + k * 32), idesc, (k > 0 || pl > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty_bar[s]);
                    umma_commit(&tfull_bar[b]);
                    issued = true;
                    if (++s == C::kStages) { s = 0; phase ^= 1; }
                    if (++b == C::kTBufs) { b = 0; tphase ^= 1; }
                }
            }
            if (!ok && issued) {
                int lb = (b + C::kTBufs - 1) % C::kTBufs;
                uint32_t lph = (b == 0) ? (tphase ^ 1) : tphase;
                mbar_drain(&tfull_bar[lb], lph);
            }
        }
      } else if (warp == 2) {
        // ------------------------------------------------------------ scale folding
        // entry [0, 128): token scale x the scale of the tile's first weight block
        // (gate / W_down rows 256 nb..), [128, 256): x the second (up / rows 256 nb + 128..);
        // the bulk copy lands the raw token scales in the second half
        int ss = 0;
        uint32_t sphase = 0;
        bool ok = true;
        const int wsb = p.w_rows / kTileM;
        for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
            TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, C::kTok);
            const int blk0 = kGated ? tc.nb : 2 * tc.nb;
            const int blk1 = kGated ? p.N / kTileM + tc.nb : 2 * tc.nb + 1;
            const float* ws0 = p.w_scale + ((size_t)tc.g * wsb + blk0) * KB;
            const float* ws1 = p.w_scale + ((size_t)tc.g * wsb + blk1) * KB;
            for (int kb = 0; kb < KB; ++kb) {
                const float s0 = __ldg(ws0 + kb);
                const float s1 = __ldg(ws1 + kb);
                if (!mbar_wait_bounded(&sfull_bar[ss], sphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                float* e = scale_ring + ss * C::kScaleFloats;
                for (int c = lane; c < tc.ntile; c += 32) {
                    const float a = e[C::kTok + c];
                    e[c] = a * s0;
                    e[C::kTok + c] = a * s1;
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&cready_bar[ss]);
                if (++ss == C::kSStages) { ss = 0; sphase ^= 1; }
            }
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(kPromoRegs));
        // ------------------------------------------------------------ promotion + epilogue
        const int pw = warp - kFirstPromoWarp;        // 0..15
        const int quarter = warp & 3;                  // TMEM lane quarter this warp may access
        const int colgrp = pw >> 2;                    // 0..3
        const int r = quarter * 32 + lane;             // token row within the tile
        const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        int ss = 0, b = 0;
        uint32_t sphase = 0, tphase = 0, ephase = 0;
        bool ok = true;
        int parity = 0;
        auto group_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(epi_bar);
            const bool res = mbar_wait_bounded(epi_bar, ephase, abort_flag, kWaitTimeoutNs);
            ephase ^= 1;
            return res;
        };
        // TMEM column of 16-column chunk c (0..3) and the acc2 pairs it feeds (8c..8c+7):
        // gated: chunks 0, 1 = gate columns 32 colgrp + [0, 32), 2, 3 = the up columns
        // (TMEM + 128); down: columns 64 colgrp + 16 c
        auto tcol = [&](int c) { return kGated ? (c >> 1) * 128 + colgrp * 32 + (c & 1) * 16 : colgrp * 64 + c * 16; };

        for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
            TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, C::kTok);
            float2 acc2[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) acc2[i] = make_float2(0.0f, 0.0f);

            for (int kb = 0; kb < KB; ++kb) {
                if (!mbar_wait_bounded(&cready_bar[ss], sphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                if (!mbar_wait_bounded(&tfull_bar[b], tphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                tc_fence_after();
                const float* e = scale_ring + ss * C::kScaleFloats;
                const float c_lo = kGated ? e[r] : e[(colgrp >> 1) * C::kTok + r];
                const float c_hi = kGated ? e[C::kTok + r] : c_lo;
                const uint32_t tbuf = lane_addr + b * C::kBufCols;
                auto fold = [&](int c, const uint32_t (&pv)[16]) {
                    const float cs = (kGated && c >= 2) ? c_hi : c_lo;
                    const float2 c2 = make_float2(cs, cs);
#pragma unroll
                    for (int j = 0; j < 16; j += 2) {
                        float2& a = acc2[8 * c + j / 2];
                        a = ffma2(make_float2(__uint_as_float(pv[j]), __uint_as_float(pv[j + 1])), c2, a);
                    }
                };
                uint32_t pa[16], pb[16];
                tmem_ld16(tbuf + tcol(0), pa);
                tmem_wait_ld();
                tmem_ld16(tbuf + tcol(1), pb);
                fold(0, pa);
                tmem_wait_ld();
                tmem_ld16(tbuf + tcol(2), pa);
                fold(1, pb);
                tmem_wait_ld();
                tmem_ld16(tbuf + tcol(3), pb);
                fold(2, pa);
                tmem_wait_ld();
                fold(3, pb);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tempty_bar[b]);
                    mbar_arrive(&sempty_bar[ss]);
                }
                if (++ss == C::kSStages) { ss = 0; sphase ^= 1; }
                if (++b == C::kTBufs) { b = 0; tphase ^= 1; }
            }
            if (!ok || *abort_flag) { ok = false; break; }

            // ---------------------------------------------------------- epilogue
            // gated: rows [nrows, ntile) of the chunk are stored as zeros (the down
            // projection reads whole 16-row groups); down: rows < nrows only
            const bool row_live = r < tc.nrows;
            const size_t row = static_cast<size_t>(tc.row0 + r);
            if (kGated) {
                // acc2[0..15]: gate columns 32 colgrp + 2i, +1; acc2[16..31]: the up columns
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float g0 = acc2[i].x, g1 = acc2[i].y;
                    const float u0 = acc2[16 + i].x, u1 = acc2[16 + i].y;
                    const float h0 = (g0 / (1.0f + expf(-g0))) * u0;
                    const float h1 = (g1 / (1.0f + expf(-g1))) * u1;
                    acc2[i] = make_float2(h0, h1);
                    amax = fmaxf(amax, fmaxf(fabsf(h0), fabsf(h1)));
                }
                float* ax = amax_x + parity * 4 * C::kTok;
                ax[colgrp * C::kTok + r] = amax;
                if (!group_sync()) { ok = false; break; }
                amax = fmaxf(fmaxf(ax[r], ax[C::kTok + r]), fmaxf(ax[2 * C::kTok + r], ax[3 * C::kTok + r]));
                parity ^= 1;
                if (r < tc.ntile) {
                    uint32_t hi[8], lo[8];
#pragma unroll
                    for (int w = 0; w < 8; ++w) { hi[w] = 0u; lo[w] = 0u; }
                    float scale = 0.0f;
                    if (row_live && amax > 0.0f) {
                        const float inv = 448.0f / amax;
#pragma unroll
                        for (int w = 0; w < 8; ++w) {
                            const float2 v0 = acc2[2 * w], v1 = acc2[2 * w + 1];
                            if constexpr (kX2) {
                                const uint32_t s0 = cvt_e4m3x2_split(__fmul_rn(v0.x, inv), __fmul_rn(v0.y, inv));
                                const uint32_t s1 = cvt_e4m3x2_split(__fmul_rn(v1.x, inv), __fmul_rn(v1.y, inv));
                                hi[w] = (s0 & 0xFFFFu) | (s1 << 16);
                                lo[w] = (s0 >> 16) | (s1 & 0xFFFF0000u);
                            } else {
                                const uint32_t q0 = cvt_e4m3x2(v0.x * inv, v0.y * inv);
                                const uint32_t q1 = cvt_e4m3x2(v1.x * inv, v1.y * inv);
                                hi[w] = q0 | (q1 << 16);
                            }
                        }
                        scale = amax / 448.0f;
                    }
                    uint8_t* outq = reinterpret_cast<uint8_t*>(p.out) + row * p.N + tc.nb * 128 + colgrp * 32;
                    uint4* o = reinterpret_cast<uint4*>(outq);
                    o[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    o[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                    if constexpr (kX2) {
                        uint4* ol = reinterpret_cast<uint4*>(outq + p.out_plane);
                        ol[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        ol[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                    }
                    if (colgrp == 0) p.out_scale[(size_t)tc.nb * p.out_ld + row] = scale;
                }
            } else if (row_live) {
                // acc2[i]: columns 64 colgrp + 2i, +1 of the tile's 256
                uint32_t w[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(acc2[i].x, acc2[i].y);
                    w[i] = *reinterpret_cast<const uint32_t*>(&h2);
                }
                __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.out) + row * p.N;
                if (p.row_out) {
                    void* dst = p.row_out[row];
                    if (dst) orow = static_cast<__nv_bfloat16*>(dst);
                }
                uint4* o = reinterpret_cast<uint4*>(orow + tc.nb * C::kWRows + colgrp * 64);
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    // rows stored to other GPUs are visible system-wide before the grid ends,
    // so a flag raised by the next launch on the stream orders them
    if (!kGated && p.row_out) __threadfence_system();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
    if (threadIdx.x == 0 && *abort_flag && p.error_word) atomicExch(p.error_word, 1);
}

// ------------------------------------------------------------------ full form on CTA pairs
// The full form (tiles of up to 128 tokens) runs on CTA pairs: a cluster of two
// CTAs on two SMs issues tcgen05.mma with cta_group::2, M = 256 weight rows x
// N <= 128 tokens per instruction, from the even CTA.  Each CTA stages its own
// 128 weight rows and half of the tile's token rows (the MMA reads both CTAs'
// shared memory) and receives its 128 rows of the product in its own TMEM.
//   gated: the pair covers output columns [128 nb, 128 nb + 128) of h; CTA r
//          holds gate rows 128 nb + 64 r + [0, 64) in TMEM lanes 0-63 and the
//          matching up rows in lanes 64-127, so SwiGLU stays inside the CTA.
//          The 1x128 requantisation needs the token's amax over both CTAs'
//          64 columns: the two CTAs swap their partial amax through
//          distributed shared memory once per tile.
//   down:  CTA r holds output rows 256 nb + 128 r + [0, 128).
// Per K block each CTA promotes 128 lanes x N columns (16 warps x one 32-column
// TMEM load), half of what one SM promotes in the one-SM form for the same
// MMA work, and its operand stage is 24 KB instead of 48 KB, so the ring is
// six stages deep.  Hand-offs: the even CTA's producer arms the stage's full
// barrier with both CTAs' bytes and both CTAs' TMA loads complete on it; the
// MMA commits release the operand stage and publish the TMEM buffer in both
// CTAs (multicast commit); both CTAs' promotion warps release a TMEM buffer
// on the even CTA's barrier.  Every wait is bounded as in the one-SM form.
constexpr int kPairTok = 128;                               // tokens per tile (UMMA N)
constexpr int kPairKbPerStage = 2;                          // K blocks per TMA load (one instruction each)
constexpr int kPairSStages = 4;
constexpr int kPairTBufs = 4;                               // 4 x 128 TMEM columns
constexpr int kPairABytes = kTileM * kBlockK;               // this CTA's 128 weight rows, one K block
constexpr int kPairBRows = kPairTok / 2;                    // this CTA's half of the tokens
constexpr int kPairBBytes = kPairBRows * kBlockK;
constexpr int kPairEpiBytes = kPairTok * 128 * 2;           // 32 KB: gated [128 tok][64] fp32, down [128][128] bf16
// scale ring entry: raw token scales [kb][128] (TMA), then the folded [kb][gate, up][128]
constexpr int kPairScaleRaw = kPairKbPerStage * kPairTok;
constexpr int kPairScaleFloats = kPairScaleRaw + kPairKbPerStage * 2 * kPairTok;
// Operand ring and shared-memory carve-up; two-plane activations (hi + lo
// residual) double the token part of a stage: [plane][kb][64 rows][128 B].
template <bool kX2>
struct PairCfg {
    static constexpr int kPlanes = kX2 ? 2 : 1;
    static constexpr int kStages = kX2 ? 2 : 3;
    static constexpr int kStageABytes = kPairKbPerStage * kPairABytes;   // [kb][128 rows][128 B]
    static constexpr int kStageBytes = kStageABytes + kPlanes * kPairKbPerStage * kPairBBytes;   // 48 / 64 KB
    static constexpr int kOffStages = 0;
    static constexpr int kOffEpi = kOffStages + kStages * kStageBytes;
    static constexpr int kOffScale = kOffEpi + kPairEpiBytes;
    static constexpr int kOffAmax = kOffScale + kPairSStages * kPairScaleFloats * 4;   // own[128], peer[2][128]
    static constexpr int kOffTables = kOffAmax + 3 * kPairTok * 4;
    static constexpr int kOffBars = kOffTables + (4 * kMaxGroups + 2) * 4;
    static constexpr int kNumBars = 2 * kStages + 3 * kPairSStages + 2 * kPairTBufs + 1 + 2;
    static constexpr int kOffMisc = kOffBars + kNumBars * 8;
    static constexpr int kSmemBytes = kOffMisc + 64 + 1024;
    static_assert(kOffBars % 8 == 0, "mbarrier alignment");
    static_assert(kStageBytes % 1024 == 0 && kStageABytes % 1024 == 0, "swizzled tiles on 1024-byte boundaries");
    static_assert((kPairScaleFloats * 4) % 128 == 0, "scale entries 128-byte aligned");
    static_assert(kPairTBufs * kPairTok <= kTmemCols, "TMEM buffers");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct PairParams {
    GemmParams g;
    int I;     // gated: intermediate size (up rows start at I within a group)
};

__device__ __forceinline__ void tma_load_3d_pair(const void* tmap, uint32_t bar_cluster, void* dst,
                                                 int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];"
        :: "r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void tma_prefetch_3d(const void* tmap, int32_t x, int32_t y, int32_t z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global [%0, {%1, %2, %3}];"
                 :: "l"(tmap), "r"(x), "r"(y), "r"(z) : "memory");
}
__device__ __forceinline__ void tma_prefetch_4d(const void* tmap, int32_t x, int32_t y, int32_t z, int32_t w) {
    asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global [%0, {%1, %2, %3, %4}];"
                 :: "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
constexpr int kPairPrefetch = 4;     // stages of weights fetched into L2 ahead of the ring

__device__ __forceinline__ void tma_load_4d_pair(const void* tmap, uint32_t bar_cluster, void* dst,
                                                 int32_t x, int32_t y, int32_t z, int32_t w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];"
        :: "r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar_cluster) : "memory");
}

template <bool kGated, bool kX2>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kNumThreads, 1)
grouped_fp8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                             const __grid_constant__ CUtensorMap tmap_s, const PairParams pp) {
    using P = PairCfg<kX2>;
    const GemmParams& p = pp.g;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

    float* scale_ring = reinterpret_cast<float*>(smem + P::kOffScale);
    float* amax_own = reinterpret_cast<float*>(smem + P::kOffAmax);
    float* amax_peer = amax_own + kPairTok;                                  // [2][128], written by the peer
    int* t_prefix = reinterpret_cast<int*>(smem + P::kOffTables);
    int* t_chunks = t_prefix + (kMaxGroups + 1);
    int* t_start = t_chunks + kMaxGroups;
    int* counts_smem = t_start + kMaxGroups;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P::kOffBars);
    uint64_t* full_bar = bars;                              // used in the even CTA
    uint64_t* empty_bar = full_bar + P::kStages;
    uint64_t* sfull_bar = empty_bar + P::kStages;
    uint64_t* sempty_bar = sfull_bar + kPairSStages;
    uint64_t* cready_bar = sempty_bar + kPairSStages;
    uint64_t* tfull_bar = cready_bar + kPairSStages;
    uint64_t* tempty_bar = tfull_bar + kPairTBufs;          // used in the even CTA
    uint64_t* epi_bar = tempty_bar + kPairTBufs;
    uint64_t* xbar = epi_bar + 1;                           // [2]: the peer's amax has landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + P::kOffMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + P::kOffMisc + 8);

    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank();             // 0: issues the MMAs
    const uint32_t peer = rank ^ 1u;
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int G = p.G;
    const int KB = p.K / kBlockK;
    const int KS = KB / kPairKbPerStage;                   // stages per tile

    // ---------------------------------------------------------------- setup
    if (warp == 0 && lane == 0) {
        for (int s = 0; s < P::kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int s = 0; s < kPairSStages; ++s) {
            mbar_init(&sfull_bar[s], 1);
            mbar_init(&sempty_bar[s], kNumPromoWarps);
            mbar_init(&cready_bar[s], 1);
        }
        for (int b = 0; b < kPairTBufs; ++b) {
            mbar_init(&tfull_bar[b], 1);
            mbar_init(&tempty_bar[b], 2 * kNumPromoWarps);
        }
        mbar_init(epi_bar, kNumPromoWarps);
        mbar_init(&xbar[0], kNumPromoWarps);
        mbar_init(&xbar[1], kNumPromoWarps);
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmap_w);
        prefetch_tmap(&tmap_a);
        prefetch_tmap(&tmap_s);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
    if (warp == 2) {
        const int nbt = kGated ? p.N / 128 : p.N / 256;     // pair row blocks per group
        int per_lane = (G + 31) / 32;
        int g0 = lane * per_lane;
        int local = 0;
        for (int i = 0; i < per_lane; ++i) {
            int g = g0 + i;
            if (g < G) {
                int cnt = p.count[g];
                int ch = (cnt + kPairTok - 1) / kPairTok;
                t_chunks[g] = ch;
                t_start[g] = p.start[g];
                counts_smem[g] = cnt;
                local += ch * nbt;
            }
        }
        int incl = local;
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < per_lane; ++i) {
            int g = g0 + i;
            if (g < G) {
                t_prefix[g] = run;
                run += t_chunks[g] * nbt;
            }
        }
        if (lane == 31) t_prefix[G] = incl;
    }
    tc_fence_before();
    __syncthreads();
    cluster.sync();          // both CTAs' barriers are initialised before any cross-CTA traffic
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int total_tiles = t_prefix[G];
    const uint16_t both = 0x3;

    if (warp < kFirstPromoWarp) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(kRoleRegs));
      if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        // per stage (two K blocks): one load of this CTA's weight rows, one of its
        // token rows, one of the tile's raw token scales
        if (lane == 0) {
            int s = 0, ss = 0;
            uint32_t phase = 0, sphase = 0;
            uint32_t sarmed_mask = 0, sarmed_phase = 0;
            uint32_t full_leader[P::kStages];
            for (int i = 0; i < P::kStages; ++i) full_leader[i] = mapa_u32(smem_u32(&full_bar[i]), 0);
            bool ok = true;
            bool issued = false;
            // weights arrive from HBM: fetch them into L2 kPairPrefetch stages ahead of
            // the ring (no shared memory), so the ring's loads mostly hit L2
            int pf_tile = cid, pf_ks = 0;
            auto pf_row = [&](int tile) {
                TileCoord t2 = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, kPairTok);
                return kGated ? t2.g * p.w_rows + t2.nb * 128 + 64 * static_cast<int>(rank)
                              : t2.g * p.w_rows + t2.nb * 256 + 128 * static_cast<int>(rank);
            };
            int pf_wrow = pf_tile < total_tiles ? pf_row(pf_tile) : 0;
            auto prefetch_next = [&]() {
                if (pf_tile >= total_tiles) return;
                if (kGated) tma_prefetch_4d(&tmap_w, 0, pf_wrow, 0, pf_ks * kPairKbPerStage);
                else tma_prefetch_3d(&tmap_w, 0, pf_wrow, pf_ks * kPairKbPerStage);
                if (++pf_ks == KS) {
                    pf_ks = 0;
                    pf_tile += ncl;
                    if (pf_tile < total_tiles) pf_wrow = pf_row(pf_tile);
                }
            };
            for (int i = 0; i < kPairPrefetch; ++i) prefetch_next();
            for (int tile = cid; tile < total_tiles && ok; tile += ncl) {
                TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, kPairTok);
                const int half = tc.ntile >> 1;
                const int wrow = kGated ? tc.g * p.w_rows + tc.nb * 128 + 64 * static_cast<int>(rank)
                                        : tc.g * p.w_rows + tc.nb * 256 + 128 * static_cast<int>(rank);
                for (int ks = 0; ks < KS; ++ks) {
                    const int kb0 = ks * kPairKbPerStage;
                    prefetch_next();
                    if (!mbar_wait_bounded(&empty_bar[s], phase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    uint8_t* st = smem + P::kOffStages + s * P::kStageBytes;
                    if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], 2 * P::kStageBytes);
                    if (kGated)   // {128 B, 64 rows, gate/up, 2 K blocks}
                        tma_load_4d_pair(&tmap_w, full_leader[s], st, 0, wrow, 0, kb0);
                    else          // {128 B, 128 rows, 2 K blocks}
                        tma_load_3d_pair(&tmap_w, full_leader[s], st, 0, wrow, kb0);
                    if constexpr (kX2)   // {128 B, 64 rows, 2 K blocks, hi/lo}
                        tma_load_4d_pair(&tmap_a, full_leader[s], st + P::kStageABytes, 0,
                                         tc.row0 + static_cast<int>(rank) * half, kb0, 0);
                    else                 // {128 B, 64 rows, 2 K blocks}
                        tma_load_3d_pair(&tmap_a, full_leader[s], st + P::kStageABytes, 0,
                                         tc.row0 + static_cast<int>(rank) * half, kb0);
                    issued = true;
                    if (++s == P::kStages) { s = 0; phase ^= 1; }

                    if (!mbar_wait_bounded(&sempty_bar[ss], sphase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    mbar_arrive_expect_tx(&sfull_bar[ss], kPairScaleRaw * 4);
                    tma_load_2d(&tmap_s, &sfull_bar[ss], scale_ring + ss * kPairScaleFloats, tc.row0, kb0);
                    sarmed_mask |= 1u << ss;
                    sarmed_phase = (sarmed_phase & ~(1u << ss)) | (sphase << ss);
                    if (++ss == kPairSStages) { ss = 0; sphase ^= 1; }
                }
            }
            if (!ok) {
                // this CTA's operand copies complete on the even CTA's barrier: give
                // them time to land before the CTA can leave (they take microseconds)
                if (issued) {
                    const uint64_t t0 = globaltimer_ns();
                    while (globaltimer_ns() - t0 < 20000000ull) { }
                }
                for (int i = 0; i < kPairSStages; ++i)
                    if (sarmed_mask & (1u << i)) mbar_drain(&sfull_bar[i], (sarmed_phase >> i) & 1u);
            }
        }
      } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        if (rank == 0 && lane == 0) {
            int s = 0, b = 0;
            uint32_t phase = 0, tphase = 0;
            bool ok = true;
            bool issued = false;
            for (int tile = cid; tile < total_tiles && ok; tile += ncl) {
                TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, kPairTok);
                const uint32_t idesc = idesc_e4m3_f32(2 * kTileM, tc.ntile);
                for (int ks = 0; ks < KS && ok; ++ks) {
                    if (!mbar_wait_bounded(&full_bar[s], phase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    const uint32_t st_addr = smem_u32(smem + P::kOffStages + s * P::kStageBytes);
                    for (int h = 0; h < kPairKbPerStage; ++h) {
                        if (!mbar_wait_bounded(&tempty_bar[b], tphase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t a_addr = st_addr + h * kPairABytes;
                        const uint32_t d = tmem_base + b * kPairTok;
                        // two-plane mode: W (hi + lo) of the K block into one partial
#pragma unroll
                        for (int pl = 0; pl < P::kPlanes; ++pl) {
                            const uint32_t b_addr = st_addr + P::kStageABytes + (pl * kPairKbPerStage + h) * kPairBBytes;
#pragma unroll
                            for (int k = 0; k < kBlockK / 32; ++k)
                                umma_f8_pair(d, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32), idesc,
                                             (k > 0 || pl > 0) ? 1u : 0u);
                        }
                        umma_commit_pair(&tfull_bar[b], both);
                        issued = true;
                        if (++b == kPairTBufs) { b = 0; tphase ^= 1; }
                    }
                    if (!ok) break;
                    umma_commit_pair(&empty_bar[s], both);
                    if (++s == P::kStages) { s = 0; phase ^= 1; }
                }
            }
            if (!ok && issued) {
                int lb = (b + kPairTBufs - 1) % kPairTBufs;
                uint32_t lph = (b == 0) ? (tphase ^ 1) : tphase;
                mbar_drain(&tfull_bar[lb], lph);
            }
        }
      } else if (warp == 2) {
        // ------------------------------------------------------------ scale folding (both CTAs)
        // c[kb][gate|up][n] = raw[kb][n] * w_scale (this CTA's weight block(s)), per stage
        int ss = 0;
        uint32_t sphase = 0;
        bool ok = true;
        const int wsb = p.w_rows / kTileM;                 // scale blocks per group
        for (int tile = cid; tile < total_tiles && ok; tile += ncl) {
            TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, kPairTok);
            // gated: gate block nb, up block I/128 + nb; down: block 2 nb + rank
            const int blk0 = kGated ? tc.nb : 2 * tc.nb + static_cast<int>(rank);
            const float* wsg = p.w_scale + ((size_t)tc.g * wsb + blk0) * KB;
            const float* wsu = p.w_scale + ((size_t)tc.g * wsb + (pp.I / kTileM) + tc.nb) * KB;
            for (int ks = 0; ks < KS; ++ks) {
                float sg[kPairKbPerStage], su[kPairKbPerStage];
#pragma unroll
                for (int h = 0; h < kPairKbPerStage; ++h) {
                    sg[h] = __ldg(wsg + ks * kPairKbPerStage + h);
                    su[h] = kGated ? __ldg(wsu + ks * kPairKbPerStage + h) : 0.0f;
                }
                if (!mbar_wait_bounded(&sfull_bar[ss], sphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                float* e = scale_ring + ss * kPairScaleFloats;
#pragma unroll
                for (int h = 0; h < kPairKbPerStage; ++h) {
                    float* f = e + kPairScaleRaw + h * 2 * kPairTok;
                    for (int c = lane; c < tc.ntile; c += 32) {
                        const float a = e[h * kPairTok + c];
                        f[c] = a * sg[h];
                        if (kGated) f[kPairTok + c] = a * su[h];
                    }
                }
                // the raw scales are overwritten by the next TMA load into this entry
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&cready_bar[ss]);
                if (++ss == kPairSStages) { ss = 0; sphase ^= 1; }
            }
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(kPromoRegs));
        // ------------------------------------------------------------ promotion + epilogue (both CTAs)
        const int pw = warp - kFirstPromoWarp;        // 0..15
        const int quarter = warp & 3;                  // TMEM lane quarter
        const int colgrp = pw >> 2;                    // token columns [32 colgrp, +32)
        const int lane_row = quarter * 32 + lane;      // TMEM lane = this CTA's weight row
        const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const uint32_t tempty_leader0 = mapa_u32(smem_u32(&tempty_bar[0]), 0);
        const uint32_t xbar_peer0 = mapa_u32(smem_u32(&xbar[0]), peer);
        float* amax_peer_remote = cluster.map_shared_rank(amax_peer, peer);   // the peer's copy of amax_peer
        int ss = 0, b = 0;
        uint32_t sphase = 0, tphase = 0, ephase = 0;
        uint32_t xphase[2] = {0, 0};
        bool ok = true;
        int it = 0;
        auto group_sync = [&]() -> bool {
            __syncwarp();
            if (lane == 0) mbar_arrive(epi_bar);
            const bool r = mbar_wait_bounded(epi_bar, ephase, abort_flag, kWaitTimeoutNs);
            ephase ^= 1;
            return r;
        };

        for (int tile = cid; tile < total_tiles && ok; tile += ncl, ++it) {
            TileCoord tc = decode_tile(tile, t_prefix, t_chunks, t_start, counts_smem, G, kPairTok);
            const bool live = colgrp * 32 < tc.ntile;
            float2 acc2[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc2[i] = make_float2(0.0f, 0.0f);
            // gated: lanes 0-63 hold gate rows, 64-127 up rows (their own scale vector)
            const int cofs = (kGated && quarter >= 2 ? kPairTok : 0) + colgrp * 32;
            for (int kb = 0; kb < KB; ++kb) {
                const int h = kb % kPairKbPerStage;
                if (h == 0 && !mbar_wait_bounded(&cready_bar[ss], sphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                if (!mbar_wait_bounded(&tfull_bar[b], tphase, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                tc_fence_after();
                if (live) {
                    uint32_t v[32];
                    tmem_ld32(lane_addr + b * kPairTok + colgrp * 32, v);
                    const float* cs = scale_ring + ss * kPairScaleFloats + kPairScaleRaw + h * 2 * kPairTok + cofs;
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 c4 = *reinterpret_cast<const float4*>(cs + j);
                        acc2[j / 2] = ffma2(make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])),
                                            make_float2(c4.x, c4.y), acc2[j / 2]);
                        acc2[j / 2 + 1] = ffma2(make_float2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3])),
                                                make_float2(c4.z, c4.w), acc2[j / 2 + 1]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive_cluster(tempty_leader0 + b * 8);
                    if (h == kPairKbPerStage - 1) mbar_arrive(&sempty_bar[ss]);
                }
                if (h == kPairKbPerStage - 1 && ++ss == kPairSStages) { ss = 0; sphase ^= 1; }
                if (++b == kPairTBufs) { b = 0; tphase ^= 1; }
            }
            if (!ok || *abort_flag) { ok = false; break; }

            // ---------------------------------------------------------- epilogue
            // acc2[i] holds token columns 32 colgrp + 2i, + 1 of this lane's row
            if (kGated) {
                float* hbuf = reinterpret_cast<float*>(smem + P::kOffEpi);   // [128 tokens][64 rows]
                if (quarter >= 2 && live) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        hbuf[(colgrp * 32 + 2 * i) * 64 + lane_row - 64] = acc2[i].x;
                        hbuf[(colgrp * 32 + 2 * i + 1) * 64 + lane_row - 64] = acc2[i].y;
                    }
                }
                if (!group_sync()) { ok = false; break; }
                if (quarter < 2 && live) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
#pragma unroll
                        for (int h2 = 0; h2 < 2; ++h2) {
                            const int c = colgrp * 32 + 2 * i + h2;
                            const float g = h2 ? acc2[i].y : acc2[i].x;
                            const float u = hbuf[c * 64 + lane_row];
                            hbuf[c * 64 + lane_row] = (g / (1.0f + expf(-g))) * u;
                        }
                    }
                }
                if (!group_sync()) { ok = false; break; }
                // per token: amax over this CTA's 64 columns; swap with the peer
                const int par = it & 1;
                for (int c = pw; c < kPairTok; c += kNumPromoWarps) {
                    float a = 0.0f;
                    if (c < tc.nrows) a = fmaxf(fabsf(hbuf[c * 64 + lane]), fabsf(hbuf[c * 64 + lane + 32]));
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
                    if (lane == 0) {
                        amax_own[c] = a;
                        amax_peer_remote[par * kPairTok + c] = a;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive_release_cluster(xbar_peer0 + par * 8);
                {
                    // the peer's 16 warps have written their amax into amax_peer[par]
                    bool got = mbar_try_wait_cluster(&xbar[par], xphase[par]);
                    const uint64_t t0 = globaltimer_ns();
                    while (!got) {
                        if (*abort_flag) break;
                        if (globaltimer_ns() - t0 > kWaitTimeoutNs) { *abort_flag = 1; break; }
                        got = mbar_try_wait_cluster(&xbar[par], xphase[par]);
                    }
                    xphase[par] ^= 1;
                    if (!got) { ok = false; break; }
                }
                uint8_t* outq = reinterpret_cast<uint8_t*>(p.out);
                const int col0 = tc.nb * 128 + 64 * static_cast<int>(rank);
                for (int c = pw; c < tc.ntile; c += kNumPromoWarps) {
                    const size_t row = static_cast<size_t>(tc.row0 + c);
                    uint8_t q0 = 0, q1 = 0, l0 = 0, l1 = 0;
                    float scale = 0.0f;
                    if (c < tc.nrows) {
                        const float amax = fmaxf(amax_own[c], amax_peer[par * kPairTok + c]);
                        if (amax > 0.0f) {
                            const float inv = 448.0f / amax;
                            if constexpr (kX2) {
                                const uint32_t q = cvt_e4m3x2_split(__fmul_rn(hbuf[c * 64 + lane], inv),
                                                                    __fmul_rn(hbuf[c * 64 + lane + 32], inv));
                                q0 = static_cast<uint8_t>(q & 0xFF);
                                q1 = static_cast<uint8_t>((q >> 8) & 0xFF);
                                l0 = static_cast<uint8_t>((q >> 16) & 0xFF);
                                l1 = static_cast<uint8_t>(q >> 24);
                            } else {
                                const uint16_t q = cvt_e4m3x2(hbuf[c * 64 + lane] * inv, hbuf[c * 64 + lane + 32] * inv);
                                q0 = static_cast<uint8_t>(q & 0xFF);
                                q1 = static_cast<uint8_t>(q >> 8);
                            }
                            scale = amax / 448.0f;
                        }
                    }
                    outq[row * p.N + col0 + lane] = q0;
                    outq[row * p.N + col0 + 32 + lane] = q1;
                    if constexpr (kX2) {
                        outq[p.out_plane + row * p.N + col0 + lane] = l0;
                        outq[p.out_plane + row * p.N + col0 + 32 + lane] = l1;
                    }
                    if (rank == 0 && lane == 0) p.out_scale[(size_t)tc.nb * p.out_ld + row] = scale;
                }
                if (!group_sync()) { ok = false; break; }
            } else {
                __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem + P::kOffEpi);   // [128 tok][128]
                if (live) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        stage[(colgrp * 32 + 2 * i) * 128 + lane_row] = __float2bfloat16_rn(acc2[i].x);
                        stage[(colgrp * 32 + 2 * i + 1) * 128 + lane_row] = __float2bfloat16_rn(acc2[i].y);
                    }
                }
                if (!group_sync()) { ok = false; break; }
                __nv_bfloat16* outy = reinterpret_cast<__nv_bfloat16*>(p.out);
                const int col0 = tc.nb * 256 + 128 * static_cast<int>(rank);
                for (int c = pw; c < tc.nrows; c += kNumPromoWarps) {
                    const uint2 v = *reinterpret_cast<const uint2*>(stage + c * 128 + lane * 4);
                    *reinterpret_cast<uint2*>(outy + static_cast<size_t>(tc.row0 + c) * p.N + col0 + lane * 4) = v;
                }
                if (!group_sync()) { ok = false; break; }
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    cluster.sync();          // the even CTA's MMAs into this CTA's TMEM and all cross-CTA arrivals are done
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
    if (threadIdx.x == 0 && *abort_flag && p.error_word) atomicExch(p.error_word, 1);
}

// ------------------------------------------------------------------ host side

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// 2-D uint8 tensor [rows][cols] (row pitch = cols bytes), box [box_rows][128],
// 128-byte swizzle, out-of-bounds rows read as zero.
bool encode_u8_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols};
    cuuint32_t box[2] = {128, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Two e4m3 planes [2][rows][cols] (lo plane `plane` bytes after hi) as a
// 3-D tensor {cols, rows, plane}, box [2][box_rows][128], 128-byte swizzle.
bool encode_u8_planes(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                      uint64_t plane) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {cols, rows, 2};
    cuuint64_t strides[2] = {cols, plane};
    cuuint32_t box[3] = {128, box_rows, 2};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Gate and up weight rows of a group as one 3-D tensor {K, rows, gate/up}
// (the up row of gate row r is r + N): box {128, 128, 2}, 128-byte swizzle.
bool encode_gate_up_3d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t K, uint64_t N) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {K, rows, 2};
    cuuint64_t strides[2] = {K, N * K};
    cuuint32_t box[3] = {128, kTileM, 2};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool kGated, bool kSmall, bool kX2>
cbwStatus_t launch_gemm(const cbwGroupedGemmArgs* a, int* error_word, cudaStream_t stream) {
    using C = GemmCfg<kGated, kSmall, kX2>;
    const int w_rows = kGated ? 2 * a->N : a->N;
    CUtensorMap tw, ta, ta64, ta128;
    if (kGated) {
        if (!encode_gate_up_3d(&tw, a->w, static_cast<uint64_t>(a->num_groups) * w_rows, a->K, a->N))
            return CBW_ERROR_INTERNAL;
    } else if (!encode_u8_2d(&tw, a->w, static_cast<uint64_t>(a->num_groups) * w_rows, a->K, kTileM)) {
        return CBW_ERROR_INTERNAL;
    }
    const uint64_t rows = static_cast<uint64_t>(a->rows), aplane = rows * static_cast<uint64_t>(a->K);
    if (kX2) {
        if (!encode_u8_planes(&ta, a->a, rows, a->K, 32, aplane) ||
            !encode_u8_planes(&ta64, a->a, rows, a->K, 64, aplane) ||
            !encode_u8_planes(&ta128, a->a, rows, a->K, 128, aplane))
            return CBW_ERROR_INTERNAL;
    } else if (!encode_u8_2d(&ta, a->a, rows, a->K, 32) || !encode_u8_2d(&ta64, a->a, rows, a->K, 64) ||
               !encode_u8_2d(&ta128, a->a, rows, a->K, 128)) {
        return CBW_ERROR_INTERNAL;
    }

    static int sm_count[kMaxDevices] = {};
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0;
    if (dev >= 0 && dev < kMaxDevices && sm_count[dev] > 0) {
        sms = sm_count[dev];
    } else {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (dev >= 0 && dev < kMaxDevices) sm_count[dev] = sms;
    }
    {
        cudaError_t e = smem_optin_once(grouped_fp8_gemm_kernel<kGated, kSmall, kX2>, C::kSmemBytes, attr_set);
        if (e != cudaSuccess) {
            std::fprintf(stderr, "cbwFp8BlockScaledGroupedGemm: shared memory opt-in (%d B) failed: %s\n",
                         C::kSmemBytes, cudaGetErrorString(e));
            return CBW_ERROR_EXECUTION_FAILED;
        }
    }
    GemmParams p;
    p.a_scale = a->a_scale;
    p.a_ld = a->a_ld;
    p.w_scale = a->w_scale;
    p.count = a->count;
    p.start = a->start;
    p.out = a->out;
    p.out_scale = a->out_scale;
    p.out_ld = a->out_ld;
    p.out_plane = static_cast<size_t>(a->rows) * a->N;
    p.G = a->num_groups;
    p.K = a->K;
    p.N = a->N;
    p.w_rows = w_rows;
    p.error_word = error_word;
    grouped_fp8_gemm_kernel<kGated, kSmall, kX2><<<sms, kNumThreads, C::kSmemBytes, stream>>>(tw, ta, ta64, ta128, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        cudaFuncAttributes fa;
        cudaFuncGetAttributes(&fa, grouped_fp8_gemm_kernel<kGated, kSmall, kX2>);
        std::fprintf(stderr,
                     "cbwFp8BlockScaledGroupedGemm: launch failed: %s (regs %d, max threads %d, smem %d B)\n",
                     cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, C::kSmemBytes);
        return CBW_ERROR_EXECUTION_FAILED;
    }
    return CBW_SUCCESS;
}

template <bool kGated, bool kX2>
cbwStatus_t launch_gemm_tm(const cbwGroupedGemmArgs* a, int* error_word, cudaStream_t stream,
                           void* const* row_out = nullptr) {
    using C = TmCfg<kGated, kX2>;
    const int w_rows = kGated ? 2 * a->N : a->N;
    CUtensorMap tw, ta, ta64, ta128;
    if (kGated) {
        if (!encode_gate_up_3d(&tw, a->w, static_cast<uint64_t>(a->num_groups) * w_rows, a->K, a->N))
            return CBW_ERROR_INTERNAL;
    } else if (!encode_u8_2d(&tw, a->w, static_cast<uint64_t>(a->num_groups) * w_rows, a->K, C::kWRows)) {
        return CBW_ERROR_INTERNAL;
    }
    const uint64_t rows = static_cast<uint64_t>(a->rows), aplane = rows * static_cast<uint64_t>(a->K);
    if (kX2) {
        if (!encode_u8_planes(&ta, a->a, rows, a->K, 32, aplane) ||
            !encode_u8_planes(&ta64, a->a, rows, a->K, 64, aplane) ||
            !encode_u8_planes(&ta128, a->a, rows, a->K, 128, aplane))
            return CBW_ERROR_INTERNAL;
    } else if (!encode_u8_2d(&ta, a->a, rows, a->K, 32) || !encode_u8_2d(&ta64, a->a, rows, a->K, 64) ||
               !encode_u8_2d(&ta128, a->a, rows, a->K, 128)) {
        return CBW_ERROR_INTERNAL;
    }
    static int sm_count[kMaxDevices] = {};
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0;
    if (dev >= 0 && dev < kMaxDevices && sm_count[dev] > 0) {
        sms = sm_count[dev];
    } else {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (dev >= 0 && dev < kMaxDevices) sm_count[dev] = sms;
    }
    {
        cudaError_t e = smem_optin_once(grouped_fp8_gemm_tm_kernel<kGated, kX2>, C::kSmemBytes, attr_set);
        if (e != cudaSuccess) {
            std::fprintf(stderr, "cbwFp8BlockScaledGroupedGemm: shared memory opt-in (%d B) failed: %s\n",
                         C::kSmemBytes, cudaGetErrorString(e));
            return CBW_ERROR_EXECUTION_FAILED;
        }
    }
    GemmParams p;
    p.a_scale = a->a_scale;
    p.a_ld = a->a_ld;
    p.w_scale = a->w_scale;
    p.count = a->count;
    p.start = a->start;
    p.out = a->out;
    p.out_scale = a->out_scale;
    p.out_ld = a->out_ld;
    p.out_plane = static_cast<size_t>(a->rows) * a->N;
    p.G = a->num_groups;
    p.K = a->K;
    p.N = a->N;
    p.w_rows = w_rows;
    p.error_word = error_word;
    p.row_out = kGated ? nullptr : row_out;
    grouped_fp8_gemm_tm_kernel<kGated, kX2><<<sms, kNumThreads, C::kSmemBytes, stream>>>(tw, ta, ta64, ta128, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        std::fprintf(stderr, "cbwFp8BlockScaledGroupedGemm: token-major launch failed: %s\n", cudaGetErrorString(e));
        return CBW_ERROR_EXECUTION_FAILED;
    }
    return CBW_SUCCESS;
}

// Tensor maps of the pair form: every load moves two K blocks.
//   weights, gated: {128 B, rows, gate/up (I rows apart), K blocks} box {128, 64, 2, 2}
//   weights, down:  {128 B, rows, K blocks} box {128, 128, 2}
//   tokens:         {128 B, rows, K blocks} box {128, 64, 2}; two planes:
//                   {128 B, rows, K blocks, hi/lo} box {128, 64, 2, 2}
//   token scales:   fp32 {a_ld, K blocks} box {128, 2}
bool encode_pair_maps(const cbwGroupedGemmArgs* a, bool gated, bool x2, CUtensorMap* tw, CUtensorMap* ta,
                      CUtensorMap* ts) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    const cuuint64_t K = static_cast<cuuint64_t>(a->K), KB = K / 128;
    const cuuint64_t wrows = static_cast<cuuint64_t>(a->num_groups) * (gated ? 2 * a->N : a->N);
    cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r;
    if (gated) {
        cuuint64_t dims[4] = {128, wrows, 2, KB};
        cuuint64_t str[3] = {K, static_cast<cuuint64_t>(a->N) * K, 128};
        cuuint32_t box[4] = {128, 64, 2, static_cast<cuuint32_t>(kPairKbPerStage)};
        r = fn(tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(a->w), dims, str, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        cuuint64_t dims[3] = {128, wrows, KB};
        cuuint64_t str[2] = {K, 128};
        cuuint32_t box[3] = {128, 128, static_cast<cuuint32_t>(kPairKbPerStage)};
        r = fn(tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(a->w), dims, str, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return false;
    {
        cuuint64_t dims[4] = {128, static_cast<cuuint64_t>(a->rows), KB, 2};
        cuuint64_t str[3] = {K, 128, static_cast<cuuint64_t>(a->rows) * K};
        cuuint32_t box[4] = {128, static_cast<cuuint32_t>(kPairBRows), static_cast<cuuint32_t>(kPairKbPerStage), 2};
        if (fn(ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, x2 ? 4 : 3, const_cast<void*>(a->a), dims, str, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    {
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(a->a_ld), KB};
        cuuint64_t str[1] = {static_cast<cuuint64_t>(a->a_ld) * 4};
        cuuint32_t box[2] = {static_cast<cuuint32_t>(kPairTok), static_cast<cuuint32_t>(kPairKbPerStage)};
        if (fn(ts, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a->a_scale), dims, str, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

template <bool kGated, bool kX2>
cbwStatus_t launch_gemm_pair(const cbwGroupedGemmArgs* a, int* error_word, cudaStream_t stream) {
    using P = PairCfg<kX2>;
    const int w_rows = kGated ? 2 * a->N : a->N;
    CUtensorMap tw, ta, ts;
    if (!encode_pair_maps(a, kGated, kX2, &tw, &ta, &ts)) return CBW_ERROR_INTERNAL;
    static int sm_count[kMaxDevices] = {};
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0;
    if (dev >= 0 && dev < kMaxDevices && sm_count[dev] > 0) {
        sms = sm_count[dev];
    } else {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (dev >= 0 && dev < kMaxDevices) sm_count[dev] = sms;
    }
    {
        cudaError_t e = smem_optin_once(grouped_fp8_gemm_pair_kernel<kGated, kX2>, P::kSmemBytes, attr_set);
        if (e != cudaSuccess) {
            std::fprintf(stderr, "cbwFp8BlockScaledGroupedGemm: shared memory opt-in (%d B) failed: %s\n",
                         P::kSmemBytes, cudaGetErrorString(e));
            return CBW_ERROR_EXECUTION_FAILED;
        }
    }
    PairParams pp;
    GemmParams& p = pp.g;
    p.a_scale = a->a_scale;
    p.a_ld = a->a_ld;
    p.w_scale = a->w_scale;
    p.count = a->count;
    p.start = a->start;
    p.out = a->out;
    p.out_scale = a->out_scale;
    p.out_ld = a->out_ld;
    p.out_plane = static_cast<size_t>(a->rows) * a->N;
    p.G = a->num_groups;
    p.K = a->K;
    p.N = a->N;
    p.w_rows = w_rows;
    p.error_word = error_word;
    pp.I = a->N;
    const int grid = (sms / 2) * 2;
    grouped_fp8_gemm_pair_kernel<kGated, kX2><<<grid, kNumThreads, P::kSmemBytes, stream>>>(tw, ta, ts, pp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        std::fprintf(stderr, "cbwFp8BlockScaledGroupedGemm: pair launch failed: %s\n", cudaGetErrorString(e));
        return CBW_ERROR_EXECUTION_FAILED;
    }
    return CBW_SUCCESS;
}

}  // namespace

namespace {

// row_out != nullptr: the token-major down form with per-row output addresses
// (CBW_ERROR_NOT_SUPPORTED, nothing launched, when another form would run)
cbwStatus_t grouped_gemm(const cbwGroupedGemmArgs* args, void* const* row_out, int* error_word, cwStream_t stream) {
    if (!args) return CBW_ERROR_INVALID_VALUE;
    const cbwGroupedGemmArgs& a = *args;
    if (a.num_groups <= 0 || a.num_groups > kMaxGroups) return CBW_ERROR_INVALID_VALUE;
    if (a.K <= 0 || a.K % 128 || a.N <= 0 || a.N % 128 || a.rows <= 0) return CBW_ERROR_INVALID_VALUE;
    if (!a.a || !a.a_scale || !a.w || !a.w_scale || !a.count || !a.start || !a.out) return CBW_ERROR_INVALID_VALUE;
    if (a.a_ld < a.rows || a.a_ld % 4) return CBW_ERROR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.w) |
         reinterpret_cast<uintptr_t>(a.a_scale) | reinterpret_cast<uintptr_t>(a.out)) & 15)
        return CBW_ERROR_INVALID_VALUE;
    const int base = a.mode & 0xF, tiles = a.mode & 0xF0;
    const bool x2 = (a.mode & CBW_GEMM_ACT_X2) != 0;
    if (a.mode & ~(0xFF | CBW_GEMM_ACT_X2)) return CBW_ERROR_INVALID_VALUE;
    if (tiles != 0 && tiles != CBW_GEMM_SMALL_TILES && tiles != CBW_GEMM_FULL_TILES && tiles != CBW_GEMM_ONE_SM_TILES &&
        tiles != CBW_GEMM_PAIR_TILES && tiles != CBW_GEMM_TOKEN_TILES)
        return CBW_ERROR_INVALID_VALUE;
    // 32-token tiles when the padded rows average at most 32 per group (decode
    // batches: a few tokens per expert), full tiles otherwise
    const bool small = tiles == CBW_GEMM_SMALL_TILES ||
                       (tiles == 0 && static_cast<long long>(a.rows) <= 32ll * a.num_groups);
    if ((tiles == CBW_GEMM_ONE_SM_TILES || tiles == CBW_GEMM_PAIR_TILES || tiles == CBW_GEMM_TOKEN_TILES) && small)
        return CBW_ERROR_INVALID_VALUE;
    const bool pair_ok = a.K % (kPairKbPerStage * kBlockK) == 0 && (base == CBW_GEMM_GATED_SWIGLU || a.N % 256 == 0);
    if (tiles == CBW_GEMM_PAIR_TILES && !pair_ok) return CBW_ERROR_INVALID_VALUE;
    // token-major tiles: 256 weight rows per tile (gate + up, or two W_down blocks)
    const bool tm_ok = base == CBW_GEMM_GATED_SWIGLU || a.N % 256 == 0;
    if (tiles == CBW_GEMM_TOKEN_TILES && !tm_ok) return CBW_ERROR_INVALID_VALUE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // The full form's default is token-major (GLM shape, 4096 tokens, one plane:
    // gate/up 1.27 ms one-SM, 1.87 ms paired; down 0.84 ms one-SM, 0.79 ms paired,
    // before the token-major form); the one-SM and pair forms stay selectable.
    const bool tm = !small && (tiles == CBW_GEMM_TOKEN_TILES || ((tiles == 0 || tiles == CBW_GEMM_FULL_TILES) && tm_ok));
    const bool pair = !tm && (tiles == CBW_GEMM_PAIR_TILES ||
                              (tiles != CBW_GEMM_ONE_SM_TILES && base == CBW_GEMM_DOWN_BF16 && pair_ok));
    if (row_out) {
        if (base != CBW_GEMM_DOWN_BF16 || !tm) return CBW_ERROR_NOT_SUPPORTED;
        return x2 ? launch_gemm_tm<false, true>(&a, error_word, st, row_out)
                  : launch_gemm_tm<false, false>(&a, error_word, st, row_out);
    }
    if (base == CBW_GEMM_GATED_SWIGLU) {
        if (!a.out_scale || a.out_ld < a.rows) return CBW_ERROR_INVALID_VALUE;
        if (x2) {
            if (small) return launch_gemm<true, true, true>(&a, error_word, st);
            if (tm) return launch_gemm_tm<true, true>(&a, error_word, st);
            return pair ? launch_gemm_pair<true, true>(&a, error_word, st) : launch_gemm<true, false, true>(&a, error_word, st);
        }
        if (small) return launch_gemm<true, true, false>(&a, error_word, st);
        if (tm) return launch_gemm_tm<true, false>(&a, error_word, st);
        return pair ? launch_gemm_pair<true, false>(&a, error_word, st) : launch_gemm<true, false, false>(&a, error_word, st);
    }
    if (base == CBW_GEMM_DOWN_BF16) {
        if (x2) {
            // the one-SM full form has no room for two token planes: token-major or
            // pairs when the shape allows them, else the 32-token form
            if (tiles == CBW_GEMM_ONE_SM_TILES) return CBW_ERROR_INVALID_VALUE;
            if (tm) return launch_gemm_tm<false, true>(&a, error_word, st);
            if (small || !pair_ok) return launch_gemm<false, true, true>(&a, error_word, st);
            return launch_gemm_pair<false, true>(&a, error_word, st);
        }
        if (small) return launch_gemm<false, true, false>(&a, error_word, st);
        if (tm) return launch_gemm_tm<false, false>(&a, error_word, st);
        return pair ? launch_gemm_pair<false, false>(&a, error_word, st) : launch_gemm<false, false, false>(&a, error_word, st);
    }
    return CBW_ERROR_INVALID_VALUE;
}

}  // namespace

extern "C" cbwStatus_t cbwFp8BlockScaledGroupedGemm(const cbwGroupedGemmArgs* args, int* error_word,
                                                    cwStream_t stream) {
    return grouped_gemm(args, nullptr, error_word, stream);
}

extern "C" cbwStatus_t cbwFp8BlockScaledGroupedGemmRowOut(const cbwGroupedGemmArgs* args, void* const* row_out,
                                                          int* error_word, cwStream_t stream) {
    if (!row_out || (reinterpret_cast<uintptr_t>(row_out) & 7)) return CBW_ERROR_INVALID_VALUE;
    return grouped_gemm(args, row_out, error_word, stream);
}
