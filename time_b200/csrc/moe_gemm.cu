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
template <bool kGated, bool kSmall = false>
struct GemmCfg {
    static constexpr int kNMax = kGated ? 128 : 256;       // token columns of the promotion layout
    static constexpr int kTileTok = kSmall ? 32 : kNMax;   // tokens per tile
    static constexpr int kStages = kSmall ? (kGated ? 4 : 9) : 3;   // operand ring
    static constexpr int kSStages = 8;                      // token-scale ring
    static constexpr int kATiles = kGated ? 2 : 1;          // gate + up
    static constexpr int kABytes = kATiles * kTileM * kBlockK;
    static constexpr int kBBytes = kTileTok * kBlockK;
    static constexpr int kStageBytes = kABytes + kBBytes;   // 48 KB; small: 36 KB gated, 20 KB down
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
    int G;
    int K;
    int N;                  // output columns per group
    int w_rows;             // weight rows per group (2N gated, N down)
    int* error_word;
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

template <bool kGated, bool kSmall>
__global__ void __launch_bounds__(kNumThreads, 1)
grouped_fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                        const __grid_constant__ CUtensorMap tmap_a,
                        const GemmParams p) {
    using C = GemmCfg<kGated, kSmall>;
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
                const int b_loads = (tc.ntile + 31) >> 5;
                const uint32_t bytes = C::kABytes + b_loads * 32 * kBlockK;
                const int wrow = tc.g * p.w_rows + tc.nb * kTileM;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!mbar_wait_bounded(&empty_bar[s], phase ^ 1, abort_flag, kWaitTimeoutNs)) { ok = false; break; }
                    uint8_t* st = smem + C::kOffStages + s * C::kStageBytes;
                    mbar_arrive_expect_tx(&full_bar[s], bytes);
                    tma_load_2d(&tmap_w, &full_bar[s], st, kb * kBlockK, wrow);
                    if (kGated) tma_load_2d(&tmap_w, &full_bar[s], st + kTileM * kBlockK, kb * kBlockK, wrow + p.N);
                    for (int r = 0; r < b_loads; ++r)
                        tma_load_2d(&tmap_a, &full_bar[s], st + C::kABytes + r * 32 * kBlockK, kb * kBlockK, tc.row0 + 32 * r);
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
#pragma unroll
                    for (int k = 0; k < kBlockK / 32; ++k) {
                        const uint64_t bdesc = umma_desc_sw128(b_addr + k * 32);
                        umma_f8(d, umma_desc_sw128(a_addr + k * 32), bdesc, idesc, k > 0 ? 1u : 0u);
                        if (kGated)
                            umma_f8(d + C::kUpOff, umma_desc_sw128(a_addr + kTileM * kBlockK + k * 32), bdesc, idesc,
                                    k > 0 ? 1u : 0u);
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
                    uint32_t packed = 0;
                    float scale = 0.0f;
                    if (c < tc.nrows) {
                        const float4 v = *reinterpret_cast<const float4*>(stage + c * 128 + lane * 4);
                        float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                        if (amax > 0.0f) {
                            const float inv = 448.0f / amax;
                            const uint32_t lo = cvt_e4m3x2(v.x * inv, v.y * inv);
                            const uint32_t hi = cvt_e4m3x2(v.z * inv, v.w * inv);
                            packed = lo | (hi << 16);
                            scale = amax / 448.0f;
                        }
                    }
                    *reinterpret_cast<uint32_t*>(outq + row * p.N + tc.nb * 128 + lane * 4) = packed;
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

template <bool kGated, bool kSmall>
cbwStatus_t launch_gemm(const cbwGroupedGemmArgs* a, int* error_word, cudaStream_t stream) {
    using C = GemmCfg<kGated, kSmall>;
    const int w_rows = kGated ? 2 * a->N : a->N;
    CUtensorMap tw, ta;
    if (!encode_u8_2d(&tw, a->w, static_cast<uint64_t>(a->num_groups) * w_rows, a->K, kTileM)) return CBW_ERROR_INTERNAL;
    if (!encode_u8_2d(&ta, a->a, static_cast<uint64_t>(a->rows), a->K, 32)) return CBW_ERROR_INTERNAL;

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
        cudaError_t e = smem_optin_once(grouped_fp8_gemm_kernel<kGated, kSmall>, C::kSmemBytes, attr_set);
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
    p.G = a->num_groups;
    p.K = a->K;
    p.N = a->N;
    p.w_rows = w_rows;
    p.error_word = error_word;
    grouped_fp8_gemm_kernel<kGated, kSmall><<<sms, kNumThreads, C::kSmemBytes, stream>>>(tw, ta, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        cudaFuncAttributes fa;
        cudaFuncGetAttributes(&fa, grouped_fp8_gemm_kernel<kGated, kSmall>);
        std::fprintf(stderr,
                     "cbwFp8BlockScaledGroupedGemm: launch failed: %s (regs %d, max threads %d, smem %d B)\n",
                     cudaGetErrorString(e), fa.numRegs, fa.maxThreadsPerBlock, C::kSmemBytes);
        return CBW_ERROR_EXECUTION_FAILED;
    }
    return CBW_SUCCESS;
}

}  // namespace

extern "C" cbwStatus_t cbwFp8BlockScaledGroupedGemm(const cbwGroupedGemmArgs* args, int* error_word,
                                                    cwStream_t stream) {
    if (!args) return CBW_ERROR_INVALID_VALUE;
    const cbwGroupedGemmArgs& a = *args;
    if (a.num_groups <= 0 || a.num_groups > kMaxGroups) return CBW_ERROR_INVALID_VALUE;
    if (a.K <= 0 || a.K % 128 || a.N <= 0 || a.N % 128 || a.rows <= 0) return CBW_ERROR_INVALID_VALUE;
    if (!a.a || !a.a_scale || !a.w || !a.w_scale || !a.count || !a.start || !a.out) return CBW_ERROR_INVALID_VALUE;
    if (a.a_ld < a.rows || a.a_ld % 4) return CBW_ERROR_INVALID_VALUE;
    if ((reinterpret_cast<uintptr_t>(a.a) | reinterpret_cast<uintptr_t>(a.w) |
         reinterpret_cast<uintptr_t>(a.a_scale) | reinterpret_cast<uintptr_t>(a.out)) & 15)
        return CBW_ERROR_INVALID_VALUE;
    const int base = a.mode & 0xF, tiles = a.mode & ~0xF;
    if (tiles != 0 && tiles != CBW_GEMM_SMALL_TILES && tiles != CBW_GEMM_FULL_TILES) return CBW_ERROR_INVALID_VALUE;
    // 32-token tiles when the padded rows average at most 32 per group (decode
    // batches: a few tokens per expert), full tiles otherwise
    const bool small = tiles == CBW_GEMM_SMALL_TILES ||
                       (tiles == 0 && static_cast<long long>(a.rows) <= 32ll * a.num_groups);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (base == CBW_GEMM_GATED_SWIGLU) {
        if (!a.out_scale || a.out_ld < a.rows) return CBW_ERROR_INVALID_VALUE;
        return small ? launch_gemm<true, true>(&a, error_word, st) : launch_gemm<true, false>(&a, error_word, st);
    }
    if (base == CBW_GEMM_DOWN_BF16)
        return small ? launch_gemm<false, true>(&a, error_word, st) : launch_gemm<false, false>(&a, error_word, st);
    return CBW_ERROR_INVALID_VALUE;
}
