// moe_prep.cu -- the memory-bound stages of the MoE FFN block for sm_100a:
// RMSNorm + FP8 quantisation, fp32 router + top-k, stable expert permutation,
// row gather and the weighted combine.  C-ABI entry points are declared in
// include/moe_layer.h.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cfloat>
#include <cstdint>
#include <mutex>

#include "sm100.cuh"
#include "moe_layer.h"

namespace {

using namespace tb;

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// ---------------------------------------------------------------- RMSNorm
// Sum of squares of one row in the reference's order
// (csrc/kernels.cu:67-79 with blockDim 256): the 256 partials
// p[L] = fma-chain over i = L, L+256, ... are reduced by the pairwise tree
// p[L] += p[L+s], s = 128..1.  Lane l of the warp owns L = l + 32m, m = 0..7,
// so strides 128, 64, 32 are lane-local and 16..1 are shuffles; every
// addition pairs the same operands as the reference's tree.
__device__ __forceinline__ float rowsumsq_ref_order(const __nv_bfloat16* x, int H, int lane) {
    float p[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) p[m] = 0.0f;
    for (int j = 0; j < H; j += 256) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int i = j + 32 * m + lane;
            if (i < H) {
                const float v = __bfloat162float(x[i]);
                p[m] = __fmaf_rn(v, v, p[m]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) p[m] = __fadd_rn(p[m], p[m + 4]);
#pragma unroll
    for (int m = 0; m < 2; ++m) p[m] = __fadd_rn(p[m], p[m + 2]);
    float s = __fadd_rn(p[0], p[1]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, o));
    return __shfl_sync(0xffffffffu, s, 0);
}

// One warp per token: rms, n = (x/rms)*gamma (stored in fp32 when n_out is
// given, for the router), 1x128 e4m3 quantisation of n.
__global__ void __launch_bounds__(256)
rmsnorm_quant_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma, int T, int H,
                     float eps, float* __restrict__ rms_out, float* __restrict__ n_out, uint8_t* __restrict__ xq,
                     float* __restrict__ xs, int xs_ld) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= T) return;
    const __nv_bfloat16* xr = x + static_cast<size_t>(warp) * H;
    const float ss = rowsumsq_ref_order(xr, H, lane);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps));
    if (rms_out && lane == 0) rms_out[warp] = rms;
    uint8_t* qr = xq + static_cast<size_t>(warp) * H;
    for (int b = 0; b < H / 128; ++b) {
        const int c = b * 128 + lane * 4;
        const uint2 raw = *reinterpret_cast<const uint2*>(xr + c);
        const float4 g = *reinterpret_cast<const float4*>(gamma + c);
        float v0 = __fmul_rn(__fdiv_rn(bf16_lo(raw.x), rms), g.x);
        float v1 = __fmul_rn(__fdiv_rn(bf16_hi(raw.x), rms), g.y);
        float v2 = __fmul_rn(__fdiv_rn(bf16_lo(raw.y), rms), g.z);
        float v3 = __fmul_rn(__fdiv_rn(bf16_hi(raw.y), rms), g.w);
        if (n_out) *reinterpret_cast<float4*>(n_out + static_cast<size_t>(warp) * H + c) = make_float4(v0, v1, v2, v3);
        float amax = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        uint32_t packed = 0;
        float scale = 0.0f;
        if (amax > 0.0f) {
            const float inv = __fdiv_rn(448.0f, amax);
            packed = static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v0, inv), __fmul_rn(v1, inv))) |
                     (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v2, inv), __fmul_rn(v3, inv))) << 16);
            scale = __fdiv_rn(amax, 448.0f);
        }
        *reinterpret_cast<uint32_t*>(qr + c) = packed;
        if (lane == 0) xs[static_cast<size_t>(b) * xs_ld + warp] = scale;
    }
}

constexpr int kRmsRowMax = 16384;   // bf16 elements of the row staged in shared memory

// One 256-thread block per token, for small T (a warp per token leaves most SMs
// idle and each warp load-latency-bound).  Same arithmetic in the same order:
// thread (m, lane) = 32m + lane accumulates the p[m] of rowsumsq_ref_order for
// its lane, the eight partials meet in shared memory, and warp 0 applies the
// same add tree and shuffle-down reduction; the 1x128 blocks are then split
// over the eight warps.
__global__ void __launch_bounds__(256)
rmsnorm_quant_block_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma, int T, int H,
                           float eps, float* __restrict__ rms_out, float* __restrict__ n_out,
                           uint8_t* __restrict__ xq, float* __restrict__ xs, int xs_ld) {
    __shared__ float part[8][32];
    __shared__ float s_rms;
    __shared__ __align__(16) __nv_bfloat16 row_s[kRmsRowMax];
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const __nv_bfloat16* xr = x + static_cast<size_t>(t) * H;
    // the row in 16-byte loads (one latency), then the reference order from shared memory
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x)
        *reinterpret_cast<uint4*>(row_s + c * 8) = *reinterpret_cast<const uint4*>(xr + c * 8);
    __syncthreads();
    {
        float p = 0.0f;
        for (int j = 0; j < H; j += 256) {
            const int i = j + threadIdx.x;
            if (i < H) {
                const float v = __bfloat162float(row_s[i]);
                p = __fmaf_rn(v, v, p);
            }
        }
        part[warp][lane] = p;
    }
    __syncthreads();
    if (warp == 0) {
        float p[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) p[m] = part[m][lane];
#pragma unroll
        for (int m = 0; m < 4; ++m) p[m] = __fadd_rn(p[m], p[m + 4]);
#pragma unroll
        for (int m = 0; m < 2; ++m) p[m] = __fadd_rn(p[m], p[m + 2]);
        float s2 = __fadd_rn(p[0], p[1]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s2 = __fadd_rn(s2, __shfl_down_sync(0xffffffffu, s2, o));
        if (lane == 0) s_rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(s2, static_cast<float>(H)), eps));
    }
    __syncthreads();
    const float rms = s_rms;
    if (rms_out && threadIdx.x == 0) rms_out[t] = rms;
    uint8_t* qr = xq + static_cast<size_t>(t) * H;
    for (int b = warp; b < H / 128; b += 8) {
        const int c = b * 128 + lane * 4;
        const uint2 raw = *reinterpret_cast<const uint2*>(row_s + c);
        const float4 g = *reinterpret_cast<const float4*>(gamma + c);
        float v0 = __fmul_rn(__fdiv_rn(bf16_lo(raw.x), rms), g.x);
        float v1 = __fmul_rn(__fdiv_rn(bf16_hi(raw.x), rms), g.y);
        float v2 = __fmul_rn(__fdiv_rn(bf16_lo(raw.y), rms), g.z);
        float v3 = __fmul_rn(__fdiv_rn(bf16_hi(raw.y), rms), g.w);
        if (n_out) *reinterpret_cast<float4*>(n_out + static_cast<size_t>(t) * H + c) = make_float4(v0, v1, v2, v3);
        float amax = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        uint32_t packed = 0;
        float scale = 0.0f;
        if (amax > 0.0f) {
            const float inv = __fdiv_rn(448.0f, amax);
            packed = static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v0, inv), __fmul_rn(v1, inv))) |
                     (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v2, inv), __fmul_rn(v3, inv))) << 16);
            scale = __fdiv_rn(amax, 448.0f);
        }
        *reinterpret_cast<uint32_t*>(qr + c) = packed;
        if (lane == 0) xs[static_cast<size_t>(b) * xs_ld + t] = scale;
    }
}

// Up to this many tokens (and hidden sizes) the block-per-token form runs
// (more SMs busy).
constexpr int kRmsBlockPerTokenMaxT = 2048;

// ---------------------------------------------------------------- top-k
// One warp selects the top K of one row of E <= 32*EPT logits with the
// reference's rule (csrc/kernels.cu:437-471): scanning e = 0..E-1, a value
// enters only if strictly greater (so the lower index wins a tie), NaN and
// values <= -FLT_MAX never enter; empty slots get index -1 and weight 0.  The
// weights are exp(v - shift) / sum over the selected slots, shift = v_max when
// v_max > 80 (the reference overflows there) and 0 otherwise.  Lane l holds
// e = l + 32j; each round takes the warp-wide (max value, min index).
template <int EPT>
__device__ __forceinline__ void topk_row(const float* row, int E, int K, int lane, int32_t* idx_out,
                                         float* w_out) {
    float v[EPT];
    bool taken[EPT];
#pragma unroll
    for (int j = 0; j < EPT; ++j) {
        const int e = lane + 32 * j;
        const float lv = (e < E) ? row[e] : -FLT_MAX;
        v[j] = (lv > -FLT_MAX) ? lv : -INFINITY;
        taken[j] = false;
    }
    float sel_v[16];
    int sel_i[16];
    for (int s = 0; s < K; ++s) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
            const int e = lane + 32 * j;
            if (!taken[j] && (v[j] > bv || (v[j] == bv && e < bi)) && v[j] > -INFINITY) { bv = v[j]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (bi == 0x7fffffff) { sel_v[s] = -FLT_MAX; sel_i[s] = -1; continue; }
        sel_v[s] = bv;
        sel_i[s] = bi;
#pragma unroll
        for (int j = 0; j < EPT; ++j)
            if (lane + 32 * j == bi) taken[j] = true;
    }
    if (lane == 0) {
        const float shift = (sel_v[0] > 80.0f) ? sel_v[0] : 0.0f;
        float sum = 0.0f;
        for (int s = 0; s < K; ++s) sum += expf(sel_v[s] - shift);
        for (int s = 0; s < K; ++s) {
            idx_out[s] = sel_i[s];
            w_out[s] = expf(sel_v[s] - shift) / sum;
        }
    }
}

// ---------------------------------------------------------------- router
// Block: 32 tokens x all experts (E <= 32*EPT).  256 threads: thread
// (tg = tid & 7, eg = tid >> 3) owns tokens 4tg..4tg+3 and experts
// eg*EPT..eg*EPT+EPT-1.  Logits accumulate with one fma per k in ascending k
// from +0.0f -- the order the router's parity is defined in.
constexpr int kRouterTok = 32;
constexpr int kRouterKC = 32;

template <int EPT>
__global__ void __launch_bounds__(256)
router_topk_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ rms,
                   const float* __restrict__ gamma, const float* __restrict__ W,
                   const float* __restrict__ bias, int T, int H, int E, int K,
                   float* __restrict__ logits_out, int32_t* __restrict__ topk_idx,
                   float* __restrict__ topk_w) {
    constexpr int EMAX = 32 * EPT;
    // the K-loop tiles and the logits table are never live at the same time
    struct Tiles {
        float n[kRouterKC][kRouterTok];
        float w[kRouterKC][EMAX + 4];
    };
    constexpr int kBytes = sizeof(Tiles) > sizeof(float) * kRouterTok * (EMAX + 1)
                               ? sizeof(Tiles) : sizeof(float) * kRouterTok * (EMAX + 1);
    __shared__ __align__(16) uint8_t buf[kBytes];
    __shared__ float rms_s[kRouterTok];
    auto& n_s = reinterpret_cast<Tiles*>(buf)->n;
    auto& w_s = reinterpret_cast<Tiles*>(buf)->w;
    auto lg_s = reinterpret_cast<float (*)[EMAX + 1]>(buf);

    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * kRouterTok;
    const int tg = tid & 7, eg = tid >> 3;
    if (tid < kRouterTok) rms_s[tid] = (t0 + tid < T) ? rms[t0 + tid] : 1.0f;

    float acc[4][EPT];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < EPT; ++e) acc[a][e] = 0.0f;

    for (int k0 = 0; k0 < H; k0 += kRouterKC) {
        __syncthreads();
        // n tile: 32 tokens x 32 k, transposed into n_s[k][t]
        for (int i = tid; i < kRouterTok * kRouterKC; i += 256) {
            const int t = i / kRouterKC, kk = i % kRouterKC;
            float v = 0.0f;
            if (t0 + t < T) {
                const float xv = __bfloat162float(x[static_cast<size_t>(t0 + t) * H + k0 + kk]);
                v = __fmul_rn(__fdiv_rn(xv, rms_s[t]), gamma[k0 + kk]);
            }
            n_s[kk][t] = v;
        }
        // W tile: E experts x 32 k, transposed into w_s[k][e]
        for (int i = tid; i < EMAX * kRouterKC; i += 256) {
            const int e = i / kRouterKC, kk = i % kRouterKC;
            w_s[kk][e] = (e < E) ? W[static_cast<size_t>(e) * H + k0 + kk] : 0.0f;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < kRouterKC; ++kk) {
            const float4 nv = *reinterpret_cast<const float4*>(&n_s[kk][tg * 4]);
            float wv[EPT];
#pragma unroll
            for (int e = 0; e < EPT; ++e) wv[e] = w_s[kk][eg * EPT + e];
#pragma unroll
            for (int e = 0; e < EPT; ++e) {
                acc[0][e] = __fmaf_rn(nv.x, wv[e], acc[0][e]);
                acc[1][e] = __fmaf_rn(nv.y, wv[e], acc[1][e]);
                acc[2][e] = __fmaf_rn(nv.z, wv[e], acc[2][e]);
                acc[3][e] = __fmaf_rn(nv.w, wv[e], acc[3][e]);
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            const int ee = eg * EPT + e;
            if (ee < E) lg_s[tg * 4 + a][ee] = bias ? __fadd_rn(acc[a][e], bias[ee]) : acc[a][e];
        }
    __syncthreads();

    // top-k: one warp per token, 4 tokens per warp
    const int warp = tid >> 5, lane = tid & 31;
    for (int tl = warp; tl < kRouterTok; tl += 8) {
        const int t = t0 + tl;
        if (t >= T) break;
        if (logits_out)
            for (int e = lane; e < E; e += 32) logits_out[static_cast<size_t>(t) * E + e] = lg_s[tl][e];
        topk_row<EPT>(lg_s[tl], E, K, lane, topk_idx + static_cast<size_t>(t) * K, topk_w + static_cast<size_t>(t) * K);
    }
}

// ---------------------------------------------------------------- tiled router
// logits[t][e] = (fma chain over k = 0..H-1 of n[t][k] * W[e][k], from +0.0f)
// + bias[e]: the same per-(t, e) order as router_topk_kernel, laid out for
// throughput instead of one block per 32 tokens.
// Scalar-FMA form of the same chains (what moe_router_logits runs): thread
// tile TI tokens x 4 experts, so one 16-byte load of a token row (four k
// steps) and of an expert row feed 4*TI FMAs each -- about 1.1 instructions
// per FMA, against ~2.4 for the packed form whose operand pairs cost register
// moves.  Block: 128 threads, 16*TI tokens x 32 experts; thread
// (tg = (lane & 3) + 4 * warp, eg = lane >> 2) owns tokens tg + 16 i and
// experts eg + 8 j, so the 4 token rows and 8 expert rows a warp reads per
// load sit in distinct banks (row pitch 68 floats: row r at bank 4r).  K in
// chunks of 64 through a cp.async double buffer.  Each chain still advances
// one fma per k in ascending k from +0.0f: bit-identical logits.
constexpr int kR3Exp = 32, kR3KC = 64, kR3Ld = kR3KC + 4, kR3Threads = 128;

template <int TI>
constexpr size_t r3_smem_bytes() { return 2 * static_cast<size_t>(16 * TI + kR3Exp) * kR3Ld * sizeof(float); }

template <int TI>
__global__ void __launch_bounds__(kR3Threads, 4)
router_logits_tile_kernel(const float* __restrict__ n, const float* __restrict__ W, const float* __restrict__ bias,
                          int T, int H, int E, float* __restrict__ logits) {
    constexpr int TT = 16 * TI;
    extern __shared__ __align__(16) float r3_smem[];
    auto n_s = reinterpret_cast<float (*)[TT][kR3Ld]>(r3_smem);                          // [2][TT][68]
    auto w_s = reinterpret_cast<float (*)[kR3Exp][kR3Ld]>(r3_smem + 2 * TT * kR3Ld);   // [2][32][68]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tg = (lane & 3) + 4 * warp, eg = lane >> 2;
    const int t0 = blockIdx.y * TT, e0 = blockIdx.x * kR3Exp;

    auto load = [&](int stage, int k0) {
        for (int c = tid; c < (TT + kR3Exp) * (kR3KC / 4); c += kR3Threads) {
            const int row = c >> 4, q = c & 15;
            if (row < TT) {
                const int t = t0 + row;
                const float* src = n + static_cast<size_t>(t < T ? t : 0) * H + k0 + q * 4;
                cp_async16(&n_s[stage][row][q * 4], src, t < T ? 16u : 0u);
            } else {
                const int r = row - TT, e = e0 + r;
                const float* src = W + static_cast<size_t>(e < E ? e : 0) * H + k0 + q * 4;
                cp_async16(&w_s[stage][r][q * 4], src, e < E ? 16u : 0u);
            }
        }
        cp_async_commit();
    };

    float acc[TI][4];
#pragma unroll
    for (int i = 0; i < TI; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    const int nchunks = H / kR3KC;
    load(0, 0);
    for (int c = 0; c < nchunks; ++c) {
        if (c + 1 < nchunks) {
            load((c + 1) & 1, (c + 1) * kR3KC);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int st = c & 1;
#pragma unroll 4
        for (int kk = 0; kk < kR3KC; kk += 4) {
            float4 a[TI], b[4];
#pragma unroll
            for (int i = 0; i < TI; ++i) a[i] = *reinterpret_cast<const float4*>(&n_s[st][tg + 16 * i][kk]);
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(&w_s[st][eg + 8 * j][kk]);
#pragma unroll
            for (int i = 0; i < TI; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[i][j] = __fmaf_rn(a[i].x, b[j].x, acc[i][j]);
                    acc[i][j] = __fmaf_rn(a[i].y, b[j].y, acc[i][j]);
                    acc[i][j] = __fmaf_rn(a[i].z, b[j].z, acc[i][j]);
                    acc[i][j] = __fmaf_rn(a[i].w, b[j].w, acc[i][j]);
                }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TI; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int t = t0 + tg + 16 * i, e = e0 + eg + 8 * j;
            if (t < T && e < E) logits[static_cast<size_t>(t) * E + e] = bias ? __fadd_rn(acc[i][j], bias[e]) : acc[i][j];
        }
}

// Top-k + softmax of the selected logits, one warp per token (8 tokens per
// 256-thread block), with the reference's selection rule (see topk_row).
template <int EPT>
__global__ void __launch_bounds__(256)
topk_softmax_kernel(const float* __restrict__ logits, int T, int E, int K, int32_t* __restrict__ topk_idx,
                    float* __restrict__ topk_w) {
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= T) return;
    topk_row<EPT>(logits + static_cast<size_t>(t) * E, E, K, threadIdx.x & 31, topk_idx + static_cast<size_t>(t) * K,
                  topk_w + static_cast<size_t>(t) * K);
}

// ---------------------------------------------------------------- permutation
// Single block (1024 threads).  Pass 1 counts pairs per local expert; the
// exclusive scan of the counts rounded up to `pad` rows gives the segment
// starts (pad 16 for the GEMM's row segments, 1 for a dense send order); pass 2 assigns each pair its
// row with a stable rank: within a warp by __match_any_sync + popc of the
// lower lanes, across the 32 warps of a 1024-pair chunk by a [32][G] table of
// per-warp counts, across chunks by a running count per group.
constexpr int kPermThreads = 1024;
constexpr int kRowPad = 16;   // segment alignment of the GEMM's row layout

__global__ void __launch_bounds__(kPermThreads)
permute_kernel(const int32_t* __restrict__ idx, int T, int K, int e_begin, int e_end, int num_shared,
               int32_t* __restrict__ counts, int32_t* __restrict__ seg_start, int32_t* __restrict__ pos,
               int32_t* __restrict__ row_token, int32_t* __restrict__ total_rows, int row_capacity,
               int* __restrict__ error_word, int pad) {
    extern __shared__ int sh[];
    const int Gr = e_end - e_begin;
    const int G = Gr + num_shared;
    int* cnt = sh;                 // [G]
    int* start = cnt + G;          // [G]
    int* running = start + G;      // [G]
    int* wtab = running + G;       // [32][G]
    __shared__ int s_total;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = T * K;

    for (int g = tid; g < G; g += kPermThreads) { cnt[g] = (g < Gr) ? 0 : T; running[g] = 0; }
    __syncthreads();
    for (int p = tid; p < P; p += kPermThreads) {
        const int e = idx[p];
        if (e >= e_begin && e < e_end) atomicAdd(&cnt[e - e_begin], 1);
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive scan of padded counts; G may exceed 32 -> serial chunks per lane
        const int per = (G + 31) / 32;
        int local = 0;
        for (int i = 0; i < per; ++i) {
            const int g = lane * per + i;
            if (g < G) local += (cnt[g] + pad - 1) / pad * pad;
        }
        int incl = local;
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < per; ++i) {
            const int g = lane * per + i;
            if (g < G) { start[g] = run; run += (cnt[g] + pad - 1) / pad * pad; }
        }
        if (lane == 31) s_total = incl;
    }
    __syncthreads();
    const int R = s_total;
    if (R > row_capacity) {
        // refuse: zero counts so no downstream kernel touches rows past capacity
        for (int g = tid; g < G; g += kPermThreads) { counts[g] = 0; seg_start[g] = 0; }
        for (int p = tid; p < P; p += kPermThreads) pos[p] = -1;
        if (tid == 0) { *total_rows = 0; if (error_word) atomicExch(error_word, 2); }
        return;
    }
    for (int g = tid; g < G; g += kPermThreads) { counts[g] = cnt[g]; seg_start[g] = start[g]; }
    if (tid == 0) *total_rows = R;
    for (int r = tid; r < R; r += kPermThreads) row_token[r] = -1;
    __syncthreads();

    const unsigned lt_mask = (1u << lane) - 1u;
    for (int c0 = 0; c0 < P; c0 += kPermThreads) {
        for (int i = tid; i < 32 * G; i += kPermThreads) wtab[i] = 0;
        __syncthreads();
        const int p = c0 + tid;
        int g = -1;
        if (p < P) {
            const int e = idx[p];
            if (e >= e_begin && e < e_end) g = e - e_begin;
        }
        const unsigned m = __match_any_sync(0xffffffffu, g);
        const int rank = __popc(m & lt_mask);
        if (g >= 0 && rank == 0) wtab[warp * G + g] = __popc(m);
        __syncthreads();
        if (p < P) {
            if (g >= 0) {
                int base = running[g];
                for (int w = 0; w < warp; ++w) base += wtab[w * G + g];
                const int r = start[g] + base + rank;
                pos[p] = r;
                row_token[r] = p / K;
            } else {
                pos[p] = -1;
            }
        }
        __syncthreads();
        for (int gg = tid; gg < Gr; gg += kPermThreads) {
            int s = 0;
            for (int w = 0; w < 32; ++w) s += wtab[w * G + gg];
            running[gg] += s;
        }
        __syncthreads();
    }
    for (int sidx = 0; sidx < num_shared; ++sidx) {
        const int g = Gr + sidx;
        for (int t = tid; t < T; t += kPermThreads) row_token[start[g] + t] = t;
    }
}

// ---------------------------------------------------------------- multi-block permutation
// The same stable counting sort as permute_kernel, spread over many blocks:
//   mp_count:   block b counts the local-expert pairs of its 256 pairs;
//   mp_scan:    one block turns the [block][group] counts into each block's
//               first row per group (exclusive over blocks), the segment
//               starts (padded) and the capacity check, and resets row_token;
//   mp_scatter: block b ranks its pairs per group (warp match_any + a
//               [warp][group] table, stable in pair order) and writes pos and
//               row_token from its block offsets.
// Results are identical to permute_kernel.
constexpr int kMpPairs = 256;   // pairs per block (one per thread)

__global__ void __launch_bounds__(kMpPairs)
mp_count_kernel(const int32_t* __restrict__ idx, int P, int e_begin, int e_end, int32_t* __restrict__ bcounts) {
    extern __shared__ int mp_sh[];
    const int Gr = e_end - e_begin;
    for (int g = threadIdx.x; g < Gr; g += kMpPairs) mp_sh[g] = 0;
    __syncthreads();
    const int p = blockIdx.x * kMpPairs + threadIdx.x;
    if (p < P) {
        const int e = idx[p];
        if (e >= e_begin && e < e_end) atomicAdd(&mp_sh[e - e_begin], 1);
    }
    __syncthreads();
    for (int g = threadIdx.x; g < Gr; g += kMpPairs) bcounts[static_cast<size_t>(blockIdx.x) * Gr + g] = mp_sh[g];
}

__global__ void __launch_bounds__(1024)
mp_scan_kernel(int32_t* __restrict__ bcounts, int nblocks, int Gr, int num_shared, int T, int pad,
               int32_t* __restrict__ counts, int32_t* __restrict__ seg_start, int32_t* __restrict__ total_rows,
               int32_t* __restrict__ row_token, int row_capacity, int* __restrict__ error_word) {
    extern __shared__ int mp_sh[];
    const int G = Gr + num_shared;
    int* cnt = mp_sh;          // [G]
    int* start = cnt + G;      // [G]
    __shared__ int s_total;
    const int tid = threadIdx.x;
    for (int g = tid; g < Gr; g += blockDim.x) {
        int run = 0;
        for (int b = 0; b < nblocks; ++b) {
            int32_t* c = bcounts + static_cast<size_t>(b) * Gr + g;
            const int v = *c;
            *c = run;                 // this block's first rank within group g
            run += v;
        }
        cnt[g] = run;
    }
    for (int g = Gr + tid; g < G; g += blockDim.x) cnt[g] = T;
    __syncthreads();
    if (tid < 32) {
        const int lane = tid;
        const int per = (G + 31) / 32;
        int local = 0;
        for (int i = 0; i < per; ++i) {
            const int g = lane * per + i;
            if (g < G) local += (cnt[g] + pad - 1) / pad * pad;
        }
        int incl = local;
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - local;
        for (int i = 0; i < per; ++i) {
            const int g = lane * per + i;
            if (g < G) { start[g] = run; run += (cnt[g] + pad - 1) / pad * pad; }
        }
        if (lane == 31) s_total = incl;
    }
    __syncthreads();
    const int R = s_total;
    if (R > row_capacity) {
        // refuse: zero counts so no downstream kernel touches rows past capacity
        for (int g = tid; g < G; g += blockDim.x) { counts[g] = 0; seg_start[g] = 0; }
        if (tid == 0) { *total_rows = -1; if (error_word) atomicExch(error_word, 2); }
        return;
    }
    for (int g = tid; g < G; g += blockDim.x) { counts[g] = cnt[g]; seg_start[g] = start[g]; }
    if (tid == 0) *total_rows = R;
    for (int r = tid; r < R; r += blockDim.x) row_token[r] = -1;
    __syncthreads();     // every reset lands before the shared-expert rows are written
    for (int g = Gr; g < G; ++g)
        for (int t = tid; t < T; t += blockDim.x) row_token[start[g] + t] = t;
}

__global__ void __launch_bounds__(kMpPairs)
mp_scatter_kernel(const int32_t* __restrict__ idx, int P, int K, int e_begin, int e_end,
                  const int32_t* __restrict__ bcounts, const int32_t* __restrict__ seg_start,
                  int32_t* __restrict__ total_rows, int32_t* __restrict__ pos, int32_t* __restrict__ row_token) {
    extern __shared__ int mp_sh[];
    const int Gr = e_end - e_begin;
    int* wtab = mp_sh;     // [8 warps][Gr]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int p = blockIdx.x * kMpPairs + tid;
    const bool refused = *total_rows < 0;
    for (int i = tid; i < 8 * Gr; i += kMpPairs) wtab[i] = 0;
    __syncthreads();
    int g = -1;
    if (p < P && !refused) {
        const int e = idx[p];
        if (e >= e_begin && e < e_end) g = e - e_begin;
    }
    const unsigned m = __match_any_sync(0xffffffffu, g);
    const int rank = __popc(m & ((1u << lane) - 1u));
    if (g >= 0 && rank == 0) wtab[warp * Gr + g] = __popc(m);
    __syncthreads();
    if (p < P) {
        if (g >= 0) {
            int base = seg_start[g] + bcounts[static_cast<size_t>(blockIdx.x) * Gr + g];
            for (int w = 0; w < warp; ++w) base += wtab[w * Gr + g];
            const int r = base + rank;
            pos[p] = r;
            row_token[r] = p / K;
        } else {
            pos[p] = -1;
        }
    }
}

// ---------------------------------------------------------------- gather
__global__ void __launch_bounds__(256)
gather_rows_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ xs, int xs_ld,
                   const int32_t* __restrict__ row_token, const int32_t* __restrict__ total_rows,
                   int row_capacity, int H, uint8_t* __restrict__ xp, float* __restrict__ xps, int xps_ld) {
    const int R = total_rows ? min(*total_rows, row_capacity) : row_capacity;
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = H / 16;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < R; r += nwarps) {
        const int t = row_token[r];
        int4* dst = reinterpret_cast<int4*>(xp + static_cast<size_t>(r) * H);
        if (t >= 0) {
            const int4* src = reinterpret_cast<const int4*>(xq + static_cast<size_t>(t) * H);
            for (int i = lane; i < vec; i += 32) dst[i] = src[i];
            for (int b = lane; b < H / 128; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = xs[static_cast<size_t>(b) * xs_ld + t];
        } else {
            const int4 z = make_int4(0, 0, 0, 0);
            for (int i = lane; i < vec; i += 32) dst[i] = z;
            for (int b = lane; b < H / 128; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = 0.0f;
        }
    }
}

// ---------------------------------------------------------------- combine
// out[t] = bf16(x + sum shared ys[shared_rows[g] + t] + sum_s fma(w, y[pos]) ),
// 8 columns per thread.  y holds the routed rows, ys the shared expert's (the
// same buffer on one GPU; with expert parallelism the routed rows come back
// from the owning ranks into their own buffer).
__global__ void __launch_bounds__(128)
combine_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ y,
               const int32_t* __restrict__ pos, const float* __restrict__ topk_w,
               const __nv_bfloat16* __restrict__ ys, const int32_t* __restrict__ shared_rows, int num_shared,
               int T, int K, int H, __nv_bfloat16* __restrict__ out) {
    const int t = blockIdx.x;
    if (t >= T) return;
    __shared__ int s_row[16 + 2];
    __shared__ float s_w[16];
    if (threadIdx.x < K) {
        s_row[threadIdx.x] = pos[static_cast<size_t>(t) * K + threadIdx.x];
        s_w[threadIdx.x] = topk_w[static_cast<size_t>(t) * K + threadIdx.x];
    }
    if (threadIdx.x < num_shared) s_row[16 + threadIdx.x] = shared_rows[threadIdx.x] + t;
    __syncthreads();
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
        const uint4 xv = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H + c);
        float a[8] = {bf16_lo(xv.x), bf16_hi(xv.x), bf16_lo(xv.y), bf16_hi(xv.y),
                      bf16_lo(xv.z), bf16_hi(xv.z), bf16_lo(xv.w), bf16_hi(xv.w)};
        for (int sidx = 0; sidx < num_shared; ++sidx) {
            const uint4 yv = *reinterpret_cast<const uint4*>(ys + static_cast<size_t>(s_row[16 + sidx]) * H + c);
            a[0] = __fadd_rn(a[0], bf16_lo(yv.x)); a[1] = __fadd_rn(a[1], bf16_hi(yv.x));
            a[2] = __fadd_rn(a[2], bf16_lo(yv.y)); a[3] = __fadd_rn(a[3], bf16_hi(yv.y));
            a[4] = __fadd_rn(a[4], bf16_lo(yv.z)); a[5] = __fadd_rn(a[5], bf16_hi(yv.z));
            a[6] = __fadd_rn(a[6], bf16_lo(yv.w)); a[7] = __fadd_rn(a[7], bf16_hi(yv.w));
        }
        for (int s = 0; s < K; ++s) {
            const int r = s_row[s];
            if (r < 0) continue;
            const float w = s_w[s];
            const uint4 yv = *reinterpret_cast<const uint4*>(y + static_cast<size_t>(r) * H + c);
            a[0] = __fmaf_rn(w, bf16_lo(yv.x), a[0]); a[1] = __fmaf_rn(w, bf16_hi(yv.x), a[1]);
            a[2] = __fmaf_rn(w, bf16_lo(yv.y), a[2]); a[3] = __fmaf_rn(w, bf16_hi(yv.y), a[3]);
            a[4] = __fmaf_rn(w, bf16_lo(yv.z), a[4]); a[5] = __fmaf_rn(w, bf16_hi(yv.z), a[5]);
            a[6] = __fmaf_rn(w, bf16_lo(yv.w), a[6]); a[7] = __fmaf_rn(w, bf16_hi(yv.w), a[7]);
        }
        uint4 o;
        o.x = (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a[1]))) << 16) | __bfloat16_as_ushort(__float2bfloat16_rn(a[0]));
        o.y = (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a[3]))) << 16) | __bfloat16_as_ushort(__float2bfloat16_rn(a[2]));
        o.z = (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a[5]))) << 16) | __bfloat16_as_ushort(__float2bfloat16_rn(a[4]));
        o.w = (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a[7]))) << 16) | __bfloat16_as_ushort(__float2bfloat16_rn(a[6]));
        *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + c) = o;
    }
}

inline moe_status_t launch_status() {
    return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

moe_status_t moe_rmsnorm_quant_n(const void* x_bf16, const float* gamma, int T, int H, float eps,
                                 float* rms_out, float* n_out, void* xq_out, float* xs_out, int xs_ld,
                                 cwStream_t stream) {
    if (T < 0 || H <= 0 || H % 128 || xs_ld < T) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!x_bf16 || !gamma || !xq_out || !xs_out) return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(x_bf16) || !aligned16(gamma) || !aligned16(xq_out)) return MOE_ERR_INVALID_ARGUMENT;
    const int blocks = (T + 7) / 8;
    if (n_out && !aligned16(n_out)) return MOE_ERR_INVALID_ARGUMENT;
    if (T <= kRmsBlockPerTokenMaxT && H <= kRmsRowMax)
        rmsnorm_quant_block_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const __nv_bfloat16*>(x_bf16), gamma, T, H, eps, rms_out, n_out,
            static_cast<uint8_t*>(xq_out), xs_out, xs_ld);
    else
        rmsnorm_quant_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const __nv_bfloat16*>(x_bf16), gamma, T, H, eps, rms_out, n_out,
            static_cast<uint8_t*>(xq_out), xs_out, xs_ld);
    return launch_status();
}

moe_status_t moe_rmsnorm_quant(const void* x_bf16, const float* gamma, int T, int H, float eps,
                               float* rms_out, void* xq_out, float* xs_out, int xs_ld,
                               cwStream_t stream) {
    return moe_rmsnorm_quant_n(x_bf16, gamma, T, H, eps, rms_out, nullptr, xq_out, xs_out, xs_ld, stream);
}

moe_status_t moe_router_logits(const float* n, const float* router_w, const float* router_bias, int T, int H,
                               int E, float* logits, cwStream_t stream) {
    if (T < 0 || H <= 0 || H % 128 || E <= 0 || E > 256) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!n || !router_w || !logits || !aligned16(n) || !aligned16(router_w)) return MOE_ERR_INVALID_ARGUMENT;
    // tokens per thread: the smallest tile whose grid fits in one wave of 148
    // SMs (a lone block is latency-bound, so a grid of <= 148 blocks finishes
    // in about one block's time, and a smaller tile is a shorter block); when
    // even 4 tokens per thread need more than one wave, 2 per thread (several
    // resident blocks per SM).  Measured on B200, H = 5120, E = 160: T = 256 ->
    // 1 (76 us), 512 -> 2 (84 us), 1024 -> 4 (123 us), 2048 / 4096 -> 2
    // (170 / 274 us).
    const int etiles = (E + kR3Exp - 1) / kR3Exp;
    auto blocks_for = [&](int t) { return etiles * ((T + 16 * t - 1) / (16 * t)); };
    const int ti = blocks_for(1) <= 148 ? 1 : (blocks_for(2) <= 148 ? 2 : (blocks_for(4) <= 148 ? 4 : 2));
    const dim3 grid(etiles, (T + 16 * ti - 1) / (16 * ti));
    if (grid.y > 65535) return MOE_ERR_UNSUPPORTED;
    static bool attr[kMaxDevices] = {};
    if (smem_optin_once(router_logits_tile_kernel<4>, static_cast<int>(r3_smem_bytes<4>()), attr) != cudaSuccess)
        return MOE_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (ti == 4)
        router_logits_tile_kernel<4><<<grid, kR3Threads, r3_smem_bytes<4>(), st>>>(n, router_w, router_bias, T, H, E,
                                                                                   logits);
    else if (ti == 2)
        router_logits_tile_kernel<2><<<grid, kR3Threads, r3_smem_bytes<2>(), st>>>(n, router_w, router_bias, T, H, E,
                                                                                   logits);
    else
        router_logits_tile_kernel<1><<<grid, kR3Threads, r3_smem_bytes<1>(), st>>>(n, router_w, router_bias, T, H, E,
                                                                                   logits);
    return launch_status();
}

moe_status_t moe_topk_softmax(const float* logits, int T, int E, int k, int32_t* topk_idx, float* topk_w,
                              cwStream_t stream) {
    if (T < 0 || E <= 0 || E > 256 || k <= 0 || k > 16 || k > E) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!logits || !topk_idx || !topk_w) return MOE_ERR_INVALID_ARGUMENT;
    const int blocks = (T + 7) / 8;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
#define TB_TOPK(EPTV) topk_softmax_kernel<EPTV><<<blocks, 256, 0, s>>>(logits, T, E, k, topk_idx, topk_w)
    switch ((E + 31) / 32) {
        case 1: TB_TOPK(1); break;
        case 2: TB_TOPK(2); break;
        case 3: TB_TOPK(3); break;
        case 4: TB_TOPK(4); break;
        case 5: TB_TOPK(5); break;
        case 6: TB_TOPK(6); break;
        case 7: TB_TOPK(7); break;
        default: TB_TOPK(8); break;
    }
#undef TB_TOPK
    return launch_status();
}

moe_status_t moe_router_topk(const void* x_bf16, const float* rms, const float* gamma,
                             const float* router_w, const float* router_bias,
                             int T, int H, int E, int k,
                             float* logits_out, int32_t* topk_idx, float* topk_w,
                             cwStream_t stream) {
    if (T < 0 || H <= 0 || H % kRouterKC || E <= 0 || E > 256 || k <= 0 || k > 16 || k > E) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!x_bf16 || !rms || !gamma || !router_w || !topk_idx || !topk_w) return MOE_ERR_INVALID_ARGUMENT;
    const int blocks = (T + kRouterTok - 1) / kRouterTok;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x_bf16);
    const int ept = (E + 31) / 32;
#define TB_ROUTER(EPTV) router_topk_kernel<EPTV><<<blocks, 256, 0, s>>>(xb, rms, gamma, router_w, router_bias, T, H, E, k, logits_out, topk_idx, topk_w)
    switch (ept) {
        case 1: TB_ROUTER(1); break;
        case 2: TB_ROUTER(2); break;
        case 3: TB_ROUTER(3); break;
        case 4: TB_ROUTER(4); break;
        case 5: TB_ROUTER(5); break;
        case 6: TB_ROUTER(6); break;
        case 7: TB_ROUTER(7); break;
        default: TB_ROUTER(8); break;
    }
#undef TB_ROUTER
    return launch_status();
}

moe_status_t moe_permute_padded(const int32_t* topk_idx, int T, int k, int e_begin, int e_end,
                                int num_shared, int32_t* counts, int32_t* seg_start, int32_t* pos,
                                int32_t* row_token, int32_t* total_rows, int row_capacity,
                                int* error_word, int pad, cwStream_t stream) {
    const int G = (e_end - e_begin) + num_shared;
    if (T < 0 || k <= 0 || e_begin < 0 || e_end < e_begin || num_shared < 0 || G <= 0 || G > 1024) return MOE_ERR_INVALID_ARGUMENT;
    if (pad < 1 || pad > 128) return MOE_ERR_INVALID_ARGUMENT;
    if (!topk_idx || !counts || !seg_start || !pos || !row_token || !total_rows || row_capacity < 0) return MOE_ERR_INVALID_ARGUMENT;
    const size_t smem = static_cast<size_t>(3 * G + 32 * G) * sizeof(int);
    if (smem > 200 * 1024) return MOE_ERR_UNSUPPORTED;
    static bool attr[kMaxDevices] = {};
    if (smem_optin_once(permute_kernel, 200 * 1024, attr) != cudaSuccess) return MOE_ERR_CUDA;
    permute_kernel<<<1, kPermThreads, smem, static_cast<cudaStream_t>(stream)>>>(
        topk_idx, T, k, e_begin, e_end, num_shared, counts, seg_start, pos, row_token, total_rows,
        row_capacity, error_word, pad);
    return launch_status();
}

moe_status_t moe_permute(const int32_t* topk_idx, int T, int k, int e_begin, int e_end,
                         int num_shared, int32_t* counts, int32_t* seg_start, int32_t* pos,
                         int32_t* row_token, int32_t* total_rows, int row_capacity,
                         int* error_word, cwStream_t stream) {
    return moe_permute_padded(topk_idx, T, k, e_begin, e_end, num_shared, counts, seg_start, pos, row_token,
                              total_rows, row_capacity, error_word, kRowPad, stream);
}

size_t moe_permute_mb_scratch_bytes(int T, int k, int e_begin, int e_end) {
    if (T < 0 || k <= 0 || e_end <= e_begin) return 0;
    const size_t nb = (static_cast<size_t>(T) * k + kMpPairs - 1) / kMpPairs;
    return nb * static_cast<size_t>(e_end - e_begin) * sizeof(int32_t);
}

moe_status_t moe_permute_mb(const int32_t* topk_idx, int T, int k, int e_begin, int e_end, int num_shared,
                            int32_t* counts, int32_t* seg_start, int32_t* pos, int32_t* row_token,
                            int32_t* total_rows, int row_capacity, int* error_word, int pad, void* scratch,
                            size_t scratch_bytes, cwStream_t stream) {
    const int Gr = e_end - e_begin;
    const int G = Gr + num_shared;
    if (T < 0 || k <= 0 || e_begin < 0 || Gr <= 0 || num_shared < 0 || G > 1024 || pad < 1 || pad > 128)
        return MOE_ERR_INVALID_ARGUMENT;
    if (!topk_idx || !counts || !seg_start || !pos || !row_token || !total_rows || row_capacity < 0 || !scratch)
        return MOE_ERR_INVALID_ARGUMENT;
    if (scratch_bytes < moe_permute_mb_scratch_bytes(T, k, e_begin, e_end)) return MOE_ERR_WORKSPACE;
    const int P = T * k;
    const int nb = (P + kMpPairs - 1) / kMpPairs;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t* bc = static_cast<int32_t*>(scratch);
    if (nb > 0) mp_count_kernel<<<nb, kMpPairs, Gr * sizeof(int), st>>>(topk_idx, P, e_begin, e_end, bc);
    mp_scan_kernel<<<1, 1024, 2 * G * sizeof(int), st>>>(bc, nb, Gr, num_shared, T, pad, counts, seg_start,
                                                         total_rows, row_token, row_capacity, error_word);
    if (nb > 0)
        mp_scatter_kernel<<<nb, kMpPairs, 8 * Gr * sizeof(int), st>>>(topk_idx, P, k, e_begin, e_end, bc, seg_start,
                                                                       total_rows, pos, row_token);
    return launch_status();
}

moe_status_t moe_gather_rows_n(const void* xq, const float* xs, int xs_ld, const int32_t* row_token,
                               const int32_t* total_rows, int row_capacity, int H, void* xp, float* xps,
                               int xps_ld, cwStream_t stream) {
    if (H <= 0 || H % 128 || !xq || !xs || !row_token || !xp || !xps || row_capacity < 0 || xps_ld < row_capacity) return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(xq) || !aligned16(xp)) return MOE_ERR_INVALID_ARGUMENT;
    if (row_capacity == 0) return MOE_OK;
    int blocks = (row_capacity + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    gather_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(xq), xs, xs_ld, row_token, total_rows, row_capacity, H,
        static_cast<uint8_t*>(xp), xps, xps_ld);
    return launch_status();
}

moe_status_t moe_gather_rows(const void* xq, const float* xs, int xs_ld, const int32_t* row_token,
                             int row_capacity, int H, void* xp, float* xps, int xps_ld,
                             cwStream_t stream) {
    return moe_gather_rows_n(xq, xs, xs_ld, row_token, nullptr, row_capacity, H, xp, xps, xps_ld, stream);
}

moe_status_t moe_combine_split(const void* x_bf16, const void* y_bf16, const int32_t* pos,
                               const float* topk_w, const void* y_shared_bf16, const int32_t* shared_rows,
                               int num_shared, int T, int k, int H, void* out_bf16, cwStream_t stream) {
    if (T < 0 || k <= 0 || k > 16 || H <= 0 || H % 8 || num_shared < 0 || num_shared > 2) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!x_bf16 || !y_bf16 || !pos || !topk_w || !out_bf16 || (num_shared && (!shared_rows || !y_shared_bf16)))
        return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(x_bf16) || !aligned16(y_bf16) || !aligned16(out_bf16) || (num_shared && !aligned16(y_shared_bf16)))
        return MOE_ERR_INVALID_ARGUMENT;
    combine_kernel<<<T, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(x_bf16), static_cast<const __nv_bfloat16*>(y_bf16), pos, topk_w,
        static_cast<const __nv_bfloat16*>(y_shared_bf16), shared_rows, num_shared, T, k, H,
        static_cast<__nv_bfloat16*>(out_bf16));
    return launch_status();
}

moe_status_t moe_combine(const void* x_bf16, const void* y_bf16, const int32_t* pos,
                         const float* topk_w, const int32_t* shared_rows, int num_shared,
                         int T, int k, int H, void* out_bf16, cwStream_t stream) {
    return moe_combine_split(x_bf16, y_bf16, pos, topk_w, y_bf16, shared_rows, num_shared, T, k, H, out_bf16,
                             stream);
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free router
// Some callers cannot hand this library any device memory beyond their inputs
// and outputs: an engine whose whole device budget is carved out of its own
// arena at start-up, or a plain C / FFI host that binds only this library and
// must not call cudaMalloc on its hot path (cudaMalloc synchronises the whole
// device).  moe_router_topk_noalloc serves them: the [T][E] fp32 logits that
// moe_router_logits + moe_topk_softmax pass between them live in this fixed
// array instead of a caller buffer.  Every GPU that loads the library holds
// it (4 MB) until the process exits.
constexpr int kNoAllocLogits = 1 << 20;   // T * E <= 1,048,576 (e.g. 4096 tokens x 256 experts)
static __device__ __align__(256) float g_router_logits_scratch[kNoAllocLogits];

namespace {

// The array's device address, looked up once per device with that device
// current (host code cannot use the array's name as a device pointer).
float* router_scratch_address(moe_status_t* status) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static float* addr[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *status = MOE_ERR_CUDA;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_router_logits_scratch) != cudaSuccess || !p) {
            *status = MOE_ERR_CUDA;
            return nullptr;
        }
        addr[dev] = static_cast<float*>(p);
    }
    *status = MOE_OK;
    return addr[dev];
}

}  // namespace

extern "C" moe_status_t moe_router_topk_noalloc(const float* n, const float* router_w, const float* router_bias,
                                                int T, int H, int E, int k, int32_t* topk_idx, float* topk_w,
                                                cwStream_t stream) {
    if (T < 0 || E <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (static_cast<long long>(T) * E > kNoAllocLogits) return MOE_ERR_WORKSPACE;   // beyond the fixed array
    if (T == 0) return MOE_OK;
    moe_status_t st = MOE_OK;
    float* logits = router_scratch_address(&st);
    if (!logits) return st;
    // every logit the top-k reads is written first: nothing needs clearing
    st = moe_router_logits(n, router_w, router_bias, T, H, E, logits, stream);
    if (st != MOE_OK) return st;
    return moe_topk_softmax(logits, T, E, k, topk_idx, topk_w, stream);
}
