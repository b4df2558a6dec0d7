// moe_prep.cu -- the memory-bound stages of the MoE FFN block for sm_100a:
// RMSNorm + FP8 quantisation, fp32 router + top-k, stable expert permutation,
// row gather and the weighted combine.  C-ABI entry points are declared in
// include/moe_layer.h.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cooperative_groups.h>
#include <cfloat>
#include <cstdint>
#include <mutex>

#include "sm100.cuh"
#include "moe_layer.h"

namespace {

using namespace tb;

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// Router column order of a row of H = 256 J floats (H % 256 == 0): element
// i = 256j + 32m + 4q + r (r = 2 r_hi + r_lo) is stored at column
//   r_lo * 128J + m * 16J + 16j + 8 r_hi + q,
// so that for fixed (r_lo, m) the 16 lanes (r_hi, q) of all J steps of the
// router's reduction (csrc/kernels.cu:412-435 with blockDim 256) form one
// contiguous run of 16J floats.
__host__ __device__ __forceinline__ int router_col(int i, int J) {
    const int r = i & 3, q = (i >> 2) & 7, m = (i >> 5) & 7, j = i >> 8;
    return (r & 1) * 128 * J + m * 16 * J + 16 * j + 8 * (r >> 1) + q;
}

// n[c .. c+3] of one row (c % 4 == 0), in the plain or the router column order.
template <bool kRc>
__device__ __forceinline__ void store_n(float* row, int c, int H, float v0, float v1, float v2, float v3) {
    if constexpr (kRc) {
        const int J = H >> 8;
        row[router_col(c, J)] = v0;
        row[router_col(c + 1, J)] = v1;
        row[router_col(c + 2, J)] = v2;
        row[router_col(c + 3, J)] = v3;
    } else {
        *reinterpret_cast<float4*>(row + c) = make_float4(v0, v1, v2, v3);
    }
}

// ---------------------------------------------------------------- RMSNorm
// Sum of squares of one row in the reference's order
// (csrc/kernels.cu:67-79 with blockDim 256): the 256 partials
// p[L] = fma-chain over i = L, L+256, ... are reduced by the pairwise tree
// p[L] += p[L+s], s = 128..1.  Lane l of the warp owns L = 8l + u, u = 0..7,
// so one 16-byte load gives a lane the eight elements of its partials in a
// 256-element chunk; strides 128..8 of the tree are shuffles (lane l + 16 ..
// l + 1, same u) and 4, 2, 1 are lane-local.  Every addition pairs the same
// operands as the reference's tree.  H % 128 == 0: a last half chunk is held
// by lanes 0-15.
__device__ __forceinline__ float rowsumsq_ref_order(const __nv_bfloat16* x, int H, int lane) {
    float p[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) p[u] = 0.0f;
    const int full = H >> 8;            // whole 256-element chunks
    int j = 0;
    for (; j + 4 <= full; j += 4) {     // four 16-byte loads in flight per lane
        uint4 r[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) r[a] = *reinterpret_cast<const uint4*>(x + (j + a) * 256 + lane * 8);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const uint32_t w[4] = {r[a].x, r[a].y, r[a].z, r[a].w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float lo = bf16_lo(w[h]), hi = bf16_hi(w[h]);
                p[2 * h] = __fmaf_rn(lo, lo, p[2 * h]);
                p[2 * h + 1] = __fmaf_rn(hi, hi, p[2 * h + 1]);
            }
        }
    }
    for (; j * 256 < H; ++j) {
        const int c = j * 256 + lane * 8;
        if (c < H) {
            const uint4 r = *reinterpret_cast<const uint4*>(x + c);
            const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float lo = bf16_lo(w[h]), hi = bf16_hi(w[h]);
                p[2 * h] = __fmaf_rn(lo, lo, p[2 * h]);
                p[2 * h + 1] = __fmaf_rn(hi, hi, p[2 * h + 1]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float v = __shfl_down_sync(0xffffffffu, p[u], o);
            if (lane < o) p[u] = __fadd_rn(p[u], v);
        }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) p[u] = __fadd_rn(p[u], p[u + 4]);
#pragma unroll
    for (int u = 0; u < 2; ++u) p[u] = __fadd_rn(p[u], p[u + 2]);
    return __shfl_sync(0xffffffffu, __fadd_rn(p[0], p[1]), 0);
}

// n[c .. c+7] of one row (c = 256 j + 8 lane), in the plain or the router
// column order.  In the router order elements c + u and c + u + 4 (u < 4)
// land in adjacent columns, so the lane writes four 8-byte pairs.
template <bool kRc>
__device__ __forceinline__ void store_n8(float* row, int c, int H, const float (&v)[8]) {
    if constexpr (kRc) {
        const int J = H >> 8, j = c >> 8, l = (c >> 3) & 31;
        const int base = (l >> 2) * 16 * J + 16 * j + 2 * (l & 3);
#pragma unroll
        for (int u = 0; u < 4; ++u)
            *reinterpret_cast<float2*>(row + (u & 1) * 128 * J + base + 8 * (u >> 1)) = make_float2(v[u], v[u + 4]);
    } else {
        *reinterpret_cast<float4*>(row + c) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(row + c + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// One warp per token: rms, n = (x/rms)*gamma (stored in fp32 when n_out is
// given, for the router), 1x128 e4m3 quantisation of n (one or two planes).
// Both passes over the row use 16-byte loads: lane l holds elements
// 256j + 8l .. +7 of chunk j, so lanes 0-15 form quantisation block 2j and
// lanes 16-31 block 2j + 1 (an amax over 16 lanes).  The second pass re-reads
// the row, which the first pass has just brought into L2.
template <bool kRc>
__global__ void __launch_bounds__(256)
rmsnorm_quant_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma, int T, int H,
                     float eps, float* __restrict__ rms_out, float* __restrict__ n_out, uint8_t* __restrict__ xq,
                     uint8_t* __restrict__ xq_lo, float* __restrict__ xs, int xs_ld) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= T) return;
    const __nv_bfloat16* xr = x + static_cast<size_t>(warp) * H;
    const float ss = rowsumsq_ref_order(xr, H, lane);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps));
    if (rms_out && lane == 0) rms_out[warp] = rms;
    uint8_t* qr = xq + static_cast<size_t>(warp) * H;
    uint8_t* lr = xq_lo ? xq_lo + static_cast<size_t>(warp) * H : nullptr;
    float* nr = n_out ? n_out + static_cast<size_t>(warp) * H : nullptr;
#pragma unroll 2
    for (int j = 0; j * 256 < H; ++j) {
        const int c = j * 256 + lane * 8;
        const bool live = c < H;            // false only for lanes 16-31 of a last half chunk
        float v[8];
        float amax = 0.0f;
        if (live) {
            const uint4 raw = *reinterpret_cast<const uint4*>(xr + c);
            const float4 g0 = *reinterpret_cast<const float4*>(gamma + c);
            const float4 g1 = *reinterpret_cast<const float4*>(gamma + c + 4);
            const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                v[2 * h] = __fmul_rn(__fdiv_rn(bf16_lo(w[h]), rms), g[2 * h]);
                v[2 * h + 1] = __fmul_rn(__fdiv_rn(bf16_hi(w[h]), rms), g[2 * h + 1]);
            }
            if (nr) store_n8<kRc>(nr, c, H, v);
#pragma unroll
            for (int u = 0; u < 8; ++u) amax = fmaxf(amax, fabsf(v[u]));
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (!live) continue;
        uint2 packed = make_uint2(0u, 0u), packed_lo = make_uint2(0u, 0u);
        float scale = 0.0f;
        if (amax > 0.0f) {
            const float inv = __fdiv_rn(448.0f, amax);
            uint32_t q[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float a = __fmul_rn(v[2 * h], inv), b = __fmul_rn(v[2 * h + 1], inv);
                q[h] = lr ? cvt_e4m3x2_split(a, b) : static_cast<uint32_t>(cvt_e4m3x2(a, b));
            }
            packed.x = (q[0] & 0xFFFFu) | (q[1] << 16);
            packed.y = (q[2] & 0xFFFFu) | (q[3] << 16);
            packed_lo.x = (q[0] >> 16) | (q[1] & 0xFFFF0000u);
            packed_lo.y = (q[2] >> 16) | (q[3] & 0xFFFF0000u);
            scale = __fdiv_rn(amax, 448.0f);
        }
        *reinterpret_cast<uint2*>(qr + c) = packed;
        if (lr) *reinterpret_cast<uint2*>(lr + c) = packed_lo;
        if ((lane & 15) == 0) xs[static_cast<size_t>(2 * j + (lane >> 4)) * xs_ld + warp] = scale;
    }
}

constexpr int kRmsRowMax = 16384;   // bf16 elements of the row staged in shared memory

// One 256-thread block per token, for small T (a warp per token leaves most SMs
// idle and each warp load-latency-bound).  Same arithmetic in the same order:
// thread (m, lane) = 32m + lane accumulates the p[m] of rowsumsq_ref_order for
// its lane, the eight partials meet in shared memory, and warp 0 applies the
// same add tree and shuffle-down reduction; the 1x128 blocks are then split
// over the eight warps.
template <bool kRc>
__global__ void __launch_bounds__(256)
rmsnorm_quant_block_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma, int T, int H,
                           float eps, float* __restrict__ rms_out, float* __restrict__ n_out,
                           uint8_t* __restrict__ xq, uint8_t* __restrict__ xq_lo, float* __restrict__ xs, int xs_ld) {
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
    uint8_t* lr = xq_lo ? xq_lo + static_cast<size_t>(t) * H : nullptr;
    for (int b = warp; b < H / 128; b += 8) {
        const int c = b * 128 + lane * 4;
        const uint2 raw = *reinterpret_cast<const uint2*>(row_s + c);
        const float4 g = *reinterpret_cast<const float4*>(gamma + c);
        float v0 = __fmul_rn(__fdiv_rn(bf16_lo(raw.x), rms), g.x);
        float v1 = __fmul_rn(__fdiv_rn(bf16_hi(raw.x), rms), g.y);
        float v2 = __fmul_rn(__fdiv_rn(bf16_lo(raw.y), rms), g.z);
        float v3 = __fmul_rn(__fdiv_rn(bf16_hi(raw.y), rms), g.w);
        if (n_out) store_n<kRc>(n_out + static_cast<size_t>(t) * H, c, H, v0, v1, v2, v3);
        float amax = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        uint32_t packed = 0, packed_lo = 0;
        float scale = 0.0f;
        if (amax > 0.0f) {
            const float inv = __fdiv_rn(448.0f, amax);
            if (lr) {   // two planes: hi, and the e4m3 residual (one scale)
                const uint32_t s0 = cvt_e4m3x2_split(__fmul_rn(v0, inv), __fmul_rn(v1, inv));
                const uint32_t s1 = cvt_e4m3x2_split(__fmul_rn(v2, inv), __fmul_rn(v3, inv));
                packed = (s0 & 0xFFFFu) | (s1 << 16);
                packed_lo = (s0 >> 16) | (s1 & 0xFFFF0000u);
            } else {
                packed = static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v0, inv), __fmul_rn(v1, inv))) |
                         (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v2, inv), __fmul_rn(v3, inv))) << 16);
            }
            scale = __fdiv_rn(amax, 448.0f);
        }
        *reinterpret_cast<uint32_t*>(qr + c) = packed;
        if (lr) *reinterpret_cast<uint32_t*>(lr + c) = packed_lo;
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
// Router logits in the reference's order (csrc/kernels.cu:412-435, launched
// with blockDim 256): for each (t, e) the 256 lane partials
//   p[l] = fma chain over i = l, l + 256, l + 512, ... < H  (ascending i, from +0.0f)
// are reduced by the pairwise tree p[l] += p[l + s] for s = 128, 64, ..., 1;
// the routing bias, when given, is added to the tree's result.  The lane
// index is split as l = 32m + 4q + r (m: bits 7..5, q: bits 4..2, r: bits
// 1..0), so the tree's levels are, in order: m bit 2, 1, 0 (s = 128, 64, 32),
// q bit 2, 1, 0 (s = 16, 8, 4), r bit 1, 0 (s = 2, 1).

// One warp, one (t, e): lane owns l = lane + 32m; levels s = 128, 64, 32 are
// lane-local, s = 16..1 shuffles (each add pairs the same operands as the
// reference's tree).  Used by the one-call router below.
__device__ __forceinline__ float warp_logit_ref_order(const float* __restrict__ a, const float* __restrict__ b,
                                                      int H, int lane) {
    float p[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) p[m] = 0.0f;
    for (int j = 0; j < H; j += 256) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int i = j + 32 * m + lane;
            if (i < H) p[m] = __fmaf_rn(a[i], b[i], p[m]);
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

// One block per token: n = (x / rms) * gamma into shared memory (the same
// fp32 operations as the RMSNorm kernels), one warp per expert logit in the
// reference order, then the top-k of the row.  The one-call router
// (moe_router_topk): a reference point for tests and small callers, not the
// layer's throughput path.
template <int EPT>
__global__ void __launch_bounds__(256)
router_topk_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ rms,
                   const float* __restrict__ gamma, const float* __restrict__ W,
                   const float* __restrict__ bias, int T, int H, int E, int K,
                   float* __restrict__ logits_out, int32_t* __restrict__ topk_idx,
                   float* __restrict__ topk_w) {
    extern __shared__ __align__(16) float rt_smem[];
    float* n_s = rt_smem;          // [H]
    float* lg_s = rt_smem + H;     // [E]
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float r = rms[t];
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        n_s[i] = __fmul_rn(__fdiv_rn(__bfloat162float(x[static_cast<size_t>(t) * H + i]), r), gamma[i]);
    __syncthreads();
    for (int e = warp; e < E; e += 8) {
        float v = warp_logit_ref_order(n_s, W + static_cast<size_t>(e) * H, H, lane);
        if (bias) v = __fadd_rn(v, bias[e]);
        if (lane == 0) lg_s[e] = v;
    }
    __syncthreads();
    if (warp == 0) {
        if (logits_out)
            for (int e = lane; e < E; e += 32) logits_out[static_cast<size_t>(t) * E + e] = lg_s[e];
        topk_row<EPT>(lg_s, E, K, lane, topk_idx + static_cast<size_t>(t) * K, topk_w + static_cast<size_t>(t) * K);
    }
}

// One warp per logit in the reference order (hidden sizes that are odd
// multiples of 128, where the tiled kernel's 256-element steps do not fit).
__global__ void __launch_bounds__(256)
router_logits_warp_kernel(const float* __restrict__ n, const float* __restrict__ W, const float* __restrict__ bias,
                          int T, int H, int E, float* __restrict__ logits) {
    const long long pair = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (pair >= static_cast<long long>(T) * E) return;
    const int t = static_cast<int>(pair / E), e = static_cast<int>(pair % E);
    float v = warp_logit_ref_order(n + static_cast<size_t>(t) * H, W + static_cast<size_t>(e) * H, H, lane);
    if (bias) v = __fadd_rn(v, bias[e]);
    if (lane == 0) logits[static_cast<size_t>(t) * E + e] = v;
}

// ---------------------------------------------------------------- tiled router
// The layer's router, persistent over 64-token x 32-expert tiles.  A cluster
// of 4 CTAs owns a tile at a time; CTA k of the cluster takes the lanes with
// l % 32 in [8k, 8k + 8) (q in {2k, 2k + 1}), so per 256-element step j it
// needs one 32-byte piece of every row (l = 32m + 8k .. +7).  Thread 0
// streams those pieces with 3-D TMA loads -- box {8 floats, 64 token rows,
// 10 steps} of n and {8 floats, 32 expert rows, 10 steps} of W, laid out in
// shared memory as [step][row][32 bytes] -- through a 4-stage ring of full and
// empty mbarriers, one stage per (m, chunk of <= 10 steps), continuing across
// the cluster's tiles.
//
// A thread owns one lane (l % 32 = 8k + lane % 8) of 8 tokens x 8 experts:
// 64 fma chains, with each one-word shared load feeding 8 fmas (16 loads per
// 64 fmas, which keeps the shared-memory pipe below the fma rate).  Within a
// warp the four 8-lane groups read two adjacent token rows and two adjacent
// expert rows, so every load is one conflict-free wavefront.  The chains of
// one m run over all j (ascending); the 8 m values are processed in the
// tree's post-order 0, 4, 2, 6, 1, 5, 3, 7 and folded with a 3-deep stack,
// which forms exactly the levels s = 128, 64, 32.  The stack lives in tensor
// memory (3 x 64 columns of the thread's TMEM lane), so the registers hold
// only the live chains.  At the end of a tile each CTA leaves its per-lane
// sums in shared memory; after a cluster barrier CTA k reduces the pairs
// [512k, 512k + 512) over the four CTAs (distributed shared memory) with the
// levels s = 16, 8, 4, 2, 1, adds the bias and writes the logit.  Every
// mbarrier wait is bounded (2 s); a CTA whose wait gives up writes NaN logits
// for its tiles (never selected by the top-k) instead of hanging.
constexpr int kRtTok = 64, kRtExp = 32;
constexpr int kRtThreads = 256;
constexpr int kRtJc = 10;                                   // steps per stage
constexpr int kRtCluster = 4;
constexpr int kRtRing = 4;
constexpr int kRtNBox = kRtJc * kRtTok * 32;                // [10 steps][64 rows][32 bytes]
constexpr int kRtWBox = kRtJc * kRtExp * 32;                // [10 steps][32 rows][32 bytes]
constexpr int kRtStageBytes = kRtNBox + kRtWBox;
constexpr int kRtRedRow = kRtExp * 8 + 16;                  // floats per token row (padding: conflict-free stores)
constexpr int kRtRedBytes = kRtTok * kRtRedRow * 4;
constexpr int kRtOffRed = kRtRing * kRtStageBytes;
constexpr int kRtOffBars = kRtOffRed + kRtRedBytes;
constexpr size_t kRtSmemBytes = kRtOffBars + 2 * kRtRing * 8 + 16 + 1024;   // + abort flag, TMEM slot, slack
constexpr uint32_t kRtTmemCols = 512;                       // 2 warps per TMEM lane quarter x 192 columns
constexpr uint64_t kRtWaitNs = 2000000000ull;
static_assert(kRtStageBytes % 1024 == 0 && kRtNBox % 1024 == 0, "TMA destinations stay 1 KB aligned");
static_assert(kRtSmemBytes <= 232448, "router shared memory");

struct RtParams {
    const float* bias;
    float* logits;
    int T, E, J;          // J = H / 256 steps
    int t_tiles, e_tiles;
};

__global__ void __cluster_dims__(kRtCluster, 1, 1) __launch_bounds__(kRtThreads, 1)
router_logits_ref_kernel(const __grid_constant__ CUtensorMap tmap_n, const __grid_constant__ CUtensorMap tmap_w,
                         const RtParams p) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(16) uint8_t rt_raw[];
    // 1 KB aligned by pointer arithmetic on the shared array itself, so the
    // compiler keeps every access below in the shared state space
    uint8_t* smem = rt_raw + ((1024u - (smem_u32(rt_raw) & 1023u)) & 1023u);
    float* red = reinterpret_cast<float*>(smem + kRtOffRed);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRtOffBars);
    uint64_t* empty = full + kRtRing;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kRtRing);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(empty + kRtRing) + 1;
    cg::cluster_group cluster = cg::this_cluster();
    const int k = static_cast<int>(cluster.block_rank());
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = lane >> 3, ln = lane & 7;
    const int tsel = 2 * (warp & 3) + (grp & 1);   // tokens tsel + 8x, x = 0..7
    const int esel = 2 * (warp >> 2) + (grp >> 1); // experts esel + 4y, y = 0..7

    const int cid = blockIdx.x / kRtCluster, ncl = gridDim.x / kRtCluster;
    const int tiles = p.t_tiles * p.e_tiles;
    const int my_tiles = cid < tiles ? (tiles - cid + ncl - 1) / ncl : 0;
    const int C = (p.J + kRtJc - 1) / kRtJc;       // chunks per m
    const int S = 8 * C;                           // stages per tile
    const long long g_total = static_cast<long long>(my_tiles) * S;
    auto m_of = [](int mi) { return ((mi & 1) << 2) | (mi & 2) | (mi >> 2); };

    auto issue = [&](long long g) {                // thread 0 only
        const int it = static_cast<int>(g / S), s = static_cast<int>(g % S);
        const int tile = cid + it * ncl;
        const int t0 = (tile / p.e_tiles) * kRtTok, e0 = (tile % p.e_tiles) * kRtExp;
        const int m = m_of(s / C), j0 = (s % C) * kRtJc;
        const int slot = static_cast<int>(g % kRtRing);
        uint8_t* st = smem + slot * kRtStageBytes;
        mbar_arrive_expect_tx(&full[slot], kRtStageBytes);
        tma_load_3d(&tmap_n, &full[slot], st, 32 * m + 8 * k, t0, j0);
        tma_load_3d(&tmap_w, &full[slot], st + kRtNBox, 32 * m + 8 * k, e0, j0);
    };

    if (tid == 0) {
        for (int i = 0; i < kRtRing; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kRtThreads / 32);
        }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmap_n);
        prefetch_tmap(&tmap_w);
    }
    __syncwarp();
    if (warp == 0) tmem_alloc(tmem_slot, kRtTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // this thread's stack: its TMEM lane (warp % 4 selects the lane quarter),
    // columns [256 * (warp / 4), + 192): slot s at + 64 s
    const uint32_t tstack = *tmem_slot + ((32u * static_cast<uint32_t>(warp & 3)) << 16) +
                            256u * static_cast<uint32_t>(warp >> 2);
    long long issued = 0;                          // thread 0: stages issued so far
    if (tid == 0)
        for (; issued < g_total && issued < kRtRing - 1; ++issued) issue(issued);

    float acc[8][8];
    auto st_slot = [&](int s) {                    // stack[s] = acc
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) r[q] = __float_as_uint(acc[4 * c + q / 8][q % 8]);
            tmem_st32(tstack + 64u * s + 32u * c, r);
        }
    };
    auto add_slot = [&](int s) {                   // acc = stack[s] + acc
        uint32_t r0[32], r1[32];
        tmem_wait_st();                            // this thread's earlier stores have landed

        tmem_ld32(tstack + 64u * s, r0);
        tmem_ld32(tstack + 64u * s + 32u, r1);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 32; ++q) {
            asm volatile("" : "+r"(r0[q]), "+r"(r1[q]));     // uses stay after the wait
            acc[q / 8][q % 8] = __fadd_rn(__uint_as_float(r0[q]), acc[q / 8][q % 8]);
            acc[4 + q / 8][q % 8] = __fadd_rn(__uint_as_float(r1[q]), acc[4 + q / 8][q % 8]);
        }
    };

    bool ok = true;
    for (int it = 0; it < my_tiles; ++it) {
        const int tile = cid + it * ncl;
        const int t0 = (tile / p.e_tiles) * kRtTok, e0 = (tile % p.e_tiles) * kRtExp;
#pragma unroll
        for (int x = 0; x < 8; ++x)
#pragma unroll
            for (int y = 0; y < 8; ++y) acc[x][y] = 0.0f;
        for (int s = 0; s < S; ++s) {
            const long long g = static_cast<long long>(it) * S + s;
            const int slot = static_cast<int>(g % kRtRing);
            if (ok && !mbar_wait_bounded(&full[slot], static_cast<uint32_t>((g / kRtRing) & 1), abort_flag, kRtWaitNs))
                ok = false;
            const int mi = s / C, j0 = (s % C) * kRtJc;
            const int jn = p.J - j0 < kRtJc ? p.J - j0 : kRtJc;
            if (ok) {
                const float* nb = reinterpret_cast<const float*>(smem + slot * kRtStageBytes) + tsel * 8 + ln;
                const float* wb = reinterpret_cast<const float*>(smem + slot * kRtStageBytes + kRtNBox) + esel * 8 + ln;
                auto step = [&](int j) {
                    float a[8], b[8];
#pragma unroll
                    for (int x = 0; x < 8; ++x) a[x] = nb[j * (kRtTok * 8) + x * 64];
#pragma unroll
                    for (int y = 0; y < 8; ++y) b[y] = wb[j * (kRtExp * 8) + y * 32];
#pragma unroll
                    for (int x = 0; x < 8; ++x)
#pragma unroll
                        for (int y = 0; y < 8; ++y) acc[x][y] = __fmaf_rn(a[x], b[y], acc[x][y]);
                };
                if (jn == kRtJc) {
#pragma unroll
                    for (int j = 0; j < kRtJc; ++j) step(j);       // constant offsets, loads run ahead
                } else {
                    for (int j = 0; j < jn; ++j) step(j);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (tid == 0 && issued < g_total && !*abort_flag) {
                // the slot of stage `issued` was last read as stage issued - kRtRing
                const long long prev = issued - kRtRing;
                if (prev < 0 || mbar_wait_bounded(&empty[issued % kRtRing], static_cast<uint32_t>((prev / kRtRing) & 1),
                                                  abort_flag, kRtWaitNs)) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(issued);
                    ++issued;
                }
            }
            if (j0 + jn == p.J) {
                // the m = m_of(mi) chains are complete: fold them into the tree
                __syncwarp();
                switch (mi) {
                    case 0: st_slot(0); break;                                  // p0
                    case 1: add_slot(0); st_slot(0); break;                     // p0 + p4
                    case 2: st_slot(1); break;                                  // p2
                    case 3: add_slot(1); add_slot(0); st_slot(0); break;        // (p0+p4) + (p2+p6)
                    case 4: st_slot(1); break;                                  // p1
                    case 5: add_slot(1); st_slot(1); break;                     // p1 + p5
                    case 6: st_slot(2); break;                                  // p3
                    default: add_slot(2); add_slot(1); add_slot(0); break;      // s = 128, 64, 32 complete
                }
                if (mi != 7) {
#pragma unroll
                    for (int x = 0; x < 8; ++x)
#pragma unroll
                        for (int y = 0; y < 8; ++y) acc[x][y] = 0.0f;
                }
            }
        }
        // this CTA's sums (q = 2k + ln / 4, r = ln % 4) per pair: red[token][expert][ln]
#pragma unroll
        for (int x = 0; x < 8; ++x)
#pragma unroll
            for (int y = 0; y < 8; ++y) red[(tsel + 8 * x) * kRtRedRow + (esel + 4 * y) * 8 + ln] = acc[x][y];
        cluster.sync();
#pragma unroll
        for (int pp = 0; pp < 2; ++pp) {
            const int pair = k * (kRtTok * kRtExp / kRtCluster) + pp * kRtThreads + tid;
            const int tl = pair / kRtExp, el = pair % kRtExp;
            float sq[8][4];   // [q][r]
#pragma unroll
            for (int kk = 0; kk < kRtCluster; ++kk) {
                const uint32_t rr = mapa_u32(smem_u32(red + tl * kRtRedRow + el * 8), static_cast<uint32_t>(kk));
                const float4 lo = ld_dsmem_f4(rr);
                const float4 hi = ld_dsmem_f4(rr + 16);
                sq[2 * kk][0] = lo.x; sq[2 * kk][1] = lo.y; sq[2 * kk][2] = lo.z; sq[2 * kk][3] = lo.w;
                sq[2 * kk + 1][0] = hi.x; sq[2 * kk + 1][1] = hi.y; sq[2 * kk + 1][2] = hi.z; sq[2 * kk + 1][3] = hi.w;
            }
            float x4[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float v0 = __fadd_rn(sq[0][r], sq[4][r]), v1 = __fadd_rn(sq[1][r], sq[5][r]);   // s = 16
                const float v2 = __fadd_rn(sq[2][r], sq[6][r]), v3 = __fadd_rn(sq[3][r], sq[7][r]);
                const float w0 = __fadd_rn(v0, v2), w1 = __fadd_rn(v1, v3);                            // s = 8
                x4[r] = __fadd_rn(w0, w1);                                                             // s = 4
            }
            float v = __fadd_rn(__fadd_rn(x4[0], x4[2]), __fadd_rn(x4[1], x4[3]));                    // s = 2, 1
            const int t = t0 + tl, e = e0 + el;
            if (t < p.T && e < p.E) {
                if (p.bias) v = __fadd_rn(v, p.bias[e]);
                p.logits[static_cast<size_t>(t) * p.E + e] = *abort_flag ? __int_as_float(0x7fc00000) : v;
            }
        }
        cluster.sync();   // the next tile's sums overwrite what the other CTAs just read
    }
    // a CTA that gave up lets the copies it issued land before it exits
    if (tid == 0 && *abort_flag) {
        for (long long g = issued - kRtRing; g < issued; ++g) {
            if (g < 0) continue;
            const uint64_t t1 = globaltimer_ns();
            while (!mbar_try_wait(&full[g % kRtRing], static_cast<uint32_t>((g / kRtRing) & 1)))
                if (globaltimer_ns() - t1 > 200000000ull) break;
        }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(*tmem_slot, kRtTmemCols);
    }
}

// ---------------------------------------------------------------- router, column-ordered inputs
// The layer's router reads n and W in the router column order (router_col
// above): the RMSNorm kernels write n in that order and
// router_columns_kernel reorders W once per forward.
//
// Persistent over 32-token x 32-expert tiles.  A cluster of 2 CTAs owns a
// tile at a time; CTA k takes the lanes with r_lo = k, whose tree level
// (s = 1) is the last one, so everything before it stays inside the CTA.
// Thread 0 streams, per (m, chunk of <= 7 steps), one 2-D TMA box of n
// {112 floats, 32 rows} and one of W through a 6-stage ring of full and
// empty mbarriers.  A thread owns one lane l' = 8 r_hi + q of 8 tokens x 8
// experts (64 fma chains; the two 16-lane halves of a warp share the token
// rows and read adjacent expert rows, 112 floats apart, so every load is one
// conflict-free wavefront).  The m chains run in the tree's post-order with
// the 3-deep stack of levels s = 128, 64, 32 in tensor memory.  At the end of
// a tile the levels s = 16, 8, 4 (q bits) and s = 2 (r_hi) are formed by
// recursive-halving shuffles inside each 16-lane group, one value per
// (token, expert) goes to a double-buffered exchange array, and after one
// cluster barrier CTA k adds the two CTAs' values (s = 1) for the pairs
// [512k, 512k + 512), adds the bias and writes the logits.  Every mbarrier
// wait is bounded (2 s); a CTA whose wait gives up writes NaN logits.
constexpr int kRcTok = 32, kRcExp = 32;
constexpr int kRcThreads = 256;
constexpr int kRcJc = 7;                                    // steps per stage (odd: see the bank note above)
constexpr int kRcCluster = 2;
constexpr int kRcRing = 6;
constexpr int kRcRow = 16 * kRcJc;                          // floats per row per stage
constexpr int kRcNBox = kRcTok * kRcRow * 4;
constexpr int kRcWBox = kRcExp * kRcRow * 4;
constexpr int kRcStageBytes = kRcNBox + kRcWBox;
constexpr int kRcXch = kRcTok * kRcExp;                     // floats per exchange buffer
constexpr int kRcOffXch = kRcRing * kRcStageBytes;
constexpr int kRcOffBars = kRcOffXch + 2 * kRcXch * 4;
constexpr size_t kRcSmemBytes = kRcOffBars + 2 * kRcRing * 8 + 16 + 1024;
constexpr uint32_t kRcTmemCols = 512;                       // 2 warps per TMEM lane quarter x 192 columns
static_assert(kRcStageBytes % 1024 == 0 && kRcNBox % 1024 == 0, "TMA destinations stay 1 KB aligned");
static_assert(kRcSmemBytes <= 232448, "router shared memory");

__global__ void __cluster_dims__(kRcCluster, 1, 1) __launch_bounds__(kRcThreads, 1)
router_logits_rc_kernel(const __grid_constant__ CUtensorMap tmap_n, const __grid_constant__ CUtensorMap tmap_w,
                        const RtParams p) {
    extern __shared__ __align__(16) uint8_t rc_raw[];
    uint8_t* smem = rc_raw + ((1024u - (smem_u32(rc_raw) & 1023u)) & 1023u);
    float* xch = reinterpret_cast<float*>(smem + kRcOffXch);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRcOffBars);
    uint64_t* empty = full + kRcRing;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kRcRing);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(empty + kRcRing) + 1;
    uint32_t k;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(k));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ln = lane & 15;                      // l' = 8 r_hi + q
    const int tsel = warp & 3;                     // tokens tsel + 4x, x = 0..7
    const int esel = 2 * (warp >> 2) + (lane >> 4);// experts esel + 4y, y = 0..7
    const int J = p.J;

    const int cid = blockIdx.x / kRcCluster, ncl = gridDim.x / kRcCluster;
    const int tiles = p.t_tiles * p.e_tiles;
    const int my_tiles = cid < tiles ? (tiles - cid + ncl - 1) / ncl : 0;
    const int C = (J + kRcJc - 1) / kRcJc;         // chunks per m
    const int S = 8 * C;                           // stages per tile
    const int g_total = my_tiles * S;
    auto m_of = [](int mi) { return ((mi & 1) << 2) | (mi & 2) | (mi >> 2); };

    int iss_tile = 0, iss_s = 0;                   // thread 0: the next stage to issue, as (tile, stage)
    auto issue = [&](int g) {                      // thread 0 only; g = iss_tile * S + iss_s
        const int tile = cid + iss_tile * ncl;
        const int t0 = (tile / p.e_tiles) * kRcTok, e0 = (tile % p.e_tiles) * kRcExp;
        const int mi = iss_s / C, j0 = (iss_s - mi * C) * kRcJc;
        const int x = static_cast<int>(k) * 128 * J + m_of(mi) * 16 * J + 16 * j0;
        const int slot = g % kRcRing;
        uint8_t* st = smem + slot * kRcStageBytes;
        mbar_arrive_expect_tx(&full[slot], kRcStageBytes);
        tma_load_2d(&tmap_n, &full[slot], st, x, t0);
        tma_load_2d(&tmap_w, &full[slot], st + kRcNBox, x, e0);
        if (++iss_s == S) { iss_s = 0; ++iss_tile; }
    };

    if (tid == 0) {
        for (int i = 0; i < kRcRing; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kRcThreads / 32);
        }
        *abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&tmap_n);
        prefetch_tmap(&tmap_w);
    }
    __syncwarp();
    if (warp == 0) tmem_alloc(tmem_slot, kRcTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // this thread's stack: its TMEM lane (warp % 4 selects the lane quarter),
    // columns [256 * (warp / 4), + 192): slot s at + 64 s
    const uint32_t tstack = *tmem_slot + ((32u * static_cast<uint32_t>(warp & 3)) << 16) +
                            256u * static_cast<uint32_t>(warp >> 2);
    int issued = 0;                                // thread 0: stages issued so far
    if (tid == 0)
        for (; issued < g_total && issued < kRcRing - 1; ++issued) issue(issued);

    float acc[8][8];
    auto st_slot = [&](int s) {                    // stack[s] = acc
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) r[q] = __float_as_uint(acc[4 * c + q / 8][q % 8]);
            tmem_st32(tstack + 64u * s + 32u * c, r);
        }
    };
    auto add_slot = [&](int s) {                   // acc = stack[s] + acc
        uint32_t r0[32], r1[32];
        tmem_wait_st();                            // this thread's earlier stores have landed
        tmem_ld32(tstack + 64u * s, r0);
        tmem_ld32(tstack + 64u * s + 32u, r1);
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 32; ++q) {
            asm volatile("" : "+r"(r0[q]), "+r"(r1[q]));     // uses stay after the wait
            acc[q / 8][q % 8] = __fadd_rn(__uint_as_float(r0[q]), acc[q / 8][q % 8]);
            acc[4 + q / 8][q % 8] = __fadd_rn(__uint_as_float(r1[q]), acc[4 + q / 8][q % 8]);
        }
    };

    bool ok = true;
    for (int it = 0; it < my_tiles; ++it) {
        const int tile = cid + it * ncl;
        const int t0 = (tile / p.e_tiles) * kRcTok, e0 = (tile % p.e_tiles) * kRcExp;
#pragma unroll
        for (int x = 0; x < 8; ++x)
#pragma unroll
            for (int y = 0; y < 8; ++y) acc[x][y] = 0.0f;
        int mi = 0, ci = 0;                        // stage s = mi * C + ci
        for (int s = 0; s < S; ++s) {
            const int g = it * S + s;
            const int slot = g % kRcRing;
            if (ok && !mbar_wait_bounded(&full[slot], static_cast<uint32_t>((g / kRcRing) & 1), abort_flag, kRtWaitNs))
                ok = false;
            const int j0 = ci * kRcJc;
            const int jn = J - j0 < kRcJc ? J - j0 : kRcJc;
            if (ok) {
                const float* nb = reinterpret_cast<const float*>(smem + slot * kRcStageBytes) + tsel * kRcRow + ln;
                const float* wb = reinterpret_cast<const float*>(smem + slot * kRcStageBytes + kRcNBox) +
                                  esel * kRcRow + ln;
                auto step = [&](int j) {
                    float a[8], b[8];
#pragma unroll
                    for (int x = 0; x < 8; ++x) a[x] = nb[x * 4 * kRcRow + 16 * j];
#pragma unroll
                    for (int y = 0; y < 8; ++y) b[y] = wb[y * 4 * kRcRow + 16 * j];
                    // two experts per packed fma (each lane an IEEE fma, RN): the
                    // same operations as the scalar chains, half the instructions
#pragma unroll
                    for (int x = 0; x < 8; ++x) {
                        const float2 ad = make_float2(a[x], a[x]);
#pragma unroll
                        for (int y = 0; y < 8; y += 2) {
                            const float2 c = __ffma2_rn(ad, make_float2(b[y], b[y + 1]),
                                                        make_float2(acc[x][y], acc[x][y + 1]));
                            acc[x][y] = c.x;
                            acc[x][y + 1] = c.y;
                        }
                    }
                };
#pragma unroll
                for (int j = 0; j < kRcJc; ++j)            // constant offsets, loads run ahead
                    if (j < jn) step(j);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (tid == 0 && issued < g_total && !*abort_flag) {
                // the slot of stage `issued` was last read as stage issued - kRcRing
                const int prev = issued - kRcRing;
                if (prev < 0 || mbar_wait_bounded(&empty[issued % kRcRing], static_cast<uint32_t>((prev / kRcRing) & 1),
                                                  abort_flag, kRtWaitNs)) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    issue(issued);
                    ++issued;
                }
            }
            if (++ci == C) {
                // the m = m_of(mi) chains are complete: fold them into the tree
                __syncwarp();
                switch (mi) {
                    case 0: st_slot(0); break;                                  // p0
                    case 1: add_slot(0); st_slot(0); break;                     // p0 + p4
                    case 2: st_slot(1); break;                                  // p2
                    case 3: add_slot(1); add_slot(0); st_slot(0); break;        // (p0+p4) + (p2+p6)
                    case 4: st_slot(1); break;                                  // p1
                    case 5: add_slot(1); st_slot(1); break;                     // p1 + p5
                    case 6: st_slot(2); break;                                  // p3
                    default: add_slot(2); add_slot(1); add_slot(0); break;      // s = 128, 64, 32 complete
                }
                if (mi != 7) {
#pragma unroll
                    for (int x = 0; x < 8; ++x)
#pragma unroll
                        for (int y = 0; y < 8; ++y) acc[x][y] = 0.0f;
                }
                ci = 0;
                ++mi;
            }
        }
        // levels s = 16, 8, 4 (lane bits 2, 1, 0: q) and s = 2 (lane bit 3:
        // r_hi) by recursive halving: at each level a lane keeps the half of
        // its pairs selected by its lane bit and adds the partner's values
        // for that half.  Afterwards lane l' holds pairs 8 q + 4 r_hi + i.
        float v[64];
#pragma unroll
        for (int x = 0; x < 8; ++x)
#pragma unroll
            for (int y = 0; y < 8; ++y) v[x * 8 + y] = acc[x][y];
        {
            const bool hi = (lane >> 2) & 1;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float send = hi ? v[i] : v[32 + i], keep = hi ? v[32 + i] : v[i];
                v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
            }
        }
        {
            const bool hi = (lane >> 1) & 1;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float send = hi ? v[i] : v[16 + i], keep = hi ? v[16 + i] : v[i];
                v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 2));
            }
        }
        {
            const bool hi = lane & 1;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float send = hi ? v[i] : v[8 + i], keep = hi ? v[8 + i] : v[i];
                v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 1));
            }
        }
        {
            const bool hi = (lane >> 3) & 1;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float send = hi ? v[i] : v[4 + i], keep = hi ? v[4 + i] : v[i];
                v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 8));
            }
        }
        // this CTA's value (r_lo = k) per pair: xch[buf][tl][el ^ 2 (tl / 4)]
        // (the XOR spreads a warp's stores over the banks, keeps el pairs adjacent)
        float* xb = xch + (it & 1) * kRcXch;
        {
            const int q = ln & 7, rh = ln >> 3;
            const int tl = tsel + 4 * q;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int el = esel + 4 * (4 * rh + i);
                xb[tl * kRcExp + (el ^ (2 * q))] = v[i];
            }
        }
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
        {
            const int pair = static_cast<int>(k) * (kRcXch / kRcCluster) + 2 * tid;   // two adjacent experts
            const int tl = pair / kRcExp, el = pair % kRcExp;
            const uint32_t a = smem_u32(xb + tl * kRcExp + (el ^ (2 * ((tl >> 2) & 7))));
            float2 c0, c1;
            asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(c0.x), "=f"(c0.y) : "r"(mapa_u32(a, 0)) : "memory");
            asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(c1.x), "=f"(c1.y) : "r"(mapa_u32(a, 1)) : "memory");
            const int t = t0 + tl;
            const bool bad = *abort_flag != 0;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int e = e0 + el + h;
                if (t < p.T && e < p.E) {
                    float val = __fadd_rn(h ? c0.y : c0.x, h ? c1.y : c1.x);                   // s = 1
                    if (p.bias) val = __fadd_rn(val, p.bias[e]);
                    p.logits[static_cast<size_t>(t) * p.E + e] = bad ? __int_as_float(0x7fc00000) : val;
                }
            }
        }
    }
    // the peer may still read this CTA's exchange array
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    // a CTA that gave up lets the copies it issued land before it exits
    if (tid == 0 && *abort_flag) {
        for (int g = issued - kRcRing; g < issued; ++g) {
            if (g < 0) continue;
            const uint64_t t1 = globaltimer_ns();
            while (!mbar_try_wait(&full[g % kRcRing], static_cast<uint32_t>((g / kRcRing) & 1)))
                if (globaltimer_ns() - t1 > 200000000ull) break;
        }
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(*tmem_slot, kRcTmemCols);
    }
}

// W (or any [rows][H] matrix) into the router column order.
__global__ void __launch_bounds__(256)
router_columns_kernel(const float* __restrict__ src, float* __restrict__ dst, int rows, int H) {
    const long long i4 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;   // 4 elements each
    const int per_row = H / 4;
    if (i4 >= static_cast<long long>(rows) * per_row) return;
    const int row = static_cast<int>(i4 / per_row), c = static_cast<int>(i4 % per_row) * 4;
    const float4 v = *reinterpret_cast<const float4*>(src + static_cast<size_t>(row) * H + c);
    float* d = dst + static_cast<size_t>(row) * H;
    const int J = H / 256;
    d[router_col(c, J)] = v.x;
    d[router_col(c + 1, J)] = v.y;
    d[router_col(c + 2, J)] = v.z;
    d[router_col(c + 3, J)] = v.w;
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
    // a thread per group (consecutive groups: coalesced rows of bcounts); the
    // counts of 16 blocks are loaded before any of them is overwritten, so a
    // group costs nblocks / 16 memory round trips instead of nblocks; each
    // block's count becomes its first rank within the group
    for (int g = tid; g < Gr; g += blockDim.x) {
        int run = 0;
        for (int b0 = 0; b0 < nblocks; b0 += 16) {
            int v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u)
                v[u] = b0 + u < nblocks ? bcounts[static_cast<size_t>(b0 + u) * Gr + g] : 0;
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                if (b0 + u < nblocks) bcounts[static_cast<size_t>(b0 + u) * Gr + g] = run;
                run += v[u];
            }
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
                   int row_capacity, int H, uint8_t* __restrict__ xp, float* __restrict__ xps, int xps_ld,
                   const uint8_t* __restrict__ xq_lo, uint8_t* __restrict__ xp_lo) {
    const int R = total_rows ? min(*total_rows, row_capacity) : row_capacity;
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int vec = H / 16;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < R; r += nwarps) {
        const int t = row_token[r];
        int4* dst = reinterpret_cast<int4*>(xp + static_cast<size_t>(r) * H);
        int4* dlo = xp_lo ? reinterpret_cast<int4*>(xp_lo + static_cast<size_t>(r) * H) : nullptr;
        if (t >= 0) {
            const int4* src = reinterpret_cast<const int4*>(xq + static_cast<size_t>(t) * H);
            for (int i = lane; i < vec; i += 32) dst[i] = src[i];
            if (dlo) {
                const int4* slo = reinterpret_cast<const int4*>(xq_lo + static_cast<size_t>(t) * H);
                for (int i = lane; i < vec; i += 32) dlo[i] = slo[i];
            }
            for (int b = lane; b < H / 128; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = xs[static_cast<size_t>(b) * xs_ld + t];
        } else {
            const int4 z = make_int4(0, 0, 0, 0);
            for (int i = lane; i < vec; i += 32) dst[i] = z;
            if (dlo)
                for (int i = lane; i < vec; i += 32) dlo[i] = z;
            for (int b = lane; b < H / 128; b += 32) xps[static_cast<size_t>(b) * xps_ld + r] = 0.0f;
        }
    }
}

// Token-major form of gather_rows_kernel for the layer: a warp takes token t
// and stores its row (both planes and its 1x128 scales) into each of its
// routed rows pos[t*K + s] >= 0 and its shared-expert rows shared_start[g] + t,
// reading the token once (the row-major gather re-reads a token for every row
// it fills, and its write stream pushes the token out of L2 in between).  A
// lane loads 8 of the row's 16-byte pieces before storing them to every
// destination.  Rows that no pair fills (row_token < 0: segment padding) are
// zeroed as the gather zeroes them, so xp and xps come out identical to
// gather_rows_kernel's.
constexpr int kScatterMaxK = 16, kScatterMaxShared = 2, kScatterPieces = 8;

__device__ __forceinline__ void scatter_plane(const int4* __restrict__ src, uint8_t* __restrict__ base, int H,
                                              int vec, int lane, const int (&r)[kScatterMaxK + kScatterMaxShared]) {
    for (int c0 = lane; c0 < vec; c0 += 32 * kScatterPieces) {
        int4 v[kScatterPieces];
#pragma unroll
        for (int u = 0; u < kScatterPieces; ++u) {
            const int c = c0 + 32 * u;
            if (c < vec) v[u] = src[c];
        }
#pragma unroll
        for (int d = 0; d < kScatterMaxK + kScatterMaxShared; ++d) {
            if (r[d] < 0) continue;
            int4* dst = reinterpret_cast<int4*>(base + static_cast<size_t>(r[d]) * H);
#pragma unroll
            for (int u = 0; u < kScatterPieces; ++u) {
                const int c = c0 + 32 * u;
                if (c < vec) dst[c] = v[u];
            }
        }
    }
}

__global__ void __launch_bounds__(256)
scatter_rows_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ xs, int xs_ld,
                    const int32_t* __restrict__ pos, int T, int K, const int32_t* __restrict__ shared_start,
                    int num_shared, const int32_t* __restrict__ row_token, const int32_t* __restrict__ total_rows,
                    int row_capacity, int H, uint8_t* __restrict__ xp, float* __restrict__ xps, int xps_ld,
                    const uint8_t* __restrict__ xq_lo, uint8_t* __restrict__ xp_lo) {
    const int R = min(*total_rows, row_capacity);
    if (R <= 0) return;
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int vec = H / 16, nblk = H / 128;
    for (int t = gw; t < T; t += nwarps) {
        int r[kScatterMaxK + kScatterMaxShared];
#pragma unroll
        for (int s = 0; s < kScatterMaxK; ++s) {
            const int v = s < K ? pos[static_cast<size_t>(t) * K + s] : -1;
            r[s] = (v >= 0 && v < R) ? v : -1;
        }
#pragma unroll
        for (int g = 0; g < kScatterMaxShared; ++g) {
            const int v = g < num_shared ? shared_start[g] + t : -1;
            r[kScatterMaxK + g] = (v >= 0 && v < R) ? v : -1;
        }
        scatter_plane(reinterpret_cast<const int4*>(xq + static_cast<size_t>(t) * H), xp, H, vec, lane, r);
        if (xp_lo) scatter_plane(reinterpret_cast<const int4*>(xq_lo + static_cast<size_t>(t) * H), xp_lo, H, vec, lane, r);
        for (int b = lane; b < nblk; b += 32) {
            const float v = xs[static_cast<size_t>(b) * xs_ld + t];
#pragma unroll
            for (int d = 0; d < kScatterMaxK + kScatterMaxShared; ++d)
                if (r[d] >= 0) xps[static_cast<size_t>(b) * xps_ld + r[d]] = v;
        }
    }
    // padding rows: zero, 32 rows looked up per step
    const int4 z = make_int4(0, 0, 0, 0);
    for (int r0 = gw * 32; r0 < R; r0 += nwarps * 32) {
        const int rr = r0 + lane;
        unsigned pad = __ballot_sync(0xffffffffu, rr < R && row_token[rr] < 0);
        while (pad) {
            const int i = __ffs(pad) - 1;
            pad &= pad - 1;
            const int row = r0 + i;
            int4* dst = reinterpret_cast<int4*>(xp + static_cast<size_t>(row) * H);
            for (int c = lane; c < vec; c += 32) dst[c] = z;
            if (xp_lo) {
                int4* dlo = reinterpret_cast<int4*>(xp_lo + static_cast<size_t>(row) * H);
                for (int c = lane; c < vec; c += 32) dlo[c] = z;
            }
            for (int b = lane; b < nblk; b += 32) xps[static_cast<size_t>(b) * xps_ld + row] = 0.0f;
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

PFN_cuTensorMapEncodeTiled_v12000 rt_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// The router's view of an fp32 [rows][H] matrix (H % 256 == 0) as a 3-D
// tensor {256 lanes l, rows, H/256 steps j} -- element (l, row, j) is
// m[row][256 j + l] -- with box {8, box_rows, 10}: a TMA load lands as
// [step][row][8 floats] in shared memory.  Rows and steps past the end read
// as zero.
bool encode_rt_map(CUtensorMap* map, const float* base, int rows, int H, int box_rows) {
    auto fn = rt_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {256, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(H / 256)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(H) * 4, 1024};
    cuuint32_t box[3] = {8, static_cast<cuuint32_t>(box_rows), kRtJc};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The router-column-ordered [rows][H] fp32 matrix as a 2-D tensor with box
// {112 floats, 32 rows}: one (r_lo, m, 7-step chunk) piece of 32 rows per load.
bool encode_rc_map(CUtensorMap* map, const float* base, int rows, int H) {
    auto fn = rt_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(H) * 4};
    cuuint32_t box[2] = {kRcRow, kRcTok};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace


namespace {
template <bool kRc>
moe_status_t rmsnorm_quant_launch(const void* x_bf16, const float* gamma, int T, int H, float eps,
                                  float* rms_out, float* n_out, void* xq_out, float* xs_out, int xs_ld,
                                  cwStream_t stream, void* xq_lo_out = nullptr) {
    if (T < 0 || H <= 0 || H % 128 || xs_ld < T) return MOE_ERR_INVALID_ARGUMENT;
    if (kRc && (H % 256 || !n_out)) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!x_bf16 || !gamma || !xq_out || !xs_out) return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(x_bf16) || !aligned16(gamma) || !aligned16(xq_out)) return MOE_ERR_INVALID_ARGUMENT;
    const int blocks = (T + 7) / 8;
    if (n_out && !aligned16(n_out)) return MOE_ERR_INVALID_ARGUMENT;
    if (xq_lo_out && !aligned16(xq_lo_out)) return MOE_ERR_INVALID_ARGUMENT;
    if (T <= kRmsBlockPerTokenMaxT && H <= kRmsRowMax)
        rmsnorm_quant_block_kernel<kRc><<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const __nv_bfloat16*>(x_bf16), gamma, T, H, eps, rms_out, n_out,
            static_cast<uint8_t*>(xq_out), static_cast<uint8_t*>(xq_lo_out), xs_out, xs_ld);
    else
        rmsnorm_quant_kernel<kRc><<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const __nv_bfloat16*>(x_bf16), gamma, T, H, eps, rms_out, n_out,
            static_cast<uint8_t*>(xq_out), static_cast<uint8_t*>(xq_lo_out), xs_out, xs_ld);
    return launch_status();
}
}  // namespace

extern "C" {

moe_status_t moe_rmsnorm_quant_n(const void* x_bf16, const float* gamma, int T, int H, float eps,
                                 float* rms_out, float* n_out, void* xq_out, float* xs_out, int xs_ld,
                                 cwStream_t stream) {
    return rmsnorm_quant_launch<false>(x_bf16, gamma, T, H, eps, rms_out, n_out, xq_out, xs_out, xs_ld, stream);
}

moe_status_t moe_rmsnorm_quant_rc(const void* x_bf16, const float* gamma, int T, int H, float eps,
                                  float* rms_out, float* n_rc_out, void* xq_out, float* xs_out, int xs_ld,
                                  cwStream_t stream) {
    return rmsnorm_quant_launch<true>(x_bf16, gamma, T, H, eps, rms_out, n_rc_out, xq_out, xs_out, xs_ld, stream);
}

moe_status_t moe_rmsnorm_quant_x2(const void* x_bf16, const float* gamma, int T, int H, float eps, float* rms_out,
                                  float* n_out, int n_router_cols, void* xq_out, void* xq_lo_out, float* xs_out,
                                  int xs_ld, cwStream_t stream) {
    if (!xq_lo_out) return MOE_ERR_INVALID_ARGUMENT;
    return n_router_cols
        ? rmsnorm_quant_launch<true>(x_bf16, gamma, T, H, eps, rms_out, n_out, xq_out, xs_out, xs_ld, stream, xq_lo_out)
        : rmsnorm_quant_launch<false>(x_bf16, gamma, T, H, eps, rms_out, n_out, xq_out, xs_out, xs_ld, stream,
                                      xq_lo_out);
}

moe_status_t moe_rmsnorm_quant(const void* x_bf16, const float* gamma, int T, int H, float eps,
                               float* rms_out, void* xq_out, float* xs_out, int xs_ld,
                               cwStream_t stream) {
    return moe_rmsnorm_quant_n(x_bf16, gamma, T, H, eps, rms_out, nullptr, xq_out, xs_out, xs_ld, stream);
}

moe_status_t moe_router_columns(const float* src, float* dst, int rows, int H, cwStream_t stream) {
    if (rows < 0 || H <= 0 || H % 256) return MOE_ERR_INVALID_ARGUMENT;
    if (rows == 0) return MOE_OK;
    if (!src || !dst || src == dst || !aligned16(src) || !aligned16(dst)) return MOE_ERR_INVALID_ARGUMENT;
    const long long n4 = static_cast<long long>(rows) * (H / 4);
    if ((n4 + 255) / 256 > 0x7fffffffll) return MOE_ERR_UNSUPPORTED;
    router_columns_kernel<<<static_cast<unsigned>((n4 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        src, dst, rows, H);
    return launch_status();
}

moe_status_t moe_router_logits_rc(const float* n_rc, const float* w_rc, const float* router_bias, int T, int H,
                                  int E, float* logits, cwStream_t stream) {
    if (T < 0 || H <= 0 || H % 256 || E <= 0 || E > 256) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!n_rc || !w_rc || !logits || !aligned16(n_rc) || !aligned16(w_rc)) return MOE_ERR_INVALID_ARGUMENT;
    CUtensorMap tn, tw;
    if (!encode_rc_map(&tn, n_rc, T, H) || !encode_rc_map(&tw, w_rc, E, H)) return MOE_ERR_CUDA;
    static bool attr[kMaxDevices] = {};
    static int max_clusters[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
    if (smem_optin_once(router_logits_rc_kernel, static_cast<int>(kRcSmemBytes), attr) != cudaSuccess)
        return MOE_ERR_CUDA;
    RtParams prm;
    prm.bias = router_bias;
    prm.logits = logits;
    prm.T = T;
    prm.E = E;
    prm.J = H / 256;
    prm.t_tiles = (T + kRcTok - 1) / kRcTok;
    prm.e_tiles = (E + kRcExp - 1) / kRcExp;
    const long long tiles = static_cast<long long>(prm.t_tiles) * prm.e_tiles;
    const long long stages = tiles * 8 * ((prm.J + kRcJc - 1) / kRcJc);
    if (tiles > 0x7fffffffll / kRcCluster || stages > 0x7fffffffll) return MOE_ERR_UNSUPPORTED;
    int ncl = dev >= 0 && dev < kMaxDevices ? max_clusters[dev] : 0;
    if (ncl <= 0) {
        // as many clusters as can be resident at once (one CTA per SM)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kRcCluster * 512);
        cfg.blockDim = dim3(kRcThreads);
        cfg.dynamicSmemBytes = kRcSmemBytes;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = kRcCluster;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&ncl, router_logits_rc_kernel, &cfg) != cudaSuccess || ncl <= 0) ncl = 64;
        if (dev >= 0 && dev < kMaxDevices) max_clusters[dev] = ncl;
    }
    const int grid = kRcCluster * static_cast<int>(tiles < ncl ? tiles : ncl);
    router_logits_rc_kernel<<<grid, kRcThreads, kRcSmemBytes, static_cast<cudaStream_t>(stream)>>>(tn, tw, prm);
    return launch_status();
}

moe_status_t moe_router_logits(const float* n, const float* router_w, const float* router_bias, int T, int H,
                               int E, float* logits, cwStream_t stream) {
    if (T < 0 || H <= 0 || H % 128 || E <= 0 || E > 256) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!n || !router_w || !logits || !aligned16(n) || !aligned16(router_w)) return MOE_ERR_INVALID_ARGUMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (H % 256) {
        // a hidden size that is an odd multiple of 128 (only small test shapes): one warp per logit
        const long long warps = static_cast<long long>(T) * E;
        if ((warps + 7) / 8 > 0x7fffffffll) return MOE_ERR_UNSUPPORTED;
        router_logits_warp_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, st>>>(n, router_w, router_bias,
                                                                                          T, H, E, logits);
        return launch_status();
    }
    CUtensorMap tn, tw;
    if (!encode_rt_map(&tn, n, T, H, kRtTok) || !encode_rt_map(&tw, router_w, E, H, kRtExp)) return MOE_ERR_CUDA;
    static bool attr[kMaxDevices] = {};
    static int max_clusters[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
    if (smem_optin_once(router_logits_ref_kernel, static_cast<int>(kRtSmemBytes), attr) != cudaSuccess)
        return MOE_ERR_CUDA;
    RtParams prm;
    prm.bias = router_bias;
    prm.logits = logits;
    prm.T = T;
    prm.E = E;
    prm.J = H / 256;
    prm.t_tiles = (T + kRtTok - 1) / kRtTok;
    prm.e_tiles = (E + kRtExp - 1) / kRtExp;
    const long long tiles = static_cast<long long>(prm.t_tiles) * prm.e_tiles;
    if (tiles > 0x7fffffffll / kRtCluster) return MOE_ERR_UNSUPPORTED;
    int ncl = dev >= 0 && dev < kMaxDevices ? max_clusters[dev] : 0;
    if (ncl <= 0) {
        // as many clusters as can be resident at once (one CTA per SM)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kRtCluster * 512);
        cfg.blockDim = dim3(kRtThreads);
        cfg.dynamicSmemBytes = kRtSmemBytes;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = kRtCluster;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&ncl, router_logits_ref_kernel, &cfg) != cudaSuccess || ncl <= 0) ncl = 32;
        if (dev >= 0 && dev < kMaxDevices) max_clusters[dev] = ncl;
    }
    const int grid = kRtCluster * static_cast<int>(tiles < ncl ? tiles : ncl);
    router_logits_ref_kernel<<<grid, kRtThreads, kRtSmemBytes, st>>>(tn, tw, prm);
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
    if (T < 0 || H <= 0 || H % 128 || E <= 0 || E > 256 || k <= 0 || k > 16 || k > E) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!x_bf16 || !rms || !gamma || !router_w || !topk_idx || !topk_w) return MOE_ERR_INVALID_ARGUMENT;
    const size_t smem = static_cast<size_t>(H + E) * sizeof(float);
    if (smem > 200 * 1024) return MOE_ERR_UNSUPPORTED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x_bf16);
    static bool attr[8][kMaxDevices] = {};
#define TB_ROUTER(EPTV)                                                                                        \
    do {                                                                                                       \
        if (smem_optin_once(router_topk_kernel<EPTV>, 200 * 1024, attr[EPTV - 1]) != cudaSuccess)              \
            return MOE_ERR_CUDA;                                                                               \
        router_topk_kernel<EPTV><<<T, 256, smem, s>>>(xb, rms, gamma, router_w, router_bias, T, H, E, k,       \
                                                      logits_out, topk_idx, topk_w);                           \
    } while (0)
    switch ((E + 31) / 32) {
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

moe_status_t moe_gather_rows_x2(const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                                const int32_t* row_token, const int32_t* total_rows, int row_capacity, int H,
                                void* xp, void* xp_lo, float* xps, int xps_ld, cwStream_t stream) {
    if (H <= 0 || H % 128 || !xq || !xs || !row_token || !xp || !xps || row_capacity < 0 || xps_ld < row_capacity) return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(xq) || !aligned16(xp)) return MOE_ERR_INVALID_ARGUMENT;
    if (!xq_lo != !xp_lo || (xq_lo && (!aligned16(xq_lo) || !aligned16(xp_lo)))) return MOE_ERR_INVALID_ARGUMENT;
    if (row_capacity == 0) return MOE_OK;
    int blocks = (row_capacity + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    gather_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(xq), xs, xs_ld, row_token, total_rows, row_capacity, H,
        static_cast<uint8_t*>(xp), xps, xps_ld, static_cast<const uint8_t*>(xq_lo), static_cast<uint8_t*>(xp_lo));
    return launch_status();
}

moe_status_t moe_scatter_rows_x2(const void* xq, const void* xq_lo, const float* xs, int xs_ld, const int32_t* pos,
                                 int T, int k, const int32_t* shared_start, int num_shared, const int32_t* row_token,
                                 const int32_t* total_rows, int row_capacity, int H, void* xp, void* xp_lo, float* xps,
                                 int xps_ld, cwStream_t stream) {
    if (H <= 0 || H % 128 || T < 0 || k <= 0 || k > kScatterMaxK || num_shared < 0 || num_shared > kScatterMaxShared ||
        row_capacity < 0 || xps_ld < row_capacity)
        return MOE_ERR_INVALID_ARGUMENT;
    if (!xq || !xs || !row_token || !total_rows || !xp || !xps || (T > 0 && !pos) || (num_shared > 0 && !shared_start))
        return MOE_ERR_INVALID_ARGUMENT;
    if (!aligned16(xq) || !aligned16(xp)) return MOE_ERR_INVALID_ARGUMENT;
    if (!xq_lo != !xp_lo || (xq_lo && (!aligned16(xq_lo) || !aligned16(xp_lo)))) return MOE_ERR_INVALID_ARGUMENT;
    if (row_capacity == 0) return MOE_OK;
    long long blocks = (static_cast<long long>(T) + 7) / 8;
    const long long pad_blocks = (static_cast<long long>(row_capacity) + 255) / 256;
    if (blocks < pad_blocks) blocks = pad_blocks;
    if (blocks > 148 * 16) blocks = 148 * 16;
    scatter_rows_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(xq), xs, xs_ld, pos, T, k, shared_start, num_shared, row_token, total_rows,
        row_capacity, H, static_cast<uint8_t*>(xp), xps, xps_ld, static_cast<const uint8_t*>(xq_lo),
        static_cast<uint8_t*>(xp_lo));
    return launch_status();
}

moe_status_t moe_gather_rows_n(const void* xq, const float* xs, int xs_ld, const int32_t* row_token,
                               const int32_t* total_rows, int row_capacity, int H, void* xp, float* xps,
                               int xps_ld, cwStream_t stream) {
    return moe_gather_rows_x2(xq, nullptr, xs, xs_ld, row_token, total_rows, row_capacity, H, xp, nullptr, xps,
                              xps_ld, stream);
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

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry-point query (this library
// links only the runtime); null when the driver does not offer it.
CtxGetCurrentFn ctx_get_current_fn() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    return fn;
}

// The array's device address, looked up once per device with that device
// current (host code cannot use the array's name as a device pointer).  The
// cache entry remembers the context it was looked up in: after a
// cudaDeviceReset the device gets a new primary context, the module is loaded
// again, and the address is looked up again instead of reusing the old one.
float* router_scratch_address(moe_status_t* status) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static float* addr[kMaxDevices] = {};
    static CUcontext ctx_of[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *status = MOE_ERR_CUDA;
        return nullptr;
    }
    // make the device's primary context current before asking which it is
    if (cudaFree(nullptr) != cudaSuccess) {
        *status = MOE_ERR_CUDA;
        return nullptr;
    }
    CUcontext ctx = nullptr;
    CtxGetCurrentFn get = ctx_get_current_fn();
    if (get && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev] || ctx_of[dev] != ctx) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_router_logits_scratch) != cudaSuccess || !p) {
            *status = MOE_ERR_CUDA;
            return nullptr;
        }
        addr[dev] = static_cast<float*>(p);
        ctx_of[dev] = ctx;
    }
    *status = MOE_OK;
    return addr[dev];
}

}  // namespace

extern "C" moe_status_t moe_router_topk_noalloc(const float* n, const float* router_w, const float* router_bias,
                                                int T, int H, int E, int k, int32_t* topk_idx, float* topk_w,
                                                cwStream_t stream) {
    // every argument check of the two kernels comes first, so a refused call launches nothing
    if (T < 0 || H <= 0 || H % 128 || E <= 0 || E > 256 || k <= 0 || k > 16 || k > E) return MOE_ERR_INVALID_ARGUMENT;
    if (static_cast<long long>(T) * E > kNoAllocLogits) return MOE_ERR_WORKSPACE;   // beyond the fixed array
    if (T == 0) return MOE_OK;
    if (!n || !router_w || !topk_idx || !topk_w || !aligned16(n) || !aligned16(router_w))
        return MOE_ERR_INVALID_ARGUMENT;
    moe_status_t st = MOE_OK;
    float* logits = router_scratch_address(&st);
    if (!logits) return st;
    // every logit the top-k reads is written first: nothing needs clearing
    st = moe_router_logits(n, router_w, router_bias, T, H, E, logits, stream);
    if (st != MOE_OK) return st;
    return moe_topk_softmax(logits, T, E, k, topk_idx, topk_w, stream);
}
