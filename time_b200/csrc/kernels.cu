// kernels.cu -- the 20 launch_* entry points of the reference engine's
// libkernels (csrc/kernels.h:12-31), rewritten for sm_100a.
//
// Numerics kept bit-for-bit with the reference kernels where the engine can
// observe them: E4M3 decode/encode (csrc/kernels.cu:7-45), the RMSNorm and
// router-logit reduction order (csrc/kernels.cu:61-85, 412-435), top-k
// tie-breaking and weights (csrc/kernels.cu:437-471), RoPE formula
// (csrc/kernels.cu:87-108), combine (csrc/kernels.cu:484-496) and the
// sequential CDF of top-p sampling (csrc/kernels.cu:236-262).  Layout: the
// reference's fp32 row-major buffers.  Work is spread over warps instead of
// the reference's single-thread loops; elementwise kernels are 16-byte
// vectorised grid-stride loops sized to the SM count.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cfloat>
#include <cstdint>

#include "kernels.h"
#include "sampling.cuh"

namespace {

using tb::warp_argmax_first;
using tb::warp_top_p;

thread_local int g_last_error = 0;

inline void record(cudaError_t e) { g_last_error = static_cast<int>(e); }
inline void record_launch() { record(cudaGetLastError()); }

inline int grid_for(size_t work, int per_block) {
    size_t b = (work + per_block - 1) / per_block;
    const size_t cap = 148 * 32;
    if (b > cap) b = cap;
    if (b == 0) b = 1;
    return static_cast<int>(b);
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// csrc/kernels.cu:7-26 (NaN code -> 0), built from the bit fields.
__device__ __forceinline__ float e4m3_decode_ref(uint32_t bits) {
    const uint32_t sign = (bits >> 7) & 1u, ex = (bits >> 3) & 0xFu, mant = bits & 7u;
    float v;
    if (ex == 0) v = static_cast<float>(mant) * 0.001953125f;       // mant * 2^-9, exact
    else if (ex == 15 && mant == 7) v = 0.0f;
    else v = __uint_as_float(((ex + 120u) << 23) | (mant << 20));   // (1 + m/8) * 2^(e-7)
    return sign ? -v : v;
}

// csrc/kernels.cu:28-45, same operations (log2f/floorf/powf/roundf).
__device__ __forceinline__ uint8_t e4m3_encode_ref(float x) {
    const int sign = (x < 0.0f) ? 1 : 0;
    const float ax = fabsf(x);
    if (isnan(x)) return 0x7F;
    if (ax == 0.0f) return static_cast<uint8_t>(sign << 7);
    if (ax >= 448.0f) return static_cast<uint8_t>((sign << 7) | 0x7E);
    if (ax < powf(2.0f, -9.0f)) return static_cast<uint8_t>(sign << 7);
    const float l2 = log2f(ax);
    int e = static_cast<int>(floorf(l2));
    if (e < -6) e = -6;
    if (e > 8) e = 8;
    const float m = ax / powf(2.0f, static_cast<float>(e)) - 1.0f;
    int mant = static_cast<int>(roundf(m * 8.0f));
    if (mant < 0) mant = 0;
    if (mant > 7) mant = 7;
    return static_cast<uint8_t>((sign << 7) | ((e + 7) << 3) | mant);
}

// ---------------------------------------------------------------- elementwise

__global__ void fp8_dequant_kernel(const uint8_t* __restrict__ in, float* __restrict__ out, size_t n, bool vec) {
    const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    if (vec) {
        const size_t n4 = n / 4;
        for (size_t i = tid; i < n4; i += stride) {
            const uint32_t w = reinterpret_cast<const uint32_t*>(in)[i];
            float4 o = make_float4(e4m3_decode_ref(w & 0xFF), e4m3_decode_ref((w >> 8) & 0xFF),
                                   e4m3_decode_ref((w >> 16) & 0xFF), e4m3_decode_ref(w >> 24));
            reinterpret_cast<float4*>(out)[i] = o;
        }
        for (size_t i = n4 * 4 + tid; i < n; i += stride) out[i] = e4m3_decode_ref(in[i]);
    } else {
        for (size_t i = tid; i < n; i += stride) out[i] = e4m3_decode_ref(in[i]);
    }
}

__global__ void f32_to_fp8_kernel(const float* __restrict__ in, uint8_t* __restrict__ out, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
        out[i] = e4m3_encode_ref(in[i]);
}

__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ o, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
        const float gv = g[i];
        const float s = gv / (1.0f + expf(-gv));
        o[i] = s * u[i];
    }
}

__global__ void gelu_kernel(float* __restrict__ d, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
        const float x = d[i];
        d[i] = 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
    }
}

__global__ void add_kernel(float* __restrict__ a, const float* __restrict__ b, size_t n, bool vec) {
    const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    size_t done = 0;
    if (vec) {
        const size_t n4 = n / 4;
        for (size_t i = tid; i < n4; i += stride) {
            float4 x = reinterpret_cast<float4*>(a)[i];
            const float4 y = reinterpret_cast<const float4*>(b)[i];
            x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
            reinterpret_cast<float4*>(a)[i] = x;
        }
        done = n4 * 4;
    }
    for (size_t i = done + tid; i < n; i += stride) a[i] += b[i];
}

__global__ void copy_kernel(const float* __restrict__ s, float* __restrict__ d, size_t n, bool vec) {
    const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    size_t done = 0;
    if (vec) {
        const size_t n4 = n / 4;
        for (size_t i = tid; i < n4; i += stride) reinterpret_cast<float4*>(d)[i] = reinterpret_cast<const float4*>(s)[i];
        done = n4 * 4;
    }
    for (size_t i = done + tid; i < n; i += stride) d[i] = s[i];
}

// ---------------------------------------------------------------- row reductions

// Reference-order sum of products of one row (256 strided fma partials + tree),
// csrc/kernels.cu:67-79 / 420-431, by one warp (lane owns partials l + 32m).
__device__ __forceinline__ float warp_dot_ref_order(const float* a, const float* b, int n, int lane) {
    float p[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) p[m] = 0.0f;
    for (int j = 0; j < n; j += 256) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int i = j + 32 * m + lane;
            if (i < n) p[m] = __fmaf_rn(a[i], b[i], p[m]);
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

__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ gamma, float* __restrict__ out,
                                int H, int rows, float eps) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + static_cast<size_t>(row) * H;
    const float ss = warp_dot_ref_order(xr, xr, H, lane);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(H)), eps));
    float* o = out + static_cast<size_t>(row) * H;
    for (int i = lane; i < H; i += 32) o[i] = __fmul_rn(__fdiv_rn(xr[i], rms), gamma[i]);
}

__global__ void moe_gate_kernel(const float* __restrict__ h, const float* __restrict__ w, float* __restrict__ logits,
                                int H, int E, int T) {
    const long long pair = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (pair >= static_cast<long long>(T) * E) return;
    const int t = static_cast<int>(pair / E), e = static_cast<int>(pair % E);
    const float v = warp_dot_ref_order(h + static_cast<size_t>(t) * H, w + static_cast<size_t>(e) * H, H, lane);
    if (lane == 0) logits[static_cast<size_t>(t) * E + e] = v;
}

// csrc/kernels.cu:437-471 semantics, one warp per token.
__global__ void moe_topk_kernel(const float* __restrict__ logits, int32_t* __restrict__ idx, float* __restrict__ wts,
                                int E, int K, int T) {
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const float* lg = logits + static_cast<size_t>(t) * E;
    const int kk = K < 16 ? K : 16;
    float sel_v[16];
    int sel_i[16];
    // selection by repeated arg-max: value descending, lower index first, values
    // not strictly greater than -FLT_MAX (incl. NaN) never selected
    int last_i = -1;
    float last_v = INFINITY;
    for (int s = 0; s < kk; ++s) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            float v = lg[e];
            if (!(v > -FLT_MAX)) continue;
            // strictly after (last_v, last_i) in (value desc, index asc) order
            const bool after = (v < last_v) || (v == last_v && e > last_i);
            if (!after) continue;
            if (v > bv || (v == bv && e < bi)) { bv = v; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (bi == 0x7fffffff) {
            for (int r = s; r < kk; ++r) { sel_v[r] = -FLT_MAX; sel_i[r] = -1; }
            break;
        }
        sel_v[s] = bv;
        sel_i[s] = bi;
        last_v = bv;
        last_i = bi;
    }
    if (lane == 0) {
        const float shift = (sel_v[0] > 80.0f) ? sel_v[0] : 0.0f;
        float sum = 0.0f;
        for (int s = 0; s < kk; ++s) sum += expf(sel_v[s] - shift);
        for (int s = 0; s < kk; ++s) {
            idx[static_cast<size_t>(t) * K + s] = sel_i[s];
            wts[static_cast<size_t>(t) * K + s] = expf(sel_v[s] - shift) / sum;
        }
    }
}

__global__ void moe_dispatch_kernel(const float* __restrict__ in, float* __restrict__ out, int H, int K, int T) {
    const int row = blockIdx.x;   // t * K + k
    if (row >= T * K) return;
    const float* src = in + static_cast<size_t>(row / K) * H;
    float* dst = out + static_cast<size_t>(row) * H;
    for (int d = threadIdx.x; d < H; d += blockDim.x) dst[d] = src[d];
}

__global__ void moe_combine_kernel(const float* __restrict__ y, const float* __restrict__ w, float* __restrict__ out,
                                   int H, int K, int T) {
    const int t = blockIdx.x;
    if (t >= T) return;
    for (int d = threadIdx.x; d < H; d += blockDim.x) {
        float acc = 0.0f;
        for (int k = 0; k < K; ++k)
            acc = __fmaf_rn(y[(static_cast<size_t>(t) * K + k) * H + d], w[static_cast<size_t>(t) * K + k], acc);
        out[static_cast<size_t>(t) * H + d] = acc;
    }
}

__global__ void softmax_kernel(float* __restrict__ data, int n) {
    float* row = data + static_cast<size_t>(blockIdx.x) * n;
    __shared__ float red[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float m = -FLT_MAX;
    for (int i = tid; i < n; i += blockDim.x) m = fmaxf(m, row[i]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (warp == 0) {
        m = lane < nw ? red[lane] : -FLT_MAX;
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red[0] = m;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    float s = 0.0f;
    for (int i = tid; i < n; i += blockDim.x) { const float e = expf(row[i] - m); row[i] = e; s += e; }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
        s = lane < nw ? red[lane] : 0.0f;
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) red[0] = s;
    }
    __syncthreads();
    s = red[0];
    for (int i = tid; i < n; i += blockDim.x) row[i] /= s;
}

__global__ void rope_kernel(float* __restrict__ q, float* __restrict__ k, int hd, int nh, int seq, int start, float theta) {
    const int si = blockIdx.x, hi = blockIdx.y;
    const int pos = start + si;
    float* qh = q + (static_cast<size_t>(si) * nh + hi) * hd;
    float* kh = k + (static_cast<size_t>(si) * nh + hi) * hd;
    const int half = hd / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float freq = 1.0f / powf(theta, static_cast<float>(2 * i) / static_cast<float>(hd));
        const float ang = freq * static_cast<float>(pos);
        const float c = cosf(ang), s = sinf(ang);
        const float q0 = qh[i], q1 = qh[i + half];
        qh[i] = q0 * c - q1 * s;
        qh[i + half] = q0 * s + q1 * c;
        const float k0 = kh[i], k1 = kh[i + half];
        kh[i] = k0 * c - k1 * s;
        kh[i + half] = k0 * s + k1 * c;
    }
}

template <typename T>
__device__ __forceinline__ float load_embed(const T* p);
template <> __device__ __forceinline__ float load_embed<uint8_t>(const uint8_t* p) { return e4m3_decode_ref(*p); }
template <> __device__ __forceinline__ float load_embed<__half>(const __half* p) { return __half2float(*p); }
template <> __device__ __forceinline__ float load_embed<float>(const float* p) { return *p; }

template <typename T>
__global__ void embedding_kernel(const T* __restrict__ table, const int64_t* __restrict__ ids, float* __restrict__ out,
                                 int H, int n) {
    const int t = blockIdx.x;
    if (t >= n) return;
    const T* row = table + static_cast<size_t>(ids[t]) * H;
    float* o = out + static_cast<size_t>(t) * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = load_embed<T>(row + i);
}

__global__ void argmax_kernel(const float* __restrict__ logits, int64_t* __restrict__ out, int V, int B) {
    const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= B) return;
    const int i = warp_argmax_first(logits + static_cast<size_t>(b) * V, V, lane);
    if (lane == 0) out[b] = i;
}

__global__ void top_p_kernel(const float* __restrict__ logits, int64_t* __restrict__ out, float temperature,
                             float top_p, int V, int B, const uint64_t* __restrict__ seeds) {
    const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= B) return;
    const int i = warp_top_p(logits + static_cast<size_t>(b) * V, V, temperature, top_p, seeds[b], lane);
    if (lane == 0) out[b] = i;
}

// Each distinct past token's logit is penalised once (the reference's
// unsynchronised threads give that result whenever duplicates do not race).
__global__ void rep_penalty_kernel(float* __restrict__ logits, const int64_t* __restrict__ past, int n, int V, float pen) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int64_t tok = past[i];
        if (tok < 0 || tok >= V) continue;
        bool first = true;
        for (int j = 0; j < i; ++j)
            if (past[j] == tok) { first = false; break; }
        if (!first) continue;
        const float v = logits[tok];
        logits[tok] = (v > 0.0f) ? v / pen : v * pen;
    }
}

// Causal attention over the current chunk, q/k/v [seq][heads][d]: one warp
// per (query, head), online softmax over keys 0..i, d <= 256.
__global__ void attn_prefill_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                    float* __restrict__ out, int nh, int hd, int seq, float scale) {
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= seq * nh) return;
    const int i = wid / nh, h = wid % nh;
    const float* qh = q + (static_cast<size_t>(i) * nh + h) * hd;
    float qv[8], acc[8];
    for (int r = 0; r < 8; ++r) { const int d = lane + 32 * r; qv[r] = d < hd ? qh[d] : 0.0f; acc[r] = 0.0f; }
    float mrun = -INFINITY, l = 0.0f;
    for (int j = 0; j <= i; ++j) {
        const float* kh = k + (static_cast<size_t>(j) * nh + h) * hd;
        float dot = 0.0f;
        for (int r = 0; r < 8; ++r) { const int d = lane + 32 * r; if (d < hd) dot += qv[r] * kh[d]; }
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float s = dot * scale;
        const float mnew = fmaxf(mrun, s);
        const float corr = expf(mrun - mnew), p = expf(s - mnew);
        l = l * corr + p;
        const float* vh = v + (static_cast<size_t>(j) * nh + h) * hd;
        for (int r = 0; r < 8; ++r) { const int d = lane + 32 * r; if (d < hd) acc[r] = acc[r] * corr + p * vh[d]; }
        mrun = mnew;
    }
    float* oh = out + (static_cast<size_t>(i) * nh + h) * hd;
    for (int r = 0; r < 8; ++r) { const int d = lane + 32 * r; if (d < hd) oh[d] = acc[r] / l; }
}

// Single-query paged GQA attention: block per head, 4 warps split the
// positions, online softmax per warp, merged through shared memory.
__global__ void attn_decode_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                                   float* __restrict__ out, const int32_t* __restrict__ pt, int page_size, int nh, int nkv,
                                   int hd, int past, float scale) {
    const int h = blockIdx.x;
    if (h >= nh) return;
    const int kvh = h / (nh / nkv);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float* qh = q + static_cast<size_t>(h) * hd;
    float qv[8], acc[8];
    for (int r = 0; r < 8; ++r) { const int d = lane + 32 * r; qv[r] = d < hd ? qh[d] : 0.0f; acc[r] = 0.0f; }
    float mrun = -INFINITY, l = 0.0f;
    for (int p = warp; p < past; p += nw) {
        const int page = pt[p / page_size], off = p % page_size;
        const size_t base = (static_cast<size_t>(page) * page_size + off) * nkv * hd + static_cast<size_t>(kvh) * hd;
        float dot = 0.0f;
        for (int r = 0; r < 8; ++r) { const int d = lane + 32 * r; if (d < hd) dot += qv[r] * kc[base + d]; }
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float s = dot * scale;
        const float mnew = fmaxf(mrun, s);
        const float corr = expf(mrun - mnew), pr = expf(s - mnew);
        l = l * corr + pr;
        for (int r = 0; r < 8; ++r) { const int d = lane + 32 * r; if (d < hd) acc[r] = acc[r] * corr + pr * vc[base + d]; }
        mrun = mnew;
    }
    __shared__ float sm[4], sl[4];
    __shared__ float sacc[4][256];
    if (lane == 0) { sm[warp] = mrun; sl[warp] = l; }
    for (int r = 0; r < 8; ++r) { const int d = lane + 32 * r; if (d < hd) sacc[warp][d] = acc[r]; }
    __syncthreads();
    float M = -INFINITY;
    for (int w = 0; w < nw; ++w) M = fmaxf(M, sm[w]);
    float L = 0.0f;
    for (int w = 0; w < nw; ++w) if (sm[w] > -INFINITY) L += sl[w] * expf(sm[w] - M);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float o = 0.0f;
        for (int w = 0; w < nw; ++w) if (sm[w] > -INFINITY) o += sacc[w][d] * expf(sm[w] - M);
        out[static_cast<size_t>(h) * hd + d] = (L > 0.0f) ? o / L : 0.0f;
    }
}

__global__ void update_kv_kernel(const float* __restrict__ k, const float* __restrict__ v, float* __restrict__ kc,
                                 float* __restrict__ vc, const int32_t* __restrict__ pt, int page_size, int nkv, int hd,
                                 int seq, int start) {
    const int si = blockIdx.x, kh = blockIdx.y;
    if (si >= seq || kh >= nkv) return;
    const int pos = start + si;
    const int page = pt[pos / page_size], off = pos % page_size;
    const size_t src = (static_cast<size_t>(si) * nkv + kh) * hd;
    const size_t dst = (static_cast<size_t>(page) * page_size + off) * nkv * hd + static_cast<size_t>(kh) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) { kc[dst + d] = k[src + d]; vc[dst + d] = v[src + d]; }
}

}  // namespace

extern "C" {

int kernels_last_error(void) { return g_last_error; }

void launch_fp8_dequantize(const void* input, void* output, size_t count, cwStream_t stream) {
    if (count == 0) { record(cudaSuccess); return; }
    const bool vec = aligned(input, 4) && aligned(output, 16);
    fp8_dequant_kernel<<<grid_for(count / 4 + 1, 256), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t*>(input), static_cast<float*>(output), count, vec);
    record_launch();
}

void launch_f32_to_fp8(const float* input, void* output, size_t count, cwStream_t stream) {
    if (count == 0) { record(cudaSuccess); return; }
    f32_to_fp8_kernel<<<grid_for(count, 256), 256, 0, (cudaStream_t)stream>>>(input, static_cast<uint8_t*>(output), count);
    record_launch();
}

void launch_rms_norm(const float* input, const float* gamma, float* output, int hidden_dim, int batch_size, float eps,
                     cwStream_t stream) {
    if (batch_size <= 0 || hidden_dim <= 0) { record(cudaSuccess); return; }
    rms_norm_kernel<<<(batch_size + 7) / 8, 256, 0, (cudaStream_t)stream>>>(input, gamma, output, hidden_dim, batch_size, eps);
    record_launch();
}

void launch_rope(float* q, float* k, int head_dim, int num_heads, int seq_len, int start_pos, float theta, cwStream_t stream) {
    if (seq_len <= 0 || num_heads <= 0) { record(cudaSuccess); return; }
    dim3 grid(seq_len, num_heads);
    rope_kernel<<<grid, 64, 0, (cudaStream_t)stream>>>(q, k, head_dim, num_heads, seq_len, start_pos, theta);
    record_launch();
}

void launch_softmax(float* input, int batch_size, int seq_len, cwStream_t stream) {
    if (batch_size <= 0 || seq_len <= 0) { record(cudaSuccess); return; }
    softmax_kernel<<<batch_size, 256, 0, (cudaStream_t)stream>>>(input, seq_len);
    record_launch();
}

void launch_swiglu(const float* gate, const float* up, float* output, size_t count, cwStream_t stream) {
    if (count == 0) { record(cudaSuccess); return; }
    swiglu_kernel<<<grid_for(count, 256), 256, 0, (cudaStream_t)stream>>>(gate, up, output, count);
    record_launch();
}

void launch_gelu(float* data, size_t count, cwStream_t stream) {
    if (count == 0) { record(cudaSuccess); return; }
    gelu_kernel<<<grid_for(count, 256), 256, 0, (cudaStream_t)stream>>>(data, count);
    record_launch();
}

void launch_embedding_lookup(const void* embedding_table, const int64_t* token_ids, float* output, int hidden_dim,
                             int num_tokens, int dtype, cwStream_t stream) {
    if (num_tokens <= 0) { record(cudaSuccess); return; }
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == 1)
        embedding_kernel<uint8_t><<<num_tokens, 256, 0, s>>>(static_cast<const uint8_t*>(embedding_table), token_ids, output, hidden_dim, num_tokens);
    else if (dtype == 2)
        embedding_kernel<__half><<<num_tokens, 256, 0, s>>>(static_cast<const __half*>(embedding_table), token_ids, output, hidden_dim, num_tokens);
    else
        embedding_kernel<float><<<num_tokens, 256, 0, s>>>(static_cast<const float*>(embedding_table), token_ids, output, hidden_dim, num_tokens);
    record_launch();
}

void launch_add_residual(float* a, const float* b, size_t count, cwStream_t stream) {
    if (count == 0) { record(cudaSuccess); return; }
    const bool vec = aligned(a, 16) && aligned(b, 16);
    add_kernel<<<grid_for(count / 4 + 1, 256), 256, 0, (cudaStream_t)stream>>>(a, b, count, vec);
    record_launch();
}

void launch_argmax(const float* logits, int64_t* output, int vocab_size, int batch_size, cwStream_t stream) {
    if (batch_size <= 0 || vocab_size <= 0) { record(cudaSuccess); return; }
    argmax_kernel<<<(batch_size + 3) / 4, 128, 0, (cudaStream_t)stream>>>(logits, output, vocab_size, batch_size);
    record_launch();
}

void launch_top_p_sampling(const float* logits, int64_t* output, float temperature, float top_p, int vocab_size,
                           int batch_size, const uint64_t* random_seeds, cwStream_t stream) {
    if (batch_size <= 0 || vocab_size <= 0) { record(cudaSuccess); return; }
    if (temperature < 0.01f)
        argmax_kernel<<<(batch_size + 3) / 4, 128, 0, (cudaStream_t)stream>>>(logits, output, vocab_size, batch_size);
    else
        top_p_kernel<<<(batch_size + 3) / 4, 128, 0, (cudaStream_t)stream>>>(logits, output, temperature, top_p, vocab_size,
                                                                            batch_size, random_seeds);
    record_launch();
}

void launch_apply_rep_penalty(float* logits, const int64_t* past_tokens, int past_len, int vocab_size, float penalty,
                              cwStream_t stream) {
    if (past_len <= 0) { record(cudaSuccess); return; }
    rep_penalty_kernel<<<(past_len + 255) / 256, 256, 0, (cudaStream_t)stream>>>(logits, past_tokens, past_len, vocab_size, penalty);
    record_launch();
}

void launch_paged_attention_prefill(const float* q, const float* k, const float* v, float* output, const int32_t* page_table,
                                    int num_pages, int page_size, int num_heads, int head_dim, int seq_len, float scale,
                                    cwStream_t stream) {
    (void)page_table; (void)num_pages; (void)page_size;
    if (seq_len <= 0 || num_heads <= 0 || head_dim <= 0 || head_dim > 256) { record(seq_len <= 0 ? cudaSuccess : cudaErrorInvalidValue); return; }
    const long long warps = static_cast<long long>(seq_len) * num_heads;
    attn_prefill_kernel<<<static_cast<unsigned>((warps + 3) / 4), 128, 0, (cudaStream_t)stream>>>(q, k, v, output, num_heads, head_dim, seq_len, scale);
    record_launch();
}

void launch_paged_attention_decode(const float* q, const float* kv_cache_k, const float* kv_cache_v, float* output,
                                   const int32_t* page_table, int num_pages, int page_size, int num_heads, int num_kv_heads,
                                   int head_dim, int past_len, float scale, cwStream_t stream) {
    (void)num_pages;
    if (num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || head_dim > 256 || num_heads % num_kv_heads) {
        record(cudaErrorInvalidValue);
        return;
    }
    attn_decode_kernel<<<num_heads, 128, 0, (cudaStream_t)stream>>>(q, kv_cache_k, kv_cache_v, output, page_table, page_size,
                                                                     num_heads, num_kv_heads, head_dim, past_len, scale);
    record_launch();
}

void launch_update_kv_cache(const float* k, const float* v, float* kv_cache_k, float* kv_cache_v, const int32_t* page_table,
                            int page_size, int num_kv_heads, int head_dim, int seq_len, int start_pos, cwStream_t stream) {
    if (seq_len <= 0 || num_kv_heads <= 0) { record(cudaSuccess); return; }
    dim3 grid(seq_len, num_kv_heads);
    update_kv_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>(k, v, kv_cache_k, kv_cache_v, page_table, page_size, num_kv_heads,
                                                              head_dim, seq_len, start_pos);
    record_launch();
}

void launch_moe_gate(const float* hidden, const void* gate_weight, float* router_logits, int hidden_dim, int num_experts,
                     int batch_size, int gate_dtype, cwStream_t stream) {
    (void)gate_dtype;
    if (batch_size <= 0 || num_experts <= 0) { record(cudaSuccess); return; }
    const long long warps = static_cast<long long>(batch_size) * num_experts;
    moe_gate_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
        hidden, static_cast<const float*>(gate_weight), router_logits, hidden_dim, num_experts, batch_size);
    record_launch();
}

void launch_moe_topk(const float* router_logits, int32_t* expert_indices, float* expert_weights, int num_experts, int top_k,
                     int batch_size, cwStream_t stream) {
    if (batch_size <= 0 || top_k <= 0) { record(cudaSuccess); return; }
    moe_topk_kernel<<<(batch_size + 3) / 4, 128, 0, (cudaStream_t)stream>>>(router_logits, expert_indices, expert_weights,
                                                                            num_experts, top_k, batch_size);
    record_launch();
}

void launch_moe_dispatch(const float* input, float* expert_inputs, const int32_t* expert_indices, int hidden_dim, int top_k,
                         int batch_size, cwStream_t stream) {
    (void)expert_indices;
    if (batch_size <= 0 || top_k <= 0) { record(cudaSuccess); return; }
    moe_dispatch_kernel<<<batch_size * top_k, 256, 0, (cudaStream_t)stream>>>(input, expert_inputs, hidden_dim, top_k, batch_size);
    record_launch();
}

void launch_moe_combine(const float* expert_outputs, const float* expert_weights, float* output, int hidden_dim, int top_k,
                        int batch_size, cwStream_t stream) {
    if (batch_size <= 0) { record(cudaSuccess); return; }
    moe_combine_kernel<<<batch_size, 256, 0, (cudaStream_t)stream>>>(expert_outputs, expert_weights, output, hidden_dim, top_k,
                                                                     batch_size);
    record_launch();
}

void launch_copy_hidden(const float* src, float* dst, size_t count, cwStream_t stream) {
    if (count == 0) { record(cudaSuccess); return; }
    const bool vec = aligned(src, 16) && aligned(dst, 16);
    copy_kernel<<<grid_for(count / 4 + 1, 256), 256, 0, (cudaStream_t)stream>>>(src, dst, count, vec);
    record_launch();
}

}  // extern "C"
