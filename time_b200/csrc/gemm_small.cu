// gemm_small.cu -- block-scaled FP8 projection for a few tokens (decode):
//
//   out[t][n] = bf16( sum_kb (sum_{k in kb} a[t][k] w[n][k]) * a_scale[kb][t] * w_scale[n/128][kb] )
//
// the 128x128-block-scaled product of the expert GEMM (kernels.fut:343-347)
// for T of at most a few hundred tokens, where a tile grid over N alone leaves
// most SMs idle (14 row blocks for the per-rank QKV of the attention block).
// The K blocks are split over the grid as well: a CTA owns 128 weight rows x
// 64 tokens x a run of K blocks, multiplies each 128-wide K block on mma.sync
// e4m3 tensor-core tiles (the accumulators live in registers, so the per-block
// scale promotion is an FMA per element), and writes an fp32 partial; a
// second kernel sums the splits in split order (deterministic) and rounds to
// bf16.  Operands are staged with cp.async into padded shared-memory rows
// (144 B: conflict-free ldmatrix).
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstdint>

#include "attn_block.h"
#include "sm100.cuh"

namespace {

using namespace tb;

constexpr int kRows = 128;        // weight rows per CTA
constexpr int kToks = 64;         // tokens per CTA
constexpr int kKB = 128;          // K block (scale granularity)
constexpr int kLd = kKB + 16;     // bytes per shared row
constexpr int kStages = 2;
constexpr int kStageBytes = (kRows + kToks) * kLd + kToks * 4;   // W rows, token rows, token scales
constexpr int kThreads = 128;
constexpr int kTargetCtas = 148;     // one wave: fewer splits, half the partial traffic

inline moe_status_t launch_status() {
    return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
// D = A (16x32 e4m3, row) * B (32x8 e4m3, col) + D, fp32
__device__ __forceinline__ void mma_e4m3(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 "
                 "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct Params {
    const uint8_t* a;       // [T][K]
    const float* a_scale;   // [K/128][a_ld]
    const uint8_t* w;       // [N][K]
    const float* w_scale;   // [N/128][K/128]
    float* part;            // [ksplit][T][N]
    __nv_bfloat16* out;     // [T][N] (ksplit == 1)
    int a_ld, T, N, K, kb_per;
};

// grid (N/128, ksplit, ceil(T/64)); warp w owns weight rows 32w..32w+31 of the
// CTA's block and all 64 tokens: 2 x 8 mma tiles.
__global__ void __launch_bounds__(kThreads, 2)
gemm_small_kernel(const Params p) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int nb = blockIdx.x, ks = blockIdx.y, tc = blockIdx.z;
    const int KB = p.K / kKB;
    const int kb0 = ks * p.kb_per, kb1 = min(KB, kb0 + p.kb_per);
    const int t0 = tc * kToks;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;

    auto load = [&](int kb, int stage) {
        uint8_t* st = sm + stage * kStageBytes;
        const uint8_t* wsrc = p.w + static_cast<size_t>(nb) * kRows * p.K + static_cast<size_t>(kb) * kKB;
        for (int c = threadIdx.x; c < kRows * (kKB / 16); c += kThreads) {
            const int r = c >> 3, q = c & 7;
            cp_async16(st + r * kLd + q * 16, wsrc + static_cast<size_t>(r) * p.K + q * 16, 16u);
        }
        uint8_t* ts = st + kRows * kLd;
        for (int c = threadIdx.x; c < kToks * (kKB / 16); c += kThreads) {
            const int r = c >> 3, q = c & 7;
            const int t = t0 + r;
            const uint8_t* src = p.a + static_cast<size_t>(t < p.T ? t : 0) * p.K + static_cast<size_t>(kb) * kKB + q * 16;
            cp_async16(ts + r * kLd + q * 16, src, t < p.T ? 16u : 0u);
        }
        float* sc = reinterpret_cast<float*>(ts + kToks * kLd);
        if (threadIdx.x < kToks / 4) {
            const int t = t0 + threadIdx.x * 4;
            const float* src = p.a_scale + static_cast<size_t>(kb) * p.a_ld + (t < p.T ? t : 0);
            cp_async16(sc + threadIdx.x * 4, src, t < p.T ? 16u : 0u);
        }
    };

    float acc[2][8][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < 8; ++n) acc[m][n][0] = acc[m][n][1] = acc[m][n][2] = acc[m][n][3] = 0.0f;

    const int nk = kb1 - kb0;
    load(kb0, 0);
    cp_async_commit();
    for (int i = 0; i < nk; ++i) {
        if (i + 1 < nk) load(kb0 + i + 1, (i + 1) % kStages);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const uint8_t* st = sm + (i % kStages) * kStageBytes;
        const uint8_t* ts = st + kRows * kLd;
        const float* sc = reinterpret_cast<const float*>(ts + kToks * kLd);
        float part[2][8][4];
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int n = 0; n < 8; ++n) part[m][n][0] = part[m][n][1] = part[m][n][2] = part[m][n][3] = 0.0f;
        const int mi = lane >> 3;
#pragma unroll
        for (int kk = 0; kk < kKB / 32; ++kk) {
            uint32_t af[2][4];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int row = warp * 32 + m * 16 + (lane & 7) + 8 * (mi & 1);
                ldsm_x4(smem_u32(st + row * kLd + kk * 32 + 16 * (mi >> 1)), af[m][0], af[m][1], af[m][2], af[m][3]);
            }
#pragma unroll
            for (int n = 0; n < 8; n += 2) {
                const int trow = n * 8 + (lane & 7) + 8 * (mi >> 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(smem_u32(ts + trow * kLd + kk * 32 + 16 * (mi & 1)), b0, b1, b2, b3);
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    mma_e4m3(part[m][n], af[m], b0, b1);
                    mma_e4m3(part[m][n + 1], af[m], b2, b3);
                }
            }
        }
        // promote: acc += part * (a_scale[t] * w_scale)
        const float sw = __ldg(p.w_scale + static_cast<size_t>(nb) * KB + kb0 + i);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const float c0 = sc[n * 8 + 2 * tq] * sw, c1 = sc[n * 8 + 2 * tq + 1] * sw;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                acc[m][n][0] = __fmaf_rn(part[m][n][0], c0, acc[m][n][0]);
                acc[m][n][1] = __fmaf_rn(part[m][n][1], c1, acc[m][n][1]);
                acc[m][n][2] = __fmaf_rn(part[m][n][2], c0, acc[m][n][2]);
                acc[m][n][3] = __fmaf_rn(part[m][n][3], c1, acc[m][n][3]);
            }
        }
        __syncthreads();   // the stage is reloaded next iteration
    }
    cp_async_wait<0>();
    __syncthreads();
    // transpose through shared memory: [64 tokens][128 rows] fp32
    float* tr = reinterpret_cast<float*>(sm);
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const int r = warp * 32 + m * 16 + g, t = n * 8 + 2 * tq;
            tr[t * kRows + r] = acc[m][n][0];
            tr[(t + 1) * kRows + r] = acc[m][n][1];
            tr[t * kRows + r + 8] = acc[m][n][2];
            tr[(t + 1) * kRows + r + 8] = acc[m][n][3];
        }
    __syncthreads();
    const int ntok = min(kToks, p.T - t0);
    for (int c = threadIdx.x; c < ntok * (kRows / 4); c += kThreads) {
        const int t = c / (kRows / 4), r4 = (c % (kRows / 4)) * 4;
        const float4 v = *reinterpret_cast<const float4*>(tr + t * kRows + r4);
        const size_t o = static_cast<size_t>(t0 + t) * p.N + static_cast<size_t>(nb) * kRows + r4;
        if (p.part) {
            *reinterpret_cast<float4*>(p.part + static_cast<size_t>(ks) * p.T * p.N + o) = v;
        } else {
            __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&lo);
            u.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(p.out + o) = u;
        }
    }
}

// out = bf16(sum over splits in split order)
__global__ void __launch_bounds__(256)
split_reduce_kernel(const float* __restrict__ part, int ksplit, size_t n, __nv_bfloat16* __restrict__ out) {
    const size_t i4 = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i4 >= n) return;
    float4 s = *reinterpret_cast<const float4*>(part + i4);
    // loads of a group issued together, then added in split order
    for (int k0 = 1; k0 < ksplit; k0 += 8) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (k0 + j < ksplit) v[j] = *reinterpret_cast<const float4*>(part + static_cast<size_t>(k0 + j) * n + i4);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (k0 + j < ksplit) { s.x += v[j].x; s.y += v[j].y; s.z += v[j].z; s.w += v[j].w; }
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(out + i4) = u;
}

void split_plan(int T, int N, int K, int* ksplit, int* kb_per) {
    const int KB = K / kKB;
    const int base = (N / kRows) * ((T + kToks - 1) / kToks);
    int want = (kTargetCtas + base - 1) / base;
    if (want < 1) want = 1;
    if (want > KB) want = KB;
    *kb_per = (KB + want - 1) / want;
    *ksplit = (KB + *kb_per - 1) / *kb_per;
}

}  // namespace

extern "C" {

size_t fp8_gemm_small_workspace_bytes(int T, int N, int K) {
    if (T <= 0 || N <= 0 || K <= 0 || N % kRows || K % kKB) return 0;
    int ks, per;
    split_plan(T, N, K, &ks, &per);
    return ks > 1 ? static_cast<size_t>(ks) * T * N * sizeof(float) : 0;
}

moe_status_t fp8_gemm_small(const void* a, const float* a_scale, int a_ld, int T, const void* w, const float* w_scale,
                            int N, int K, void* out_bf16, void* workspace, size_t workspace_bytes, cwStream_t stream) {
    if (T < 0 || N <= 0 || K <= 0 || N % kRows || K % kKB || a_ld < T || a_ld % 4) return MOE_ERR_INVALID_ARGUMENT;
    if (T == 0) return MOE_OK;
    if (!a || !a_scale || !w || !w_scale || !out_bf16) return MOE_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(a_scale) |
         reinterpret_cast<uintptr_t>(out_bf16)) & 15)
        return MOE_ERR_INVALID_ARGUMENT;
    int ks, per;
    split_plan(T, N, K, &ks, &per);
    const size_t need = ks > 1 ? static_cast<size_t>(ks) * T * N * sizeof(float) : 0;
    if (need && (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15)))
        return MOE_ERR_WORKSPACE;
    static bool attr[kMaxDevices] = {};
    const int smem = kStages * kStageBytes > kToks * kRows * 4 ? kStages * kStageBytes : kToks * kRows * 4;
    if (smem_optin_once(gemm_small_kernel, smem, attr) != cudaSuccess) return MOE_ERR_CUDA;
    Params p;
    p.a = static_cast<const uint8_t*>(a);
    p.a_scale = a_scale;
    p.w = static_cast<const uint8_t*>(w);
    p.w_scale = w_scale;
    p.part = ks > 1 ? static_cast<float*>(workspace) : nullptr;
    p.out = static_cast<__nv_bfloat16*>(out_bf16);
    p.a_ld = a_ld;
    p.T = T;
    p.N = N;
    p.K = K;
    p.kb_per = per;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid(N / kRows, ks, (T + kToks - 1) / kToks);
    if (grid.z > 65535) return MOE_ERR_UNSUPPORTED;
    gemm_small_kernel<<<grid, kThreads, smem, st>>>(p);
    moe_status_t s = launch_status();
    if (s != MOE_OK || ks == 1) return s;
    const size_t n = static_cast<size_t>(T) * N;
    split_reduce_kernel<<<static_cast<int>((n / 4 + 255) / 256), 256, 0, st>>>(p.part, ks, n, p.out);
    return launch_status();
}

}  // extern "C"
