// engine_kernels.cu -- the serving engine's own kernels around the layers:
//
//   embedding gather   bf16 table rows -> bf16 hidden rows (16-byte copies)
//   final RMSNorm      bf16 rows -> bf16 rows for the lm_head GEMM
//   batched sampler    one warp per row: greedy or top-p with the row's own
//                      temperature, top_p and seed (sampling.cuh, the rules of
//                      the legacy launch_top_p_sampling)
//
// The reference engine embeds into fp32 (launch_embedding_lookup,
// src/terra/engine.t:1387) and samples one request per launch
// (engine.t:1446-1451); here a decode step embeds and samples every request of
// the batch in one launch each.
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cstdint>

#include "engine_kernels.h"
#include "sampling.cuh"

namespace {

// One block per row; a token id outside [0, V) gives a zero row and error 1.
__global__ void __launch_bounds__(128)
embed_kernel(const __nv_bfloat16* __restrict__ table, const int64_t* __restrict__ ids, int V, int H,
             __nv_bfloat16* __restrict__ out, int* __restrict__ error_word) {
    const int r = blockIdx.x;
    const int64_t id = ids[r];
    uint4* o = reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * H);
    const bool ok = id >= 0 && id < V;
    if (!ok && threadIdx.x == 0 && error_word) atomicExch(error_word, 1);
    const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(ok ? id : 0) * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) o[i] = ok ? src[i] : make_uint4(0, 0, 0, 0);
}

// out = bf16(x * rsqrt(mean(x^2) + eps) * gamma), one 256-thread block per row.
__global__ void __launch_bounds__(256)
final_norm_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma, int H, float eps,
                  __nv_bfloat16* __restrict__ out) {
    const int r = blockIdx.x;
    const __nv_bfloat16* xr = x + static_cast<size_t>(r) * H;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = __bfloat162float(xr[i]);
        ss += v * v;
    }
    __shared__ float red[8];
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float inv = rsqrtf(tot / static_cast<float>(H) + eps);
    __nv_bfloat16* orow = out + static_cast<size_t>(r) * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        orow[i] = __float2bfloat16_rn(__bfloat162float(xr[i]) * inv * gamma[i]);
}

__global__ void __launch_bounds__(128)
sample_kernel(const float* __restrict__ logits, int V, int R, const float* __restrict__ temperature,
              const float* __restrict__ top_p, const uint64_t* __restrict__ seeds, int64_t* __restrict__ out) {
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= R) return;
    const int i = tb::warp_sample(logits + static_cast<size_t>(r) * V, V, temperature[r], top_p[r], seeds[r], lane);
    if (lane == 0) out[r] = i;
}

inline cudaError_t last() { return cudaGetLastError(); }

}  // namespace

namespace tb_engine {

cudaError_t embed_rows(const void* table, const int64_t* ids, int R, int V, int H, void* out, int* error_word,
                       cudaStream_t st) {
    if (R <= 0) return cudaSuccess;
    embed_kernel<<<R, 128, 0, st>>>(static_cast<const __nv_bfloat16*>(table), ids, V, H,
                                    static_cast<__nv_bfloat16*>(out), error_word);
    return last();
}

cudaError_t final_norm_rows(const void* x, const float* gamma, int R, int H, float eps, void* out, cudaStream_t st) {
    if (R <= 0) return cudaSuccess;
    final_norm_kernel<<<R, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), gamma, H, eps,
                                         static_cast<__nv_bfloat16*>(out));
    return last();
}

cudaError_t sample_rows(const float* logits, int R, int V, const float* temperature, const float* top_p,
                        const uint64_t* seeds, int64_t* out, cudaStream_t st) {
    if (R <= 0) return cudaSuccess;
    sample_kernel<<<(R + 3) / 4, 128, 0, st>>>(logits, V, R, temperature, top_p, seeds, out);
    return last();
}

}  // namespace tb_engine
