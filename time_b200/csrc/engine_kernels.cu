// engine_kernels.cu -- the serving engine's own kernels around the layers:
//
//   embedding gather   bf16 table rows -> bf16 hidden rows (16-byte copies)
//   final RMSNorm      bf16 rows -> bf16 rows for the lm_head GEMM
//   batched sampler    one warp per row: greedy or top-p with the row's own
//                      temperature, top_p and seed (sampling.cuh, the rules of
//                      the legacy launch_top_p_sampling)
//   rows all-gather    several GPUs of one process: each rank stores its slice
//                      of rows into every rank's buffer (peer stores), the last
//                      block raises the rank's flag on every rank, and a wait
//                      kernel holds the stream until every rank's flag is up
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

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t gtimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// This rank's rows [off16, off16 + n16) (16-byte units) into every other
// rank's buffer; the last block to finish (all its puts fenced) raises
// flags[r][me] = ++epoch on every rank r.
__global__ void __launch_bounds__(256)
rows_allgather_kernel(const tb_engine::GatherSet G, const uint4* __restrict__ src, size_t off16, size_t n16,
                      uint32_t* __restrict__ epoch, unsigned int* __restrict__ done_blocks) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint4 v = src[off16 + i];
        for (int r = 0; r < G.world; ++r)
            if (r != G.me) static_cast<uint4*>(G.x[r])[off16 + i] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int prev = atomicAdd(done_blocks, 1u);
        if (prev == gridDim.x - 1) {
            *done_blocks = 0;
            const uint32_t e = *epoch + 1u;
            *epoch = e;
            __threadfence_system();
            for (int r = 0; r < G.world; ++r) st_release_sys(G.flags[r] + G.me, e);
        }
    }
}

// Until every rank's flag in this rank's array reaches this rank's epoch
// (bounded: error word 3 after timeout_ns).
__global__ void rows_allgather_wait_kernel(const tb_engine::GatherSet G, const uint32_t* __restrict__ epoch,
                                           unsigned long long timeout_ns, int* __restrict__ error_word) {
    if (threadIdx.x != 0) return;
    const uint32_t e = *epoch;
    const uint64_t t0 = gtimer_ns();
    for (int s = 0; s < G.world; ++s) {
        while (ld_acquire_sys(G.flags[G.me] + s) < e) {
            if (gtimer_ns() - t0 > timeout_ns) {
                if (error_word) atomicExch(error_word, 3);
                return;
            }
            __nanosleep(100);
        }
    }
}

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

cudaError_t rows_allgather(const GatherSet& G, const void* src, size_t row0, size_t rows, size_t H, uint32_t* epoch,
                           unsigned int* done_blocks, unsigned long long timeout_ns, int* error_word,
                           cudaStream_t st) {
    if (G.world < 1 || G.world > kMaxGatherRanks || G.me < 0 || G.me >= G.world || H % 8) return cudaErrorInvalidValue;
    const size_t off16 = row0 * H / 8, n16 = rows * H / 8;
    const int blocks = static_cast<int>(n16 == 0 ? 1 : (n16 + 255) / 256 < 1184 ? (n16 + 255) / 256 : 1184);
    rows_allgather_kernel<<<blocks, 256, 0, st>>>(G, static_cast<const uint4*>(src), off16, n16, epoch, done_blocks);
    if (last() != cudaSuccess) return cudaErrorLaunchFailure;
    rows_allgather_wait_kernel<<<1, 32, 0, st>>>(G, epoch, timeout_ns, error_word);
    return last();
}

}  // namespace tb_engine
