// engine_kernels.h -- launchers of engine_kernels.cu (internal to engine.so).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace tb_engine {

// out bf16 [R][H] = table bf16 [V][H] rows ids[r]; H % 8 == 0.
cudaError_t embed_rows(const void* table, const int64_t* ids, int R, int V, int H, void* out, int* error_word,
                       cudaStream_t st);
// out bf16 [R][H] = RMSNorm(x bf16 [R][H]) * gamma.
cudaError_t final_norm_rows(const void* x, const float* gamma, int R, int H, float eps, void* out, cudaStream_t st);
// out[r] = the token sampled from logits fp32 [R][V] row r.
cudaError_t sample_rows(const float* logits, int R, int V, const float* temperature, const float* top_p,
                        const uint64_t* seeds, int64_t* out, cudaStream_t st);

}  // namespace tb_engine
