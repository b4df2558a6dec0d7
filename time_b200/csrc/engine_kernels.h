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

// Several GPUs of one process: every rank's row buffer and flag array
// ([kMaxGatherRanks] uint32, zeroed at creation), as device pointers.
constexpr int kMaxGatherRanks = 8;
struct GatherSet {
    void* x[kMaxGatherRanks];
    uint32_t* flags[kMaxGatherRanks];
    int world, me;
};
// Rows [row0, row0 + rows) of bf16 [*][H] src (this rank's buffer G.x[G.me])
// into every rank's buffer at the same rows, then wait until every rank has
// put its rows (each rank passes its own slice; every rank calls it once per
// gather, in the same order).  epoch / done_blocks: this rank's device
// counters (zeroed at creation).  A wait past timeout_ns sets *error_word = 3.
cudaError_t rows_allgather(const GatherSet& G, const void* src, size_t row0, size_t rows, size_t H, uint32_t* epoch,
                           unsigned int* done_blocks, unsigned long long timeout_ns, int* error_word,
                           cudaStream_t st);

}  // namespace tb_engine
