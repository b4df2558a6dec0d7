// sampling.cuh -- per-row token selection shared by the legacy sampling
// entry points (kernels.cu) and the serving engine's batched sampler.  One
// warp per row of fp32 logits.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

namespace tb {

// First index of the maximum, reference semantics (csrc/kernels.cu:220-234:
// row[0] NaN -> 0; NaN never wins).
__device__ __forceinline__ int warp_argmax_first(const float* row, int V, int lane) {
    const float r0 = row[0];
    if (isnan(r0)) return 0;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = lane; i < V; i += 32) {
        const float v = row[i];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    return (bi == 0x7fffffff) ? 0 : bi;
}

// csrc/kernels.cu:236-262: max, sum of exp((l - max)/T) in index order, then
// the first index whose running sum reaches rand * top_p * sum, rand the low
// 32 bits of `seed` / 2^32.  The fp32 running sums are formed in index order
// exactly as the reference's loop; the warp only parallelises the expf
// evaluations.
__device__ __forceinline__ int warp_top_p(const float* row, int V, float temperature, float top_p, uint64_t seed,
                                          int lane) {
    float m = row[0];
    {
        float lm = -INFINITY;
        for (int i = lane; i < V; i += 32) lm = fmaxf(lm, row[i]);
        for (int o = 16; o > 0; o >>= 1) lm = fmaxf(lm, __shfl_xor_sync(0xffffffffu, lm, o));
        if (!isnan(m)) m = lm;
    }
    float sum = 0.0f;
    for (int base = 0; base < V; base += 32) {
        const int i = base + lane;
        const float e = (i < V) ? expf((row[i] - m) / temperature) : 0.0f;
        const int cnt = min(32, V - base);
        for (int j = 0; j < cnt; ++j) sum += __shfl_sync(0xffffffffu, e, j);
    }
    const float threshold = top_p * sum;
    const float rv = static_cast<float>(seed & 0xFFFFFFFFull) / 4294967296.0f;
    const float target = rv * threshold;
    float cum = 0.0f;
    int selected = 0;
    bool found = false;
    for (int base = 0; base < V && !found; base += 32) {
        const int i = base + lane;
        const float e = (i < V) ? expf((row[i] - m) / temperature) : 0.0f;
        const int cnt = min(32, V - base);
        for (int j = 0; j < cnt; ++j) {
            cum += __shfl_sync(0xffffffffu, e, j);
            if (cum >= target) { selected = base + j; found = true; break; }
        }
    }
    return selected;
}

// The legacy launch_top_p_sampling rule: temperature < 0.01 is greedy.
__device__ __forceinline__ int warp_sample(const float* row, int V, float temperature, float top_p, uint64_t seed,
                                           int lane) {
    return temperature < 0.01f ? warp_argmax_first(row, V, lane) : warp_top_p(row, V, temperature, top_p, seed, lane);
}

}  // namespace tb
