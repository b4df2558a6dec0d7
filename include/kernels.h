/*
 * kernels.h -- element-wise / normalisation / routing kernels (libkernels.so),
 * drop-in for the reference engine's csrc/kernels.h.
 *
 * The 20 launch_* entry points keep the reference's names, argument order and
 * fp32 row-major layouts (csrc/kernels.h:12-31) so that the engine's layer
 * forward (src/terra/engine.t:1235-1371) runs on them unchanged.  They return
 * void as the reference's do; the last launch error of the calling thread is
 * kept and can be read with kernels_last_error() (an addition: the reference
 * reports nothing).
 *
 * Implementations are new sm_100a kernels in time_b200/csrc/kernels.cu.
 * Where the reference's behaviour has a defect that callers can observe, the
 * behaviour kept is stated beside the declaration.
 */
#ifndef KERNELS_H
#define KERNELS_H

#include <stdint.h>
#include <stddef.h>
#include "cuda_wrappers.h"

#ifdef __cplusplus
extern "C" {
#endif

/* csrc/kernels.h:12; E4M3 byte -> fp32, no scale.  The NaN codes 0x7F/0xFF
 * decode to 0 as on the reference GPU (csrc/kernels.cu:18-19). */
void launch_fp8_dequantize(const void* input, void* output, size_t count, cwStream_t stream);
/* csrc/kernels.h:13; fp32 -> E4M3 with the reference's own encoder
 * (csrc/kernels.cu:28-45: round-half-away mantissa, clamp at 7, saturate to
 * 0x7E, NaN -> 0x7F).  The MoE path uses RNE instead (moe_layer.h). */
void launch_f32_to_fp8(const float* input, void* output, size_t count, cwStream_t stream);
/* csrc/kernels.h:14; out = x / sqrt(mean(x^2) + eps) * gamma, one row per token.
 * The sum of squares follows the reference's order bit for bit: 256 strided
 * fma partials, then a pairwise tree (csrc/kernels.cu:61-85). */
void launch_rms_norm(const float* input, const float* gamma, float* output, int hidden_dim, int batch_size, float eps, cwStream_t stream);
/* csrc/kernels.h:15; rotate-half RoPE over the full head_dim of q and k, both
 * laid out [seq][num_heads][head_dim] as the reference indexes them
 * (csrc/kernels.cu:87-108). */
void launch_rope(float* q, float* k, int head_dim, int num_heads, int seq_len, int start_pos, float theta, cwStream_t stream);
/* csrc/kernels.h:16; in-place row softmax. */
void launch_softmax(float* input, int batch_size, int seq_len, cwStream_t stream);
/* csrc/kernels.h:17; out = silu(gate) * up. */
void launch_swiglu(const float* gate, const float* up, float* output, size_t count, cwStream_t stream);
/* csrc/kernels.h:18; in-place tanh-GELU. */
void launch_gelu(float* data, size_t count, cwStream_t stream);
/* csrc/kernels.h:19; dtype 1 = E4M3, 2 = fp16, otherwise fp32 table. */
void launch_embedding_lookup(const void* embedding_table, const int64_t* token_ids, float* output, int hidden_dim, int num_tokens, int dtype, cwStream_t stream);
/* csrc/kernels.h:20; a += b. */
void launch_add_residual(float* a, const float* b, size_t count, cwStream_t stream);
/* csrc/kernels.h:21; first index of the row maximum. */
void launch_argmax(const float* logits, int64_t* output, int vocab_size, int batch_size, cwStream_t stream);
/* csrc/kernels.h:22; temperature < 0.01 falls back to argmax; otherwise the
 * reference's CDF inversion over the unsorted vocabulary with threshold
 * top_p * sum (csrc/kernels.cu:236-262). */
void launch_top_p_sampling(const float* logits, int64_t* output, float temperature, float top_p, int vocab_size, int batch_size, const uint64_t* random_seeds, cwStream_t stream);
/* csrc/kernels.h:23; logits of past tokens: >0 divided by penalty, else multiplied. */
void launch_apply_rep_penalty(float* logits, const int64_t* past_tokens, int past_len, int vocab_size, float penalty, cwStream_t stream);
/* csrc/kernels.h:24; causal attention over the current chunk ([seq][heads][d]),
 * page_table/num_pages/page_size accepted and unused as in the reference.
 * Unlike the reference (csrc/kernels.cu:282,293) it has no 1024-key cap. */
void launch_paged_attention_prefill(const float* q, const float* k, const float* v, float* output, const int32_t* page_table, int num_pages, int page_size, int num_heads, int head_dim, int seq_len, float scale, cwStream_t stream);
/* csrc/kernels.h:25; single-query GQA attention over a paged cache
 * [page][slot][kv_head][d], kv_head = head / (num_heads / num_kv_heads). */
void launch_paged_attention_decode(const float* q, const float* kv_cache_k, const float* kv_cache_v, float* output, const int32_t* page_table, int num_pages, int page_size, int num_heads, int num_kv_heads, int head_dim, int past_len, float scale, cwStream_t stream);
/* csrc/kernels.h:26; scatter k/v rows into their pages. */
void launch_update_kv_cache(const float* k, const float* v, float* kv_cache_k, float* kv_cache_v, const int32_t* page_table, int page_size, int num_kv_heads, int head_dim, int seq_len, int start_pos, cwStream_t stream);
/* csrc/kernels.h:27; logits[t][e] = sum_i hidden[t][i] * W[e][i] in fp32.
 * gate_dtype is accepted and ignored (weights are read as fp32) exactly as in
 * the reference (csrc/kernels.cu:589-592).  The sum follows the reference's
 * order bit for bit (256 strided fma partials + pairwise tree,
 * csrc/kernels.cu:412-435). */
void launch_moe_gate(const float* hidden, const void* gate_weight, float* router_logits, int hidden_dim, int num_experts, int batch_size, int gate_dtype, cwStream_t stream);
/* csrc/kernels.h:28; per token: top_k largest logits (strict '>', so the lower
 * expert index wins a tie; NaN never selected; top_k <= 16), weights =
 * softmax over the selected logits (csrc/kernels.cu:437-471). */
void launch_moe_topk(const float* router_logits, int32_t* expert_indices, float* expert_weights, int num_experts, int top_k, int batch_size, cwStream_t stream);
/* csrc/kernels.h:29; replicates every token top_k times into [T][top_k][H];
 * expert_indices is accepted and unused, as in csrc/kernels.cu:473-482. */
void launch_moe_dispatch(const float* input, float* expert_inputs, const int32_t* expert_indices, int hidden_dim, int top_k, int batch_size, cwStream_t stream);
/* csrc/kernels.h:30; out[t] = sum_k w[t][k] * y[t][k] over [T][top_k][H]. */
void launch_moe_combine(const float* expert_outputs, const float* expert_weights, float* output, int hidden_dim, int top_k, int batch_size, cwStream_t stream);
/* csrc/kernels.h:31; dst = src. */
void launch_copy_hidden(const float* src, float* dst, size_t count, cwStream_t stream);

/* Addition: the cudaError_t (as int) of the last launch_* call made by this
 * thread, 0 if it succeeded.  Reading it does not clear it. */
int kernels_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* KERNELS_H */
