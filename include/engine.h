/* engine.h -- the decoder serving engine (time_b200/lib/engine.so): a GLM-4.x
 * FP8 model's layers run batched over the requests in flight, one process
 * per GPU.
 *
 * Replaces the reference's engine.so (src/terra/engine.t, exported at
 * engine.t:1905-1921 and bound by src/server/engine_wrapper.py:64-98): the
 * first seven functions below keep its names, argument order, return values
 * and error values, so the reference's NativeEngine loads this library
 * unchanged.  What differs, by design:
 *   - run_batch_decode_ext runs the unfinished requests together (the
 *     reference loops run_decode_step per request, engine.t:1877-1903), and
 *     prefill_opaque admits a request whose prompt then runs with the next
 *     decode step, batched with every other admitted prompt (the reference
 *     runs each prompt at once, engine.t:1373-1410): a step's rows are every
 *     position without K/V yet, request by request, in forwards of at most
 *     prefill_chunk rows, the last forward ending with each request's newest
 *     position -- the rows that are sampled;
 *   - layers are the B200 attention block (attn_block.h) and MoE layer
 *     (moe_layer.h) with bf16 activations, FP8 weights with 128x128 block
 *     scales and bf16 KV pages; the first `first_k_dense_replace` layers run
 *     their dense FFN as a one-expert MoE layer (weight 1.0);
 *   - positions are causal: prefill writes the K/V of prompt positions
 *     0..L-2 and every decode step runs the last known token at position
 *     past_len - 1, attending over positions 0..past_len - 1 (the reference's
 *     decode re-runs that token at position past_len, engine.t:1418-1428);
 *   - a request finishes after max_tokens generated tokens or at max_seq
 *     total tokens (the reference compares max_tokens with the prompt plus
 *     generated length, engine.t:1495-1497);
 *   - sampling follows the reference's GPU path (engine.t:1446-1451): greedy
 *     below temperature 0.01, else its top-p CDF inversion with the seed
 *     (request_id * 31 + past_len * 17) * 6364136223846793005 +
 *     1442695040888963407; rep_penalty is accepted and, as on the
 *     reference's GPU path, not applied.
 * num_gpus > 1 in init_engine is served by this process's current GPU (a
 * multi-GPU deployment runs one engine process per GPU).
 */
#ifndef TIME_B200_ENGINE_H
#define TIME_B200_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "attn_block.h"
#include "moe_layer.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct glm_engine glm_engine_t;

/* ---------------------------------------------- the reference's engine.so */

/* model_dir holds config.json and the safetensors checkpoint
 * (model.safetensors.index.json + shards, or model.safetensors).  NULL on
 * any failure (missing or malformed files, unsupported shapes, device memory
 * short), with a line on stderr. */
glm_engine_t* init_engine(const char* model_dir, int32_t max_batch, int32_t max_seq, int32_t num_gpus);

/* Creates a request (a request slot, the KV pages of its prompt) and returns
 * its state, or NULL (seq_len outside [1, max_seq], a token outside the
 * vocabulary, no free request slot or KV pages).  The prompt's positions
 * 0..seq_len-2 run through the layers with the next decode step. */
void* prefill_opaque(glm_engine_t* engine, int64_t request_id, const int64_t* token_ids, int32_t seq_len,
                     float temperature, float top_p, float rep_penalty, int32_t max_tokens);

/* One token for one request: 0, or -1 (engine NULL / not initialised), -2
 * (state NULL), -3 (out of KV pages, the request is finished), -4 (device
 * error). */
int32_t decode_step_opaque(glm_engine_t* engine, void* state, int64_t* next_token_out, int32_t* is_done_out);

void free_request_opaque(glm_engine_t* engine, void* state);
void free_engine(glm_engine_t* engine);

/* engine.t:1814-1831: 0 hidden, 1 layers, 2 attention heads, 3 vocabulary,
 * 4 routed experts, 5 top-k, 6 GPUs, 7 max batch, 8 max sequence, 9 KV pages
 * in use, 10 KV pages in all, 11 requests, 12 checkpoint tensors, 13 GPU in
 * use (1); -1 for anything else. */
int64_t get_engine_info(glm_engine_t* engine, int32_t info_type);

/* One decode step for every non-NULL, unfinished state, batched into one
 * forward; NULL or finished states give token 0 and done 1, as do requests
 * that ran out of KV pages.  0, -1 (engine NULL), -4 (device error: every
 * state's done is set). */
int32_t run_batch_decode_ext(glm_engine_t* engine, void* const* states, int32_t num_states, int64_t* out_tokens,
                             int32_t* out_done);

/* ---------------------------------------------- builder (weights in memory) */

typedef struct {
    int hidden;              /* multiple of 128 */
    int num_layers;
    int first_dense;         /* layers [0, first_dense) have a dense FFN */
    int num_q_heads, num_kv_heads, head_dim, rotary_dim;   /* head_dim 128 */
    int vocab_size;
    int num_experts, top_k, moe_intermediate, num_shared;
    int dense_intermediate;
    float rope_theta, rms_eps;
    int max_batch;           /* requests in flight (decode rows) */
    int max_seq;             /* tokens per request, prompt + generated */
    int prefill_chunk;       /* rows per forward (admitted prompts are cut to it); 0 = 2048 */
    int num_cache_pages;     /* 16-token KV pages shared by all requests; 0 = max_batch * ceil(max_seq / 16) */
    int num_gpus;            /* GPUs of this process, from the current device on; 0 or 1 = one */
} glm_engine_config_t;

/* Creates an engine whose weights the caller provides (device memory that
 * must outlive the engine; several layers may share one weight set).  The KV
 * caches, activations and workspaces are allocated here.  The first request
 * waits for the device once, so the weights may still be in flight on any
 * stream until then.
 *
 * num_gpus = N > 1: one process drives devices d .. d + N - 1 (d = the
 * current device; peer access is enabled between them).  Rank r holds query
 * heads [r nq/N, (r+1) nq/N) and KV heads [r nkv/N, (r+1) nkv/N) of every
 * attention layer (tensor parallel, the o_proj partials summed over the
 * ranks in rank order), routed experts [r E/N, (r+1) E/N) of every MoE layer
 * and the shared expert (expert parallel over NVLink peer memory), and the
 * dense FFNs whole.  Each forward runs every layer's attention on all rows on
 * every rank; the FFN of rows [r R/N, (r+1) R/N) runs on rank r and the rows
 * are gathered to every rank (peer stores) before the next layer.  Rank 0
 * holds the requests and computes the final norm, the lm_head and the
 * sampling.  Weights come per rank (glm_engine_set_layer_rank,
 * glm_engine_set_embedding_rank) on that rank's device. */
moe_status_t glm_engine_create(const glm_engine_config_t* cfg, glm_engine_t** out);

/* embed bf16 [vocab][hidden], final_norm fp32 [hidden], lm_head bf16
 * [vocab][hidden] (may equal embed for tied embeddings). */
moe_status_t glm_engine_set_embedding(glm_engine_t* engine, const void* embed_bf16, const float* final_norm,
                                      const void* lm_head_bf16);

/* Layer `layer`'s attention (tp 1 layout of attn_block_weights_t) and FFN: a
 * MoE layer's moe_layer_weights_t, or for layer < first_dense a dense FFN as
 * one expert (w13 [2 I][H], w2 [H][I], router fields ignored). */
moe_status_t glm_engine_set_layer(glm_engine_t* engine, int layer, const attn_block_weights_t* attn,
                                  const moe_layer_weights_t* ffn);

/* num_gpus > 1: rank `rank`'s weights, on that rank's device.  Attention in
 * the rank's tp layout (w_qkv rows: its query heads, then its KV heads' k and
 * v rows; w_o columns of its query heads), the MoE layer's local experts then
 * the shared expert (router fields whole), a dense FFN whole.  The embedding
 * table on every rank; final_norm and lm_head are read on rank 0 only (NULL
 * elsewhere).  With one GPU these equal glm_engine_set_layer /
 * glm_engine_set_embedding for rank 0. */
moe_status_t glm_engine_set_layer_rank(glm_engine_t* engine, int rank, int layer, const attn_block_weights_t* attn,
                                       const moe_layer_weights_t* ffn);
moe_status_t glm_engine_set_embedding_rank(glm_engine_t* engine, int rank, const void* embed_bf16,
                                           const float* final_norm, const void* lm_head_bf16);

/* fp32 logits [rows][vocab] of the last decode step's rows (rows in the
 * order of the states passed to it, finished ones skipped) into host memory. */
moe_status_t glm_engine_copy_logits(glm_engine_t* engine, float* host_out, int rows);

/* Test hooks, for checking the layers one by one.  Routing capture: when on,
 * each MoE layer's top-k ids and weights of every row of a decode step (all
 * its forwards, rows in the step's order) are kept; glm_engine_copy_routing
 * copies layer `layer`'s first `rows` [rows][top_k] of the last step.  Capture
 * synchronises after every forward. */
moe_status_t glm_engine_set_capture(glm_engine_t* engine, int on);
moe_status_t glm_engine_copy_routing(glm_engine_t* engine, int layer, int rows, int32_t* idx_host, float* w_host);
/* A request's KV page ids (up to max_pages into out); returns the number of
 * pages it holds, or -1 for an unknown state. */
int glm_engine_request_pages(glm_engine_t* engine, const void* state, int32_t* out, int max_pages);
/* Pages [page, page + npages) of layer `layer`'s K and V caches (bf16
 * [npages][16][num_kv_heads][128]) into host memory. */
moe_status_t glm_engine_copy_kv(glm_engine_t* engine, int layer, int page, int npages, void* k_host, void* v_host);

/* Reads and clears every layer's device error word (synchronises). */
moe_status_t glm_engine_check_error(glm_engine_t* engine);

/* Per-stage device time of the last decode step when timing is on (ms):
 * [0] embedding, [1] attention blocks, [2] FFN layers, [3] final norm +
 * lm_head + sampling.  Timing adds events between layers; off by default. */
moe_status_t glm_engine_set_timing(glm_engine_t* engine, int on);
moe_status_t glm_engine_stage_ms(glm_engine_t* engine, float* out4);

/* Device bytes the engine allocates for `cfg` beyond the weights. */
size_t glm_engine_device_bytes(const glm_engine_config_t* cfg);

#ifdef __cplusplus
}
#endif

#endif /* TIME_B200_ENGINE_H */
