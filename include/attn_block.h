/* attn_block.h -- paged-KV decode attention entry points (libkernels.so).
 *
 * No counterpart in the reference's C-ABI: the reference engine runs
 * attention through launch_rope / launch_update_kv_cache /
 * launch_paged_attention_decode (csrc/kernels.h; fp32, one block per head,
 * src/terra/engine.t:1269-1310), which stay exported unchanged.  These are
 * the B200 path for the tensor-parallel attention half of the decoder layer
 * at decode (one new token per sequence): bf16 KV pages, GQA groups of up to
 * 16 query heads per KV head, head_dim 128, 16-token pages.
 *
 * Layouts (device memory, row-major):
 *   qkv        bf16 [B][(nq + 2 nkv) * 128]  q heads, then k heads, then v heads
 *   q          bf16 [B][nq][128]             rotated queries
 *   k/v cache  bf16 [pages][16][nkv][128]    the reference's page layout
 *                                             (kernels.cu:394-410) in bf16
 *   page_table int32 [B][max_pages]           physical page of each 16-token page
 *   seq_lens   int32 [B]                      tokens to attend over (new token included)
 * Calls are stream-ordered and allocate nothing.
 */
#ifndef TIME_B200_ATTN_BLOCK_H
#define TIME_B200_ATTN_BLOCK_H

#include <stddef.h>
#include <stdint.h>

#include "moe_layer.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Partial rotate-half RoPE (kernels.cu:87-108 restricted to the first `rot`
 * dims: pairs (i, i + rot/2), angle = float(pos) * inv_freq[i], inv_freq[i] =
 * theta^(-2i/rot) given by the caller, device [rot/2]) on the q and k heads of
 * each token's qkv row, then k and v written to page slot pos % 16 of page
 * page_table[b][pos / 16] (kernels.cu:394-410 in bf16) and the rotated q to
 * q_out; seq_lens_out (optional, [B]) receives pos + 1, the tokens the
 * decode step attends over.  A position outside the page table sets
 * *error_word = 4, a page id outside [0, num_cache_pages) sets 6; the token is
 * skipped either way. */
moe_status_t attn_rope_kv_write(const void* qkv_bf16, int B, int nq, int nkv, int head_dim, int rot,
                                const float* inv_freq, const int32_t* positions, const int32_t* page_table,
                                int max_pages, int page_size, int num_cache_pages, void* q_out_bf16, void* k_cache,
                                void* v_cache, int32_t* seq_lens_out, int* error_word, cwStream_t stream);

/* The same for rows that are tokens of several sequences (prefill chunks,
 * batches indexed by request slot): row b uses page-table row row_seq[b] of
 * page_table [num_seqs][max_pages].  A row whose row_seq is outside
 * [0, num_seqs) is skipped (seq_lens_out 0) and sets *error_word = 7. */
moe_status_t attn_rope_kv_write_rows(const void* qkv_bf16, int B, int nq, int nkv, int head_dim, int rot,
                                     const float* inv_freq, const int32_t* positions, const int32_t* row_seq,
                                     int num_seqs, const int32_t* page_table, int max_pages, int page_size,
                                     int num_cache_pages, void* q_out_bf16, void* k_cache, void* v_cache,
                                     int32_t* seq_lens_out, int* error_word, cwStream_t stream);

/* Bytes of the split-partials workspace for attn_decode_paged. */
size_t attn_decode_workspace_bytes(int B, int nq, int max_splits);

/* Decode attention (kernels.fut:245-279; GQA kernels.cu:331):
 * out[b][h] = sum_j softmax_j(q[b][h] . k_j * scale) v_j over positions
 * j < seq_lens[b] of sequence b's pages.  The context is cut into splits of
 * split_tokens (a multiple of 16, at most 8192) tokens, at most max_splits per sequence
 * (max_splits * split_tokens >= the longest sequence).  out_bf16: bf16
 * [B][nq][128].  When out_q is given, each head's row is also quantised to
 * e4m3 (1x128, scale = amax / 448) into out_q [B][nq * 128] with scales
 * out_s [nq][out_ld] -- the activation layout of cbwFp8BlockScaledGroupedGemm.
 * Checked on the device: a sequence longer than max_pages * 16 or
 * max_splits * split_tokens is cut there (*error_word = 5); a page id outside
 * [0, num_cache_pages) reads as zeros (*error_word = 6). */
moe_status_t attn_decode_paged(const void* q_bf16, const void* k_cache, const void* v_cache, int num_cache_pages,
                               const int32_t* page_table, int max_pages, const int32_t* seq_lens, int B, int nq,
                               int nkv, int head_dim, int page_size, float scale, int split_tokens, int max_splits,
                               void* workspace, size_t workspace_bytes, void* out_bf16, void* out_q, float* out_s,
                               int out_ld, int* error_word, cwStream_t stream);

/* The same over rows of several sequences: row b attends over the first
 * seq_lens[b] positions of page-table row row_seq[b] (null: b).  Rows whose
 * row_seq is outside [0, num_seqs) get zeros. */
moe_status_t attn_decode_paged_rows(const void* q_bf16, const void* k_cache, const void* v_cache,
                                    int num_cache_pages, const int32_t* page_table, int max_pages,
                                    const int32_t* row_seq, int num_seqs, const int32_t* seq_lens, int B, int nq,
                                    int nkv, int head_dim, int page_size, float scale, int split_tokens,
                                    int max_splits, void* workspace, size_t workspace_bytes, void* out_bf16,
                                    void* out_q, float* out_s, int out_ld, int* error_word, cwStream_t stream);

/* attn_decode_paged_rows with prefill rows first: rows [0, num_prefill_rows)
 * -- prompt positions, normally runs of consecutive positions of one
 * sequence (prefill chunks) -- are attended by a prefill kernel that stages
 * each K/V page once for a block of 16 rows and all their query heads, each
 * row over positions 0..positions[r] of its sequence with one online softmax
 * over the pages in order, so a row's bits do not depend on the other rows of
 * the call; rows [num_prefill_rows, B) (decode steps) by the split decode
 * kernel.  Same arguments, outputs and checks as attn_decode_paged_rows;
 * a row gets different last bits from the two kernels. */
moe_status_t attn_paged_rows(const void* q_bf16, const void* k_cache, const void* v_cache, int num_cache_pages,
                             const int32_t* page_table, int max_pages, const int32_t* row_seq, int num_seqs,
                             const int32_t* seq_lens, int B, int num_prefill_rows, int nq, int nkv, int head_dim,
                             int page_size, float scale, int split_tokens, int max_splits, void* workspace,
                             size_t workspace_bytes, void* out_bf16, void* out_q, float* out_s, int out_ld,
                             int* error_word, cwStream_t stream);

/* out[t][i] = bf16(residual[t][i] + sum_{r < tp} partial_r[t][i]), the ranks
 * summed in fp32 in order 0..tp-1 so every rank gets the same bits.
 * partials_dev: device array of tp pointers (this GPU's buffers, or peer
 * buffers mapped into this GPU), each bf16 [T][H]; H % 8 == 0. */
moe_status_t attn_tp_reduce_residual(const void* const* partials_dev, int tp, const void* residual_bf16, int T, int H,
                                     void* out_bf16, cwStream_t stream);

/* Block-scaled FP8 projection for a few tokens (decode):
 * out[t][n] = bf16(sum_kb (sum_{k in kb} a[t][k] w[n][k]) * a_scale[kb][t] * w_scale[n/128][kb])
 * with a e4m3 [T][K], a_scale [K/128][a_ld] (a_ld >= T, a multiple of 4), w
 * e4m3 [N][K], w_scale [N/128][K/128]; N and K multiples of 128.  The K
 * blocks are split over the grid; the partial sums are added in split order
 * (deterministic) in `workspace` (fp8_gemm_small_workspace_bytes).  The same
 * product as cbwFp8BlockScaledGroupedGemm's down mode for one group, sized
 * for T up to a few hundred. */
size_t fp8_gemm_small_workspace_bytes(int T, int N, int K);
moe_status_t fp8_gemm_small(const void* a, const float* a_scale, int a_ld, int T, const void* w, const float* w_scale,
                            int N, int K, void* out_bf16, void* workspace, size_t workspace_bytes, cwStream_t stream);

/* ---------------------------------------------------------------- the block
 * One decode step of the tensor-parallel attention half of the decoder layer
 * for one TP rank (the reference's engine.t:1269-1310 sequence with the spec's
 * all-reduce after o_proj, kernels.fut:605-607):
 *   h = rmsnorm(x) -> e4m3 1x128;  qkv = W_qkv h (bf16);  partial RoPE, page
 *   write;  decode attention over pos + 1 tokens;  e4m3 rows;  partial =
 *   W_o attn (bf16, this rank's heads);  out = x + sum over ranks of partial
 *   (fp32, rank order).
 * Weights of this rank: w_qkv e4m3 [(nq + 2 nkv) * 128][hidden] (q heads, k,
 * v) with fp32 scales [rows / 128][hidden / 128]; w_o e4m3 [hidden][nq * 128]
 * with scales [hidden / 128][nq]; gamma fp32 [hidden].  The weight and cache
 * memory stays the caller's. */
typedef struct attn_block attn_block_t;

typedef struct {
    int hidden;
    int num_q_heads;        /* this rank's query heads */
    int num_kv_heads;       /* this rank's KV heads (a GQA group is at most 16 query heads) */
    int head_dim;           /* 128 */
    int rotary_dim;         /* rotated leading dims of each head (even, <= 128) */
    float rope_theta;
    float eps;              /* RMSNorm */
    int max_batch;          /* sequences per call */
    int max_pages_per_seq;  /* columns of the page table */
    int max_context;        /* longest sequence (tokens, new one included) */
    int tp_size, tp_rank;
} attn_block_config_t;

typedef struct {
    const float* gamma;
    const void* w_qkv;
    const float* s_qkv;
    const void* w_o;
    const float* s_o;
} attn_block_weights_t;

moe_status_t attn_block_create(const attn_block_config_t* cfg, const attn_block_weights_t* weights,
                               attn_block_t** out);
moe_status_t attn_block_destroy(attn_block_t* block);
/* Device workspace of one call (the caller's; one per stream). */
size_t attn_block_workspace_bytes(const attn_block_t* block);
/* Context split of the decode kernel for a call of max_batch rows (tokens);
 * a call with fewer rows may cut contexts finer (about two CTAs per SM at
 * half the longest context, never more partials than the workspace holds). */
int attn_block_split_tokens(const attn_block_t* block);

/* tp_size > 1: each rank allocates attn_block_peer_bytes bytes that every rank
 * maps (CUDA IPC / symmetric memory), zero-fills them, waits until all ranks
 * have, and passes the mapped pointers (256-byte aligned), rank order, once
 * per block (a second call is refused).  Every
 * rank must then call attn_block_decode every step, in the same order.  The
 * step keeps its pairing state on the device, so a step may be captured in a
 * CUDA graph and replayed (positions and page tables updated in place). */
size_t attn_block_peer_bytes(const attn_block_t* block);
moe_status_t attn_block_set_peer_buffers(attn_block_t* block, void* const* peer_bufs, int n);

/* One decode step: out_bf16 [B][hidden] = x + attention block output.
 * positions [B]: the new token's position (its K/V go to that slot of the
 * page table); page_table [B][max_pages_per_seq]; caches bf16
 * [num_cache_pages][16][num_kv_heads][128]. */
moe_status_t attn_block_decode(attn_block_t* block, const void* x_bf16, int B, const int32_t* positions,
                               const int32_t* page_table, int num_cache_pages, void* k_cache, void* v_cache,
                               void* out_bf16, void* workspace, size_t workspace_bytes, cwStream_t stream);

/* The rank's o_proj partial (bf16 [B][hidden]) without the TP sum or the
 * residual: for callers that reduce elsewhere, and for checking several
 * ranks' partials on one GPU (attn_tp_reduce_residual sums them). */
moe_status_t attn_block_decode_partial(attn_block_t* block, const void* x_bf16, int B, const int32_t* positions,
                                       const int32_t* page_table, int num_cache_pages, void* k_cache, void* v_cache,
                                       void* partial_bf16, void* workspace, size_t workspace_bytes, cwStream_t stream);

/* Rows of several sequences in one call -- a prefill chunk (consecutive
 * positions of one or more prompts) or a decode batch indexed by request
 * slot: row r is the token at positions[r] of the sequence whose page-table
 * row is row_seq[r] (page_table [num_seqs][max_pages_per_seq]; row_seq null
 * means row r -> r).  Every row's K/V is written before any row attends, and
 * row r attends over positions 0..positions[r] of its sequence, so the rows
 * of one prompt are causal.  R <= max_batch.  attn_block_decode is this call
 * with row_seq null and num_seqs = B. */
moe_status_t attn_block_forward(attn_block_t* block, const void* x_bf16, int R, const int32_t* positions,
                                const int32_t* row_seq, int num_seqs, const int32_t* page_table, int num_cache_pages,
                                void* k_cache, void* v_cache, void* out_bf16, void* workspace, size_t workspace_bytes,
                                cwStream_t stream);
moe_status_t attn_block_forward_partial(attn_block_t* block, const void* x_bf16, int R, const int32_t* positions,
                                        const int32_t* row_seq, int num_seqs, const int32_t* page_table,
                                        int num_cache_pages, void* k_cache, void* v_cache, void* partial_bf16,
                                        void* workspace, size_t workspace_bytes, cwStream_t stream);

/* attn_block_forward with prompt rows first: rows [0, prefill_rows) are
 * positions of prompts (prefill chunks) and are attended by the prefill
 * kernel of attn_paged_rows, whose per-row result does not depend on how the
 * prompts are packed into calls; rows [prefill_rows, R) by split decode.
 * attn_block_forward is this call with prefill_rows = 0. */
moe_status_t attn_block_prefill(attn_block_t* block, const void* x_bf16, int R, const int32_t* positions,
                                const int32_t* row_seq, int num_seqs, int prefill_rows, const int32_t* page_table,
                                int num_cache_pages, void* k_cache, void* v_cache, void* out_bf16, void* workspace,
                                size_t workspace_bytes, cwStream_t stream);
moe_status_t attn_block_prefill_partial(attn_block_t* block, const void* x_bf16, int R, const int32_t* positions,
                                        const int32_t* row_seq, int num_seqs, int prefill_rows,
                                        const int32_t* page_table, int num_cache_pages, void* k_cache, void* v_cache,
                                        void* partial_bf16, void* workspace, size_t workspace_bytes,
                                        cwStream_t stream);

/* Reads and clears the device error word (synchronises `stream`):
 * MOE_ERR_DEVICE_TIMEOUT for a wait that gave up, MOE_ERR_INVALID_ARGUMENT for
 * positions, lengths, page ids or sequence rows outside the given tables. */
moe_status_t attn_block_check_error(attn_block_t* block, cwStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TIME_B200_ATTN_BLOCK_H */
