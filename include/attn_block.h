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
 * q_out.  A position outside the page table sets *error_word = 4, a page id
 * outside [0, num_cache_pages) sets 6; the token is skipped either way. */
moe_status_t attn_rope_kv_write(const void* qkv_bf16, int B, int nq, int nkv, int head_dim, int rot,
                                const float* inv_freq, const int32_t* positions, const int32_t* page_table,
                                int max_pages, int page_size, int num_cache_pages, void* q_out_bf16, void* k_cache,
                                void* v_cache, int* error_word, cwStream_t stream);

/* Bytes of the split-partials workspace for attn_decode_paged. */
size_t attn_decode_workspace_bytes(int B, int nq, int max_splits);

/* Decode attention (kernels.fut:245-279; GQA kernels.cu:331):
 * out[b][h] = sum_j softmax_j(q[b][h] . k_j * scale) v_j over positions
 * j < seq_lens[b] of sequence b's pages.  The context is cut into splits of
 * split_tokens (a multiple of 16) tokens, at most max_splits per sequence
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

/* out[t][i] = bf16(residual[t][i] + sum_{r < tp} partial_r[t][i]), the ranks
 * summed in fp32 in order 0..tp-1 so every rank gets the same bits.
 * partials_dev: device array of tp pointers (this GPU's buffers, or peer
 * buffers mapped into this GPU), each bf16 [T][H]; H % 8 == 0. */
moe_status_t attn_tp_reduce_residual(const void* const* partials_dev, int tp, const void* residual_bf16, int T, int H,
                                     void* out_bf16, cwStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TIME_B200_ATTN_BLOCK_H */
