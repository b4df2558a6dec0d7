/* attn_oracle.h -- CPU restatement of the decode-attention path (test
 * infrastructure only; see attn_oracle.c for the reference lines followed). */
#ifndef ATTN_ORACLE_H
#define ATTN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void orc_gemm_fp8_block(const uint8_t* xq, const float* xs, int rows, const uint8_t* w, const float* ws, int N,
                        int K, float* out);
void orc_rope_inv_freq(int rot, float theta, float* inv_freq);
void orc_rope_partial(float* x, int heads, int d, int rot, int pos, const float* inv_freq);
void orc_attn_decode_paged(const float* q, const float* k_cache, const float* v_cache, const int32_t* page_table,
                           int seq_len, int nq, int nkv, int d, int page_size, float scale, float* out);

#ifdef __cplusplus
}
#endif

#endif /* ATTN_ORACLE_H */
