/*
 * attn_oracle.c -- CPU restatement of the reference's decode-attention path
 * (RoPE, paged KV cache, GQA decode attention) and of the block-scaled FP8
 * projection the new build runs it with.
 * TEST INFRASTRUCTURE ONLY (checker for tests/ and the CPU baseline of the
 * attention measurement); the product libraries never call it.
 *
 * Pinning: orc_attn_decode_paged with fp32 inputs and orc_rope_partial with
 * rot == head_dim are checked against the reference's own kernels
 * (kernel_paged_attention_decode, kernel_rope in csrc/kernels.cu, run on a B200;
 * fixture tests/golden/ref_kernels.npz).  The partial-rotary restriction, bf16
 * pages and the FP8 projections are new-build semantics: parity unpinned for
 * those parts.
 */
#include "attn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "moe_oracle.h"

/* out[r][o] = sum_kb (sum_{i in kb} dec(xq[r][i]) dec(w[o][i])) * xs[r][kb] * ws[o/128][kb]
 * in double: the 128x128 block-scaled projection of kernels.fut:343-347 with
 * 1x128-quantised activations (the kernels' rounding points). */
void orc_gemm_fp8_block(const uint8_t* xq, const float* xs, int rows, const uint8_t* w, const float* ws, int N,
                        int K, float* out) {
    float lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = orc_e4m3_decode((uint8_t)i);
    const int KB = K / 128;
    for (int r = 0; r < rows; ++r) {
        const uint8_t* xr = xq + (size_t)r * K;
        for (int o = 0; o < N; ++o) {
            const uint8_t* wr = w + (size_t)o * K;
            double acc = 0.0;
            for (int kb = 0; kb < KB; ++kb) {
                double d = 0.0;
                for (int i = kb * 128; i < kb * 128 + 128; ++i) d += (double)lut[xr[i]] * lut[wr[i]];
                acc += d * ((double)xs[(size_t)r * KB + kb] * ws[(size_t)(o / 128) * KB + kb]);
            }
            out[(size_t)r * N + o] = (float)acc;
        }
    }
}

/* inv_freq[i] = theta^(-2i/rot), i < rot/2, rounded once to fp32. */
void orc_rope_inv_freq(int rot, float theta, float* inv_freq) {
    for (int i = 0; i < rot / 2; ++i) inv_freq[i] = (float)pow((double)theta, -2.0 * i / (double)rot);
}

/* Rotate-half RoPE of kernels.cu:87-108 on the first `rot` dims of each of
 * `heads` rows of length d: pairs (i, i + rot/2), angle = float(pos) *
 * inv_freq[i] in fp32 (as the kernel forms it), cos/sin evaluated in double
 * and rounded to fp32. */
void orc_rope_partial(float* x, int heads, int d, int rot, int pos, const float* inv_freq) {
    const int half = rot / 2;
    for (int h = 0; h < heads; ++h) {
        float* xh = x + (size_t)h * d;
        for (int i = 0; i < half; ++i) {
            const float ang = (float)pos * inv_freq[i];
            const float c = (float)cos((double)ang), s = (float)sin((double)ang);
            const float x0 = xh[i], x1 = xh[i + half];
            xh[i] = x0 * c - x1 * s;
            xh[i + half] = x0 * s + x1 * c;
        }
    }
}

/* Decode attention for one sequence (kernels.fut:245-279): for each query
 * head h (kv head h / (nq / nkv), kernels.cu:331), scores q.k_j * scale over
 * positions j < seq_len read through the page table from caches laid out
 * [page][page_size][nkv][d] (kernels.cu:394-410), max-subtracted softmax, then
 * sum_j p_j v_j.  Accumulation in double. */
void orc_attn_decode_paged(const float* q, const float* k_cache, const float* v_cache, const int32_t* page_table,
                           int seq_len, int nq, int nkv, int d, int page_size, float scale, float* out) {
    const int group = nq / nkv;
    double* sc = (double*)malloc(sizeof(double) * (seq_len > 0 ? seq_len : 1));
    for (int h = 0; h < nq; ++h) {
        const int kvh = h / group;
        const float* qh = q + (size_t)h * d;
        double mx = -HUGE_VAL;
        for (int j = 0; j < seq_len; ++j) {
            const int phys = page_table[j / page_size];
            const float* kr = k_cache + (((size_t)phys * page_size + j % page_size) * nkv + kvh) * d;
            double dot = 0.0;
            for (int i = 0; i < d; ++i) dot += (double)qh[i] * kr[i];
            sc[j] = dot * scale;
            if (sc[j] > mx) mx = sc[j];
        }
        double sum = 0.0;
        for (int j = 0; j < seq_len; ++j) {
            sc[j] = exp(sc[j] - mx);
            sum += sc[j];
        }
        for (int i = 0; i < d; ++i) {
            double acc = 0.0;
            for (int j = 0; j < seq_len; ++j) {
                const int phys = page_table[j / page_size];
                const float* vr = v_cache + (((size_t)phys * page_size + j % page_size) * nkv + kvh) * d;
                acc += sc[j] * vr[i];
            }
            out[(size_t)h * d + i] = seq_len > 0 ? (float)(acc / sum) : 0.0f;
        }
    }
    free(sc);
}
