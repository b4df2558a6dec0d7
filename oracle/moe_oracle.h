/*
 * moe_oracle.h -- CPU restatement of the reference engine's MoE decoder-layer
 * path.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and the
 * CPU-baseline leg of bench.py call it as the checker.  The product (the
 * libraries under time_b200/) never links or calls it.
 *
 * Every function names the reference lines it restates.  Paths are relative
 * to the kollarsandor/time source tree.
 *
 * Parity status:
 *   - FP8 decode/encode, RMSNorm, router logits (reference order), top-k and
 *     combine restate csrc/kernels.cu.  They are pinned by the reference's own
 *     codec test values (tests/test_smoke.py:5-56) and by golden vectors that
 *     the reference's CUDA kernels produced (tests/golden/, made by
 *     tests/golden/make_ref_golden.py from oracle/_ref on a GPU box).
 *   - Block scales, shared expert, 1x128 activation quantisation, bf16 I/O
 *     and the stable expert permutation have no counterpart in the reference:
 *     "parity unpinned" (defined by this project, not by reference tests).
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- scalar codecs ---------------- */

/* E4M3 -> fp32 as the reference GPU decodes it (csrc/kernels.cu:7-26): no
 * scale, exponent bias 7, subnormals m*2^-9, the NaN codes (S.1111.111) -> 0. */
float orc_e4m3_decode_ref(uint8_t b);
/* E4M3 (OCP "fn" variant) -> fp32 with NaN codes -> NaN.  This is the format
 * the MoE path stores (same bits as the reference's format for every code but
 * the NaN code, which the encoder below never produces). */
float orc_e4m3_decode(uint8_t b);
/* fp32 -> E4M3 with the reference's encoder (csrc/kernels.cu:28-45): log2f
 * exponent, roundf mantissa clamped to [0,7] (no carry), saturation 0x7E,
 * NaN -> 0x7F.  Used only for the codec parity test. */
uint8_t orc_e4m3_encode_ref(float x);
/* fp32 -> E4M3 round-to-nearest-even, saturating to +-448, NaN -> 0x7F: the
 * semantics of PTX cvt.rn.satfinite.e4m3x2.f32, which the MoE kernels use. */
uint8_t orc_e4m3_encode_rne(float x);
/* bf16 <-> fp32 (round-to-nearest-even; NaN kept quiet). */
float orc_bf16_to_f32(uint16_t b);
uint16_t orc_f32_to_bf16(float x);

/* ---------------- reference-order kernels ---------------- */

/* RMSNorm, csrc/kernels.cu:61-85: per row the sum of squares is 256
 * strided fma partials (lane l sums i = l, l+256, ... in order) reduced by the
 * pairwise tree 128,64,...,1; rms = sqrtf(ss/H + eps); out = (x/rms)*gamma. */
void orc_rmsnorm_ref(const float* x, const float* gamma, float* out,
                     int hidden, int rows, float eps);
/* Same reduction; returns only rms[row]. */
void orc_rms_ref(const float* x, float* rms, int hidden, int rows, float eps);

/* Router logits in the reference order, csrc/kernels.cu:412-435:
 * logits[t][e] = tree256(fma partials of hidden[t] . W[e]). */
void orc_moe_gate_ref(const float* hidden, const float* w, float* logits,
                      int hidden_dim, int num_experts, int tokens);
/* The MoE layer's router logits: orc_moe_gate_ref's value for each (t, e)
 * (the reference's 256-lane fma partials and pairwise tree) + bias[e] in fp32
 * when bias != NULL. */
void orc_moe_router_logits(const float* hidden, const float* w, const float* bias,
                           float* logits, int hidden_dim, int num_experts, int tokens);

/* Top-k, csrc/kernels.cu:437-471: insertion with strict '>' from -FLT_MAX, so
 * the lower expert index wins a tie and NaN is never selected (slot index
 * stays -1, weight 0).  Weights are exp(v)/sum exp(v) over the selected slots
 * in slot order, as the reference computes them; when the largest selected
 * logit exceeds 80 (where the reference's expf overflows) the max-subtracted
 * form exp(v - v0)/sum exp(v - v0) is used instead. */
void orc_moe_topk_ref(const float* logits, int32_t* idx, float* weights,
                      int num_experts, int top_k, int tokens);

/* ---------------- MoE FFN block (hot path) ---------------- */

typedef struct {
    int hidden;        /* H, multiple of 128 */
    int num_experts;   /* E routed experts */
    int top_k;         /* k <= 16 */
    int intermediate;  /* I, multiple of 128 */
    int num_shared;    /* 0 or 1 shared expert (expert index E) */
    float eps;         /* RMSNorm epsilon */
} orc_moe_cfg;

typedef struct {
    const float* gamma;        /* [H] RMSNorm weight */
    const float* router_w;     /* [E][H] fp32 */
    const float* router_bias;  /* [E] fp32 or NULL */
    const uint8_t* w13;        /* [E+S][2I][H] e4m3: rows [0,I) gate, [I,2I) up */
    const float* s13;          /* [E+S][2I/128][H/128] block scales */
    const uint8_t* w2;         /* [E+S][H][I] e4m3 */
    const float* s2;           /* [E+S][H/128][I/128] block scales */
} orc_moe_weights;

/* Stable counting sort of the pairs p = t*k + s by expert id (ascending id,
 * ascending p within an id), followed by the shared expert's rows (all tokens
 * in order).  Each group's segment starts at a multiple of `pad` rows.
 *   counts[G], seg_start[G] (G = E + num_shared), pos[T*k] = row of each pair
 *   (-1 if the pair's index is < 0), row_token[R] = token of each row or -1
 *   for padding rows.  Returns R (total rows incl. padding).
 * Semantics follow the per-expert token order of kernels.fut:385-396
 * restricted to assigned pairs. */
int orc_moe_permute(const int32_t* idx, int tokens, int top_k, int num_experts,
                    int num_shared, int pad, int32_t* counts, int32_t* seg_start,
                    int32_t* pos, int32_t* row_token, int row_capacity);

/* 1x128 activation quantisation of one row of `cols` values:
 * per 128-block amax; inv = 448/amax; q = rne_satfinite(v*inv); s = amax/448;
 * an all-zero block gets q = 0, s = 0. */
void orc_quant_row_1x128(const float* v, int cols, uint8_t* q, float* s);

/* Two-term 1x128 quantisation (the kernels' CBW_GEMM_ACT_X2 format): q as
 * above, and the residual's e4m3 byte ql = rne_satfinite(u - decode(q)) with
 * u = v*inv (fp32 product and difference), one scale s for both. */
void orc_quant_row_1x128_x2(const float* v, int cols, uint8_t* q, uint8_t* ql, float* s);

/* MoE FFN block forward for `tokens` tokens:
 *   n = RMSNorm_ref(x) ; logits = gate_ref(n) (+bias) ; top-k (ref)
 *   routed/shared expert MLP y = W2 . (silu(W_gate . n) * (W_up . n))
 *   out = bf16( x + y_shared + sum_s w[t][s] * y[t][s] )
 * mode 0 ("q"): mirrors the rounding points of the B200 kernels: n quantised
 *   1x128 to e4m3 (RNE), block-scaled dot products accumulated in double, h
 *   quantised 1x128, y rounded to bf16 before the combine.
 * mode 1 ("ref"): fp32 activations end to end with dequantised weights, the
 *   reference's arithmetic (kernels.fut:343-368, engine.t:1317-1347).
 * mode 2 ("q2"): mode 0 with the two-term activations of
 *   orc_quant_row_1x128_x2 (activation = s * (decode(q) + decode(ql))), the
 *   kernels' two-plane mode.
 * Optional outputs (may be NULL): idx [T][k], weights [T][k], logits [T][E].
 * threads: OpenMP threads (<= 0 means the library default). */
void orc_moe_ffn_forward(const orc_moe_cfg* cfg, const orc_moe_weights* w,
                         const uint16_t* x_bf16, uint16_t* out_bf16, int tokens,
                         int mode, int32_t* idx_out, float* weights_out,
                         float* logits_out, int threads);

/* Same, for a precomputed routing (idx/weights given) -- used to evaluate
 * the expert path alone, and by the EP tests. */
void orc_moe_ffn_experts(const orc_moe_cfg* cfg, const orc_moe_weights* w,
                         const uint16_t* x_bf16, const int32_t* idx,
                         const float* weights, uint16_t* out_bf16, int tokens,
                         int mode, int threads);

#ifdef __cplusplus
}
#endif

#endif /* MOE_ORACLE_H */
