/*
 * moe_oracle.c -- CPU restatement of the reference MoE decoder-layer path.
 * TEST INFRASTRUCTURE ONLY (checker for tests/, the smoke check and the
 * CPU-baseline leg of bench.py); the product libraries never call it.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  Floating
 * point contraction is off so that every fma below is explicit and every
 * other operation is a single IEEE-rounded fp32 operation, which is what makes
 * the reference-order functions bit-reproducible against the CUDA kernels.
 *
 * Pinning: the codec, RMSNorm, router-logit and top-k functions are checked
 * against outputs of the reference's own csrc/kernels.cu (compiled unmodified
 * into oracle/_ref/ and run on a B200; fixture tests/golden/ref_kernels.npz,
 * test tests/test_golden_ref.py) and against the reference's only test values
 * (tests/test_smoke.py:5-56).  The expert MLP with 128x128 block scales, the
 * shared expert and bf16 I/O (orc_moe_ffn_*) are new-build semantics with no
 * runnable reference counterpart: parity unpinned for those functions.
 */
#include "moe_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------- scalar codecs ---------------- */

static inline float u32_as_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_as_u32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* csrc/kernels.cu:7-26 */
float orc_e4m3_decode_ref(uint8_t bits) {
    int sign = (bits >> 7) & 1;
    int exp = (bits >> 3) & 0xF;
    int mant = bits & 0x7;
    float val;
    if (exp == 0) {
        val = (mant == 0) ? 0.0f : (float)mant * ldexpf(1.0f, -9);
    } else if (exp == 15 && mant == 7) {
        val = 0.0f;  /* the reference GPU decodes the NaN code to zero */
    } else {
        val = (1.0f + (float)mant / 8.0f) * ldexpf(1.0f, exp - 7);
    }
    return sign ? -val : val;
}

float orc_e4m3_decode(uint8_t bits) {
    if ((bits & 0x7F) == 0x7F) return NAN;
    float v = orc_e4m3_decode_ref(bits);
    /* keep the sign of zero: 0x80 is -0 */
    if (bits == 0x80) return -0.0f;
    return v;
}

/* csrc/kernels.cu:28-45, statement for statement. */
uint8_t orc_e4m3_encode_ref(float x) {
    int sign = (x < 0.0f) ? 1 : 0;
    float ax = fabsf(x);
    if (isnan(x)) return 0x7F;
    if (ax == 0.0f) return (uint8_t)(sign << 7);
    if (ax >= 448.0f) return (uint8_t)((sign << 7) | 0x7E);
    if (ax < powf(2.0f, -9.0f)) return (uint8_t)(sign << 7);
    float log2_ax = log2f(ax);
    int e = (int)floorf(log2_ax);
    if (e < -6) e = -6;
    if (e > 8) e = 8;
    int exp_bits = e + 7;
    float m = ax / powf(2.0f, (float)e) - 1.0f;
    int mant = (int)roundf(m * 8.0f);
    if (mant < 0) mant = 0;
    if (mant > 7) mant = 7;
    return (uint8_t)((sign << 7) | (exp_bits << 3) | mant);
}

/* Round-to-nearest-even E4M3 with saturation, written from the format
 * definition (bias 7, 3 mantissa bits, subnormal step 2^-9, max 448). */
uint8_t orc_e4m3_encode_rne(float x) {
    if (isnan(x)) return 0x7F;
    uint8_t sign = signbit(x) ? 0x80 : 0x00;
    float ax = fabsf(x);
    if (ax >= 448.0f) return sign | 0x7E;           /* satfinite (inf too) */
    if (ax < ldexpf(1.0f, -6)) {
        /* subnormal range: value = q * 2^-9, q in [0, 8]; q == 8 is the
         * smallest normal, whose code is also 8 (exp 1, mant 0). */
        float q = nearbyintf(ax * 512.0f);            /* exact scaling, RNE */
        return sign | (uint8_t)q;
    }
    int e;
    float m = frexpf(ax, &e);                         /* ax = m * 2^e, m in [0.5,1) */
    m *= 2.0f; e -= 1;                                /* m in [1,2) */
    float mq = nearbyintf((m - 1.0f) * 8.0f);         /* exact operands, RNE */
    int mi = (int)mq;
    if (mi == 8) { mi = 0; e += 1; }
    int eb = e + 7;
    if (eb > 15 || (eb == 15 && mi == 7)) return sign | 0x7E;
    return sign | (uint8_t)((eb << 3) | mi);
}

float orc_bf16_to_f32(uint16_t b) { return u32_as_f32((uint32_t)b << 16); }

uint16_t orc_f32_to_bf16(float x) {
    uint32_t u = f32_as_u32(x);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) {
        return (uint16_t)((u >> 16) | 0x0040u);      /* quiet NaN */
    }
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}

/* ---------------- reference-order kernels ---------------- */

/* The 256-lane partial + pairwise-tree reduction used by the reference's
 * kernel_rms_norm (csrc/kernels.cu:67-79) and kernel_moe_gate
 * (csrc/kernels.cu:420-431) with blockDim.x = 256. */
static float tree256_dot(const float* a, const float* b, int n) {
    float partial[256];
    for (int l = 0; l < 256; ++l) {
        float s = 0.0f;
        for (int i = l; i < n; i += 256) s = fmaf(a[i], b[i], s);
        partial[l] = s;
    }
    for (int stride = 128; stride > 0; stride >>= 1)
        for (int l = 0; l < stride; ++l) partial[l] = partial[l] + partial[l + stride];
    return partial[0];
}

void orc_rms_ref(const float* x, float* rms, int hidden, int rows, float eps) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * hidden;
        float ss = tree256_dot(xr, xr, hidden);
        rms[r] = sqrtf(ss / (float)hidden + eps);
    }
}

/* csrc/kernels.cu:61-85 */
void orc_rmsnorm_ref(const float* x, const float* gamma, float* out,
                     int hidden, int rows, float eps) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * hidden;
        float ss = tree256_dot(xr, xr, hidden);
        float rms = sqrtf(ss / (float)hidden + eps);
        float* o = out + (size_t)r * hidden;
        for (int i = 0; i < hidden; ++i) o[i] = (xr[i] / rms) * gamma[i];
    }
}

/* csrc/kernels.cu:412-435 */
void orc_moe_gate_ref(const float* hidden, const float* w, float* logits,
                      int hidden_dim, int num_experts, int tokens) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tokens; ++t)
        for (int e = 0; e < num_experts; ++e)
            logits[(size_t)t * num_experts + e] =
                tree256_dot(hidden + (size_t)t * hidden_dim, w + (size_t)e * hidden_dim, hidden_dim);
}

/* The MoE layer's router: the reference's logits (csrc/kernels.cu:412-435,
 * the same tree256_dot) plus the new-build routing bias, added in fp32 after
 * the tree (bias may be NULL). */
void orc_moe_router_logits(const float* hidden, const float* w, const float* bias,
                           float* logits, int hidden_dim, int num_experts, int tokens) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tokens; ++t)
        for (int e = 0; e < num_experts; ++e) {
            float s = tree256_dot(hidden + (size_t)t * hidden_dim, w + (size_t)e * hidden_dim, hidden_dim);
            if (bias) s = s + bias[e];
            logits[(size_t)t * num_experts + e] = s;
        }
}

/* csrc/kernels.cu:437-471 */
void orc_moe_topk_ref(const float* logits, int32_t* idx, float* weights,
                      int num_experts, int top_k, int tokens) {
    int kk = top_k < 16 ? top_k : 16;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tokens; ++t) {
        const float* lg = logits + (size_t)t * num_experts;
        float mv[16];
        int mi[16];
        for (int k = 0; k < kk; ++k) { mv[k] = -FLT_MAX; mi[k] = -1; }
        for (int e = 0; e < num_experts; ++e) {
            float val = lg[e];
            for (int k = 0; k < kk; ++k) {
                if (val > mv[k]) {
                    for (int j = kk - 1; j > k; --j) { mv[j] = mv[j - 1]; mi[j] = mi[j - 1]; }
                    mv[k] = val; mi[k] = e;
                    break;
                }
            }
        }
        float shift = (mv[0] > 80.0f) ? mv[0] : 0.0f;
        float sum = 0.0f;
        for (int k = 0; k < kk; ++k) sum += expf(mv[k] - shift);
        for (int k = 0; k < kk; ++k) {
            idx[(size_t)t * top_k + k] = mi[k];
            weights[(size_t)t * top_k + k] = expf(mv[k] - shift) / sum;
        }
        for (int k = kk; k < top_k; ++k) {
            idx[(size_t)t * top_k + k] = -1;
            weights[(size_t)t * top_k + k] = 0.0f;
        }
    }
}

/* ---------------- MoE FFN block ---------------- */

int orc_moe_permute(const int32_t* idx, int tokens, int top_k, int num_experts,
                    int num_shared, int pad, int32_t* counts, int32_t* seg_start,
                    int32_t* pos, int32_t* row_token, int row_capacity) {
    int G = num_experts + num_shared;
    int P = tokens * top_k;
    for (int g = 0; g < G; ++g) counts[g] = 0;
    for (int p = 0; p < P; ++p)
        if (idx[p] >= 0 && idx[p] < num_experts) counts[idx[p]]++;
    for (int g = num_experts; g < G; ++g) counts[g] = tokens;
    int row = 0;
    for (int g = 0; g < G; ++g) {
        seg_start[g] = row;
        row += ((counts[g] + pad - 1) / pad) * pad;
    }
    int R = row;
    if (row_token) {
        for (int r = 0; r < R && r < row_capacity; ++r) row_token[r] = -1;
    }
    if (G <= 0) return 0;
    int* fill = (int*)calloc((size_t)(unsigned)G, sizeof(int));
    for (int p = 0; p < P; ++p) {
        int e = idx[p];
        if (e < 0 || e >= num_experts) { pos[p] = -1; continue; }
        int r = seg_start[e] + fill[e]++;
        pos[p] = r;
        if (row_token && r < row_capacity) row_token[r] = p / top_k;
    }
    for (int g = num_experts; g < G; ++g)
        for (int t = 0; t < tokens; ++t)
            if (row_token && seg_start[g] + t < row_capacity) row_token[seg_start[g] + t] = t;
    free(fill);
    return R;
}

void orc_quant_row_1x128(const float* v, int cols, uint8_t* q, float* s) {
    for (int b = 0; b < cols / 128; ++b) {
        const float* vb = v + b * 128;
        float amax = 0.0f;
        for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(vb[i]));
        if (amax == 0.0f) {
            for (int i = 0; i < 128; ++i) q[b * 128 + i] = 0;
            s[b] = 0.0f;
            continue;
        }
        float inv = 448.0f / amax;
        for (int i = 0; i < 128; ++i) q[b * 128 + i] = orc_e4m3_encode_rne(vb[i] * inv);
        s[b] = amax / 448.0f;
    }
}

void orc_quant_row_1x128_x2(const float* v, int cols, uint8_t* q, uint8_t* ql, float* s) {
    for (int b = 0; b < cols / 128; ++b) {
        const float* vb = v + b * 128;
        float amax = 0.0f;
        for (int i = 0; i < 128; ++i) amax = fmaxf(amax, fabsf(vb[i]));
        if (amax == 0.0f) {
            for (int i = 0; i < 128; ++i) q[b * 128 + i] = ql[b * 128 + i] = 0;
            s[b] = 0.0f;
            continue;
        }
        float inv = 448.0f / amax;
        for (int i = 0; i < 128; ++i) {
            float u = vb[i] * inv;
            uint8_t hi = orc_e4m3_encode_rne(u);
            q[b * 128 + i] = hi;
            ql[b * 128 + i] = orc_e4m3_encode_rne(u - orc_e4m3_decode(hi));
        }
        s[b] = amax / 448.0f;
    }
}

static float silu_f(float g) { return g / (1.0f + expf(-g)); }

/* One expert MLP for one token: kernels.fut:343-347 with block scales.
 * mode 0: activations given as (q, s) 1x128-quantised; mode 1: fp32 n;
 * mode 2: two-term (q, ql, s), activation = s * (decode(q) + decode(ql)). */
static void expert_mlp_one(const orc_moe_cfg* cfg, const orc_moe_weights* w, int e,
                           int mode, const float* n, const uint8_t* nq, const uint8_t* nql, const float* ns,
                           const float* lut, float* hbuf, uint8_t* hq, uint8_t* hql, float* hs,
                           float* y) {
    const int H = cfg->hidden, I = cfg->intermediate;
    const int KB1 = H / 128, KB2 = I / 128;
    const uint8_t* W13 = w->w13 + (size_t)e * 2 * I * H;
    const float* S13 = w->s13 + (size_t)e * (2 * I / 128) * KB1;
    const uint8_t* W2 = w->w2 + (size_t)e * H * I;
    const float* S2 = w->s2 + (size_t)e * (H / 128) * KB2;
    for (int j = 0; j < I; ++j) {
        double g = 0.0, u = 0.0;
        const uint8_t* wg = W13 + (size_t)j * H;
        const uint8_t* wu = W13 + (size_t)(I + j) * H;
        for (int kb = 0; kb < KB1; ++kb) {
            float sg = S13[(j / 128) * KB1 + kb];
            float su = S13[((I + j) / 128) * KB1 + kb];
            double dg = 0.0, du = 0.0;
            if (mode != 1) {
                for (int i = kb * 128; i < kb * 128 + 128; ++i) {
                    float a = mode == 2 ? lut[nq[i]] + lut[nql[i]] : lut[nq[i]];
                    dg += (double)a * lut[wg[i]];
                    du += (double)a * lut[wu[i]];
                }
                g += dg * ((double)ns[kb] * sg);
                u += du * ((double)ns[kb] * su);
            } else {
                for (int i = kb * 128; i < kb * 128 + 128; ++i) {
                    dg += (double)n[i] * lut[wg[i]];
                    du += (double)n[i] * lut[wu[i]];
                }
                g += dg * sg;
                u += du * su;
            }
        }
        hbuf[j] = silu_f((float)g) * (float)u;
    }
    if (mode == 0) orc_quant_row_1x128(hbuf, I, hq, hs);
    if (mode == 2) orc_quant_row_1x128_x2(hbuf, I, hq, hql, hs);
    for (int o = 0; o < H; ++o) {
        const uint8_t* wd = W2 + (size_t)o * I;
        double acc = 0.0;
        for (int kb = 0; kb < KB2; ++kb) {
            float sd = S2[(o / 128) * KB2 + kb];
            double d = 0.0;
            if (mode != 1) {
                for (int i = kb * 128; i < kb * 128 + 128; ++i)
                    d += (double)(mode == 2 ? lut[hq[i]] + lut[hql[i]] : lut[hq[i]]) * lut[wd[i]];
                acc += d * ((double)hs[kb] * sd);
            } else {
                for (int i = kb * 128; i < kb * 128 + 128; ++i) d += (double)hbuf[i] * lut[wd[i]];
                acc += d * sd;
            }
        }
        float yv = (float)acc;
        y[o] = (mode != 1) ? orc_bf16_to_f32(orc_f32_to_bf16(yv)) : yv;
    }
}

static void ffn_experts_impl(const orc_moe_cfg* cfg, const orc_moe_weights* w,
                             const uint16_t* x_bf16, const float* nrm,
                             const int32_t* idx, const float* weights,
                             uint16_t* out_bf16, int tokens, int mode, int threads) {
    const int H = cfg->hidden, I = cfg->intermediate, K = cfg->top_k;
    float lut[256];
    for (int b = 0; b < 256; ++b) lut[b] = orc_e4m3_decode((uint8_t)b);
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
        float* xf = (float*)malloc(sizeof(float) * H);
        float* acc = (float*)malloc(sizeof(float) * H);
        float* y = (float*)malloc(sizeof(float) * H);
        float* hbuf = (float*)malloc(sizeof(float) * I);
        uint8_t* hq = (uint8_t*)malloc(I);
        uint8_t* hql = (uint8_t*)malloc(I);
        float* hs = (float*)malloc(sizeof(float) * (I / 128));
        uint8_t* nq = (uint8_t*)malloc(H);
        uint8_t* nql = (uint8_t*)malloc(H);
        float* ns = (float*)malloc(sizeof(float) * (H / 128));
#pragma omp for schedule(dynamic, 1)
        for (int t = 0; t < tokens; ++t) {
            const float* n = nrm + (size_t)t * H;
            for (int i = 0; i < H; ++i) xf[i] = orc_bf16_to_f32(x_bf16[(size_t)t * H + i]);
            if (mode == 0) orc_quant_row_1x128(n, H, nq, ns);
            if (mode == 2) orc_quant_row_1x128_x2(n, H, nq, nql, ns);
            for (int i = 0; i < H; ++i) acc[i] = xf[i];
            for (int sidx = 0; sidx < cfg->num_shared; ++sidx) {
                expert_mlp_one(cfg, w, cfg->num_experts + sidx, mode, n, nq, nql, ns, lut, hbuf, hq, hql, hs, y);
                for (int i = 0; i < H; ++i) acc[i] += y[i];
            }
            for (int s = 0; s < K; ++s) {
                int e = idx[(size_t)t * K + s];
                if (e < 0 || e >= cfg->num_experts) continue;
                float wt = weights[(size_t)t * K + s];
                expert_mlp_one(cfg, w, e, mode, n, nq, nql, ns, lut, hbuf, hq, hql, hs, y);
                for (int i = 0; i < H; ++i) acc[i] = fmaf(wt, y[i], acc[i]);
            }
            for (int i = 0; i < H; ++i) out_bf16[(size_t)t * H + i] = orc_f32_to_bf16(acc[i]);
        }
        free(xf); free(acc); free(y); free(hbuf); free(hq); free(hql); free(hs); free(nq); free(nql); free(ns);
    }
}

static float* normed_rows(const orc_moe_cfg* cfg, const orc_moe_weights* w,
                          const uint16_t* x_bf16, int tokens) {
    const int H = cfg->hidden;
    float* xf = (float*)malloc(sizeof(float) * (size_t)tokens * H);
    float* n = (float*)malloc(sizeof(float) * (size_t)tokens * H);
    for (size_t i = 0; i < (size_t)tokens * H; ++i) xf[i] = orc_bf16_to_f32(x_bf16[i]);
    orc_rmsnorm_ref(xf, w->gamma, n, H, tokens, cfg->eps);
    free(xf);
    return n;
}

void orc_moe_ffn_forward(const orc_moe_cfg* cfg, const orc_moe_weights* w,
                         const uint16_t* x_bf16, uint16_t* out_bf16, int tokens,
                         int mode, int32_t* idx_out, float* weights_out,
                         float* logits_out, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
    const int E = cfg->num_experts, K = cfg->top_k;
    float* n = normed_rows(cfg, w, x_bf16, tokens);
    float* logits = (float*)malloc(sizeof(float) * (size_t)tokens * E);
    int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * (size_t)tokens * K);
    float* wts = (float*)malloc(sizeof(float) * (size_t)tokens * K);
    orc_moe_router_logits(n, w->router_w, w->router_bias, logits, cfg->hidden, E, tokens);
    orc_moe_topk_ref(logits, idx, wts, E, K, tokens);
    ffn_experts_impl(cfg, w, x_bf16, n, idx, wts, out_bf16, tokens, mode, threads);
    if (idx_out) memcpy(idx_out, idx, sizeof(int32_t) * (size_t)tokens * K);
    if (weights_out) memcpy(weights_out, wts, sizeof(float) * (size_t)tokens * K);
    if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)tokens * E);
    free(n); free(logits); free(idx); free(wts);
}

void orc_moe_ffn_experts(const orc_moe_cfg* cfg, const orc_moe_weights* w,
                         const uint16_t* x_bf16, const int32_t* idx,
                         const float* weights, uint16_t* out_bf16, int tokens,
                         int mode, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
    float* n = normed_rows(cfg, w, x_bf16, tokens);
    ffn_experts_impl(cfg, w, x_bf16, n, idx, weights, out_bf16, tokens, mode, threads);
    free(n);
}
