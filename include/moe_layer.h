/*
 * moe_layer.h -- B200-native MoE FFN block of a GLM-4.x decoder layer.
 *
 * These entry points have no counterpart in the reference's C-ABI: the
 * reference's libkernels/libcublaswrap cannot express block-scaled FP8,
 * grouped expert GEMMs, bf16 activations or expert parallelism
 * (csrc/kernels.h:12-31, csrc/cublas_wrappers.h:51-67).  They replace the MoE
 * branch of the reference's layer forward, src/terra/engine.t:1310-1369
 * (post-attention RMSNorm -> moe_gate -> moe_topk -> moe_dispatch -> per-slot
 * dequant + SGEMM gate/up -> swiglu -> dequant + SGEMM down -> moe_combine ->
 * add_residual), whose intended semantics are spelled out in
 * src/futhark/kernels.fut:324-368 (moe_router, moe_expert_mlp, moe_forward).
 *
 * Conventions
 *   - Plain pointers and sizes only.  Device pointers unless stated.  The
 *     caller owns every buffer; nothing here allocates device memory except
 *     moe_layer_create (its handle's small state) -- the forward takes a
 *     caller-provided workspace.
 *   - Layouts are row-major.  Activations: [tokens][hidden] bf16.  Weights
 *     are [out][in] (K-major) e4m3 bytes with fp32 block scales over 128x128
 *     blocks, scale layout [out/128][in/128] per expert ("weight_scale_inv"
 *     convention: real weight = decode(q) * scale).
 *   - Streams are cwStream_t (a cudaStream_t, cuda_wrappers.h).
 *   - Every function returns an moe_status_t; 0 is success.  A device-side
 *     wait that gave up (no progress for ~2 s) is reported as
 *     MOE_ERR_DEVICE_TIMEOUT by moe_layer_check_error / the forward.
 */
#ifndef MOE_LAYER_H
#define MOE_LAYER_H

#include <stdint.h>
#include <stddef.h>
#include "cuda_wrappers.h"
#include "nccl_wrappers.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    MOE_OK = 0,
    MOE_ERR_INVALID_ARGUMENT = 1,
    MOE_ERR_CUDA = 2,
    MOE_ERR_UNSUPPORTED = 3,
    MOE_ERR_DEVICE_TIMEOUT = 4,
    MOE_ERR_NCCL = 5,
    MOE_ERR_WORKSPACE = 6
} moe_status_t;

const char* moe_status_string(moe_status_t status);

/* ------------------------------------------------------------------ layer */

typedef struct {
    int hidden;          /* H, multiple of 128 */
    int num_experts;     /* E routed experts (global) */
    int top_k;           /* 1..16 */
    int intermediate;    /* I, multiple of 128 */
    int num_shared;      /* 0 or 1 shared expert */
    float rms_eps;       /* post-attention RMSNorm epsilon */
    int max_tokens;      /* tokens per forward call on this rank */
    int ep_size;         /* expert-parallel ranks (1 = single GPU) */
    int ep_rank;         /* this rank; owns experts [r*E/ep, (r+1)*E/ep) */
} moe_layer_config_t;

typedef struct {
    const float* norm_gamma;   /* [H] fp32 */
    const float* router_w;     /* [E][H] fp32 (all experts, replicated) */
    const float* router_bias;  /* [E] fp32 or NULL, added to the logits */
    /* Local experts first (E/ep_size of them, in global order), then the
     * shared expert if num_shared == 1.  Gate rows [0,I) then up rows [I,2I). */
    const void* w13;           /* [E_local+S][2I][H] e4m3 */
    const float* s13;          /* [E_local+S][2I/128][H/128] */
    const void* w2;            /* [E_local+S][H][I] e4m3 */
    const float* s2;           /* [E_local+S][H/128][I/128] */
} moe_layer_weights_t;

typedef struct moe_layer moe_layer_t;

/* Validates the shapes and allocates the handle's small state (device error
 * word; with ep_size > 1 a pinned host buffer for the exchanged counts).
 * `comm` is an ncwComm_t over the ep_size ranks, rank ep_rank being this
 * process (NULL when ep_size == 1, or when the peer-memory exchange is used:
 * a forward with ep_size > 1 and neither a communicator nor peer buffers
 * returns MOE_ERR_INVALID_ARGUMENT).  Weight pointers must stay valid.  With
 * ep_size > 1 every rank must call the forward with the same max_tokens and
 * may pass at most max_tokens tokens. */
moe_status_t moe_layer_create(const moe_layer_config_t* cfg, const moe_layer_weights_t* w,
                              ncwComm_t comm, moe_layer_t** out);
moe_status_t moe_layer_destroy(moe_layer_t* layer);

/* Workspace the forward needs for max_tokens tokens (bytes). */
size_t moe_layer_workspace_bytes(const moe_layer_t* layer);

/* out = x + MoE(RMSNorm(x)) for `num_tokens` <= max_tokens tokens:
 *   RMSNorm (reference order) -> router logits (fp32) -> top-k (reference
 *   tie-break) -> stable expert permutation -> FP8 1x128 activation quant ->
 *   grouped block-scaled FP8 gate/up GEMM + SwiGLU + FP8 requant -> grouped
 *   down GEMM (bf16) -> weighted combine + shared expert + residual (bf16).
 * x and out may not alias.  Stream-ordered; no host synchronisation when
 * ep_size == 1 or with peer buffers set (moe_layer_set_peer_buffers).  With
 * the NCCL exchange (ep_size > 1, no peer buffers) the per-peer token counts
 * are read back once per call (one host sync). */
moe_status_t moe_layer_forward(moe_layer_t* layer, const void* x_bf16, void* out_bf16,
                               int num_tokens, void* workspace, size_t workspace_bytes,
                               cwStream_t stream);

/* Same, with the routing supplied by the caller ([T][top_k] expert ids and
 * weights on the device) instead of computed from router_w. */
moe_status_t moe_layer_forward_routed(moe_layer_t* layer, const void* x_bf16,
                                      const int32_t* topk_idx, const float* topk_w,
                                      void* out_bf16, int num_tokens, void* workspace,
                                      size_t workspace_bytes, cwStream_t stream);

/* Routing of the last forward (device pointers into the workspace):
 * topk_idx [T][k] int32, topk_w [T][k] fp32, counts [E_local+S] int32. */
moe_status_t moe_layer_last_routing(const moe_layer_t* layer, const void* workspace,
                                    const int32_t** topk_idx, const float** topk_w,
                                    const int32_t** group_counts);

/* Stage timing: when `events` is non-NULL, every later forward records
 * events[i] on its stream right before stage i and events[MOE_NUM_STAGES]
 * after the last one (stages: 0 RMSNorm+quant, 1 router+top-k, 2 permute,
 * 3 gather, 4 gate/up GEMM, 5 down GEMM, 6 combine; a routed forward records
 * an empty router stage).  Pass NULL to stop.  The events stay owned by the
 * caller. */
#define MOE_NUM_STAGES 7
moe_status_t moe_layer_set_stage_events(moe_layer_t* layer, cwEvent_t* events);

/* Expert parallelism over NVLink peer memory instead of NCCL.  Every rank
 * allocates one buffer of moe_layer_peer_bytes() bytes that all ranks map
 * (CUDA IPC / a symmetric-memory allocator), zero-fills it, and -- after every
 * rank has zero-filled its own -- passes the n = ep_size pointers as mapped in
 * this process (peer_bufs[ep_rank] is its own, 256-byte aligned).  From then on
 * the forward exchanges counts, rows and outputs with its own kernels (P2P
 * stores, system-scope flags with bounded waits): no NCCL call and no host
 * synchronisation; a peer that stops answering ends the waits after at most
 * 20 s with MOE_ERR_DEVICE_TIMEOUT from moe_layer_check_error.  NULL switches
 * back to the NCCL exchange.  0 bytes when ep_size == 1. */
size_t moe_layer_peer_bytes(const moe_layer_t* layer);
moe_status_t moe_layer_set_peer_buffers(moe_layer_t* layer, void* const* peer_bufs, int n);

/* Which rank computes which routed expert (ep_size > 1).  slot_of_expert
 * (host, [E]) is a permutation of 0..E-1: expert e is computed by rank
 * slot / (E/ep_size) as its local expert slot % (E/ep_size); the rank's w13 /
 * s13 / w2 / s2 then hold its experts in local-slot order (then the shared
 * expert).  Every rank must set the same permutation.  The default is the
 * contiguous placement of the spec's shard_experts (slot = e); a placement
 * that spreads the frequently routed experts evens the ranks' work.  Outputs
 * do not change: every expert row is computed the same way wherever it runs.
 * Copies the table to the device (the one allocation, freed by
 * moe_layer_destroy); NULL restores the contiguous placement. */
moe_status_t moe_layer_set_expert_placement(moe_layer_t* layer, const int32_t* slot_of_expert);

/* No counterpart in the reference.  Which form of the grouped GEMM the
 * forward runs: CBW_GEMM_SMALL_TILES (the decode form), CBW_GEMM_FULL_TILES,
 * or 0 for the default rule -- the decode form when the call averages at most
 * 16 routed tokens per expert, counting max_tokens x ep_size tokens when
 * ep_size > 1 (the same count on every rank) and the call's tokens on one
 * GPU.  The two forms add a row's K blocks in different orders, so outputs
 * differ in the last bits between them; an expert-parallel layer and a
 * one-GPU layer give bit-identical outputs when they run the same form.
 * CBW_GEMM_ONE_SM_TILES, CBW_GEMM_PAIR_TILES or CBW_GEMM_TOKEN_TILES force
 * that variant of the full form on both GEMMs (bit-identical to one another;
 * a GEMM whose shape or activation format has no such variant fails the
 * forward with MOE_ERR_INVALID_ARGUMENT). */
moe_status_t moe_layer_set_gemm_form(moe_layer_t* layer, int form);

/* No counterpart in the reference.  Activation format of the two expert
 * GEMMs: planes = 1 (e4m3 with one scale per 1x128 block, as FP8 serving
 * stacks run it) or planes = 2 (two-term e4m3, hi + lo residual with the same
 * scale -- CBW_GEMM_ACT_X2: twice the tensor-core work, about 7 significant
 * bits per activation instead of 4, which keeps the layer within the
 * tolerance of an fp32-activation evaluation).  The workspace size depends on
 * it: query moe_layer_workspace_bytes after setting it.  With expert
 * parallelism the dispatched rows carry both planes (moe_ep_row_bytes(H) + H
 * bytes), so set it before moe_layer_peer_bytes / moe_layer_set_peer_buffers
 * (changing it afterwards returns MOE_ERR_INVALID_ARGUMENT). */
moe_status_t moe_layer_set_act_planes(moe_layer_t* layer, int planes);
moe_status_t moe_layer_get_act_planes(const moe_layer_t* layer, int* planes);

/* Reads and clears the device error word (synchronises `stream`). */
moe_status_t moe_layer_check_error(moe_layer_t* layer, cwStream_t stream);

/* -------------------------------------------------------------- components
 * The stages of the forward, exposed for the engine and for parity tests.
 * T = tokens, H = hidden, E = experts, k = top_k, G = groups (experts + shared).
 */

/* Per token: rms = sqrtf(sum(x^2)/H + eps) with the reference's reduction
 * order (csrc/kernels.cu:61-85); n = (x / rms) * gamma (fp32); then n is
 * quantised per 128-column block: xq = e4m3_rne(n * 448/amax),
 * xs[blk][t] = amax/448 (xs is [H/128][xs_ld]).  rms_out may be NULL. */
moe_status_t moe_rmsnorm_quant(const void* x_bf16, const float* gamma, int T, int H, float eps,
                               float* rms_out, void* xq_out, float* xs_out, int xs_ld,
                               cwStream_t stream);

/* moe_rmsnorm_quant that also stores n = (x/rms)*gamma in fp32 ([T][H],
 * 16-byte aligned) when n_out is not NULL -- the router's input. */
moe_status_t moe_rmsnorm_quant_n(const void* x_bf16, const float* gamma, int T, int H, float eps,
                                 float* rms_out, float* n_out, void* xq_out, float* xs_out,
                                 int xs_ld, cwStream_t stream);

/* Router logits from the stored n in the reference's summation order
 * (csrc/kernels.cu:412-435 with blockDim 256): for each (t, e) the 256 lane
 * partials p[l] = fma-chain over i = l, l+256, ... of n[t][i]*W[e][i] from
 * +0.0f, reduced by the pairwise tree p[l] += p[l+s], s = 128..1, then
 * + bias[e] -- bit-identical to the reference's kernel_moe_gate and to the
 * logits moe_router_topk computes; H a multiple of 128, E <= 256. */
moe_status_t moe_router_logits(const float* n, const float* router_w, const float* router_bias,
                               int T, int H, int E, float* logits, cwStream_t stream);

/* No counterpart in the reference.  The "router column order" of a [rows][H]
 * fp32 matrix (H a multiple of 256, J = H/256): element i = 256j + 32m + 4q + r
 * (r = 2*r_hi + r_lo) of a row is stored at column
 *     r_lo*128J + m*16J + 16j + 8*r_hi + q,
 * which groups the lanes of the reference's reduction so that the layer's
 * router streams long contiguous runs and splits the lanes over a CTA pair
 * at the last tree level.  moe_router_columns writes src in that order to
 * dst (no aliasing); moe_rmsnorm_quant_rc is moe_rmsnorm_quant_n with n
 * (required) written in that order; moe_router_logits_rc takes n and W in
 * that order and returns exactly the logits of moe_router_logits on the
 * plain matrices (E <= 256). */
moe_status_t moe_router_columns(const float* src, float* dst, int rows, int H, cwStream_t stream);
moe_status_t moe_rmsnorm_quant_rc(const void* x_bf16, const float* gamma, int T, int H, float eps,
                                  float* rms_out, float* n_rc_out, void* xq_out, float* xs_out,
                                  int xs_ld, cwStream_t stream);
moe_status_t moe_router_logits_rc(const float* n_rc, const float* w_rc, const float* router_bias,
                                  int T, int H, int E, float* logits, cwStream_t stream);

/* No counterpart in the reference.  Two-term e4m3 activations ("x2", the
 * input format of CBW_GEMM_ACT_X2): per 128-column block one scale s =
 * amax/448 and two e4m3 planes, hi = e4m3_rne(v/s) (the same bytes as the
 * one-plane quantisation) and lo = e4m3_rne(v/s - decode(hi)), so that
 * v ~= s * (decode(hi) + decode(lo)) with about 7 significant bits.
 * moe_rmsnorm_quant_x2 is moe_rmsnorm_quant_n (n_router_cols = 0) or
 * moe_rmsnorm_quant_rc (n_router_cols = 1) that also writes the lo plane
 * ([T][H], xq_lo_out, required); n_out may be NULL with n_router_cols = 0.
 * moe_gather_rows_x2 is moe_gather_rows that also moves the lo plane
 * (xq_lo and xp_lo both given, or both NULL); total_rows (device, may be
 * NULL) bounds the rows written. */
moe_status_t moe_rmsnorm_quant_x2(const void* x_bf16, const float* gamma, int T, int H, float eps,
                                  float* rms_out, float* n_out, int n_router_cols, void* xq_out,
                                  void* xq_lo_out, float* xs_out, int xs_ld, cwStream_t stream);
moe_status_t moe_gather_rows_x2(const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                                const int32_t* row_token, const int32_t* total_rows, int row_capacity,
                                int H, void* xp, void* xp_lo, float* xps, int xps_ld, cwStream_t stream);

/* The rows of moe_gather_rows_x2, written token by token: token t's row
 * (planes and scales) goes to each of its routed rows pos[t*k + s] >= 0 and to
 * its shared-expert rows shared_start[g] + t (g < num_shared <= 2; device
 * array); rows with row_token < 0 are zeroed.  xp, xp_lo and xps end up
 * identical to moe_gather_rows_x2's for the same permutation, with each token
 * read once.  k <= 16. */
moe_status_t moe_scatter_rows_x2(const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                                 const int32_t* pos, int T, int k, const int32_t* shared_start,
                                 int num_shared, const int32_t* row_token, const int32_t* total_rows,
                                 int row_capacity, int H, void* xp, void* xp_lo, float* xps, int xps_ld,
                                 cwStream_t stream);

/* Top-k + weights of given logits [T][E] with the same rule as
 * moe_router_topk. */
moe_status_t moe_topk_softmax(const float* logits, int T, int E, int k, int32_t* topk_idx,
                              float* topk_w, cwStream_t stream);

/* No counterpart in the reference.  moe_router_logits followed by
 * moe_topk_softmax for callers that cannot provide device memory beyond their
 * inputs and outputs -- an engine that carves all of its device memory out of
 * its own arena at start-up, or a plain C / FFI host that must not call
 * cudaMalloc on its hot path (it synchronises the whole device).  The [T][E]
 * fp32 logits between the two kernels live in a fixed array inside this
 * library (4 MB on every GPU that loads it, held until the process exits);
 * the call allocates nothing.  Same results, bit for bit, as the two-call
 * path.  Limits and rules:
 *   - T * E <= 1048576 (e.g. 4096 tokens x 256 experts); larger requests
 *     return MOE_ERR_WORKSPACE and launch nothing.
 *   - The first call on a device looks up the array's device address for
 *     that device (make it before any stream capture on that device).
 *   - Every call on a device uses the same array: calls that can overlap on
 *     the GPU (different streams without ordering between them) race.  No
 *     part of the array needs to start at zero: every logit read is first
 *     written by the same call. */
moe_status_t moe_router_topk_noalloc(const float* n, const float* router_w,
                                     const float* router_bias, int T, int H, int E, int k,
                                     int32_t* topk_idx, float* topk_w, cwStream_t stream);

/* Router: the logits of moe_router_logits (reference summation order),
 * n recomputed from x, rms, gamma exactly as above; then the
 * reference's top-k (strict '>' from -FLT_MAX: lower index wins ties, NaN
 * never chosen; csrc/kernels.cu:437-471) and weights exp(v)/sum exp(v) over
 * the selected slots (max-subtracted when the top logit exceeds 80).
 * logits_out may be NULL. */
moe_status_t moe_router_topk(const void* x_bf16, const float* rms, const float* gamma,
                             const float* router_w, const float* router_bias,
                             int T, int H, int E, int k,
                             float* logits_out, int32_t* topk_idx, float* topk_w,
                             cwStream_t stream);

/* Stable counting sort of the (token, slot) pairs by expert id (the pair
 * order t*k+s is kept within an expert), experts [e_begin, e_end) only,
 * followed by `num_shared` groups holding every token in order.  Segments
 * start at multiples of 16 rows.  Outputs (device): counts[G], seg_start[G],
 * pos[T*k] (row of each pair, -1 when its expert is not local or invalid),
 * row_token[row_capacity] (token of each row, -1 for padding/unused rows),
 * total_rows[1].  Fails on the device (error word) if row_capacity is too
 * small. */
moe_status_t moe_permute(const int32_t* topk_idx, int T, int k, int e_begin, int e_end,
                         int num_shared, int32_t* counts, int32_t* seg_start, int32_t* pos,
                         int32_t* row_token, int32_t* total_rows, int row_capacity,
                         int* error_word, cwStream_t stream);

/* xp[r] = xq[row_token[r]] (zero row when row_token[r] < 0) and
 * xps[blk][r] = xs[blk][row_token[r]] for r < row_capacity. */
moe_status_t moe_gather_rows(const void* xq, const float* xs, int xs_ld, const int32_t* row_token,
                             int row_capacity, int H, void* xp, float* xps, int xps_ld,
                             cwStream_t stream);

/* out[t] = bf16( x[t] + sum_{shared g} y[seg_start[g]+t]
 *               + sum_s w[t][s] * y[pos[t*k+s]] )   (pos < 0 skipped).
 * The additions run in that order in fp32 (fma for the weighted terms). */
moe_status_t moe_combine(const void* x_bf16, const void* y_bf16, const int32_t* pos,
                         const float* topk_w, const int32_t* shared_rows, int num_shared,
                         int T, int k, int H, void* out_bf16, cwStream_t stream);

/* moe_permute with segment starts aligned to `pad` rows (1..128) instead of
 * 16; pad = 1 gives the dense expert-sorted order the EP dispatch sends. */
moe_status_t moe_permute_padded(const int32_t* topk_idx, int T, int k, int e_begin, int e_end,
                                int num_shared, int32_t* counts, int32_t* seg_start, int32_t* pos,
                                int32_t* row_token, int32_t* total_rows, int row_capacity,
                                int* error_word, int pad, cwStream_t stream);

/* moe_permute_padded spread over many blocks (one 256-pair block per slice
 * of the pairs, a scan block, a scatter pass): identical outputs, for large
 * T*k.  `scratch` (device, moe_permute_mb_scratch_bytes(T, k, e_begin, e_end)
 * bytes) holds per-block counts.  On refusal (row_capacity too small)
 * total_rows is -1, counts are zero and the error word is 2. */
size_t moe_permute_mb_scratch_bytes(int T, int k, int e_begin, int e_end);
moe_status_t moe_permute_mb(const int32_t* topk_idx, int T, int k, int e_begin, int e_end,
                            int num_shared, int32_t* counts, int32_t* seg_start, int32_t* pos,
                            int32_t* row_token, int32_t* total_rows, int row_capacity,
                            int* error_word, int pad, void* scratch, size_t scratch_bytes,
                            cwStream_t stream);

/* moe_combine with the shared expert's rows read from y_shared_bf16 (at
 * shared_rows[g] + t) and the routed rows from y_bf16 (at pos). */
moe_status_t moe_combine_split(const void* x_bf16, const void* y_bf16, const int32_t* pos,
                               const float* topk_w, const void* y_shared_bf16,
                               const int32_t* shared_rows, int num_shared, int T, int k, int H,
                               void* out_bf16, cwStream_t stream);

/* ------------------------------------------------------ expert parallelism
 * Rank r of ep_size owns routed experts [r*E/ep, (r+1)*E/ep) (the spec's
 * shard_experts, src/futhark/kernels.fut:640-647) and tokens of its own; the
 * exchange is the spec's all_to_all (kernels.fut:612-617) done with
 * ncwAllToAllv.  A dispatched row is "packed": H e4m3 bytes, H/128 fp32
 * scales, zero padding to moe_ep_row_bytes(H) bytes. */

/* Bytes of one packed row (0 if H is not a positive multiple of 128). */
size_t moe_ep_row_bytes(int H);

/* Host-side plan of both all-to-alls.  send_expert_counts[E] = this rank's
 * pairs per global expert (E = ep_size * experts_per_rank); recv_counts
 * [ep_size][experts_per_rank] = rows peer p sends for each local expert.
 * Outputs per peer (arrays of ep_size): rows sent/received and their
 * first-row offsets in the dense send/receive buffers, plus both totals
 * (either total pointer may be NULL). */
moe_status_t moe_ep_plan_host(int ep_size, int experts_per_rank, const int32_t* send_expert_counts,
                              const int32_t* recv_counts, size_t* send_rows, size_t* send_offsets,
                              size_t* recv_rows, size_t* recv_offsets, size_t* send_total,
                              size_t* recv_total);

/* packed[r] = (xq[row_token[r]], xs[:, row_token[r]]) for r < *num_rows
 * (num_rows on the device, clamped to row_capacity). */
moe_status_t moe_ep_pack_rows(const void* xq, const float* xs, int xs_ld, const int32_t* row_token,
                              const int32_t* num_rows, int row_capacity, int H, void* packed,
                              cwStream_t stream);

/* From recv_counts[ep_size][experts_per_rank] (device) build the local GEMM
 * row layout: local expert j's segment holds the rows of source 0, 1, ... in
 * their received order, segments start at multiples of 16, and `num_shared`
 * (0 or 1) shared-expert segment of T_local rows follows.  Outputs (device):
 * counts[G], seg_start[G], total_rows[1], row_src[row_capacity] (received row,
 * -1 padding, -(t+2) own token t) and recv_dst[received rows] (GEMM row of
 * every received row).  Over capacity: zero counts and error word 2. */
moe_status_t moe_ep_recv_plan(const int32_t* recv_counts, int ep_size, int experts_per_rank,
                              int T_local, int num_shared, int32_t* counts, int32_t* seg_start,
                              int32_t* total_rows, int32_t* row_src, int32_t* recv_dst,
                              int row_capacity, int recv_capacity, int* error_word,
                              cwStream_t stream);

/* GEMM input rows: xp[r] / xps[:, r] from packed row row_src[r] (>= 0), from
 * own token -(row_src[r]+2) of xq/xs (<= -2), or zeros (-1); r < *total_rows. */
moe_status_t moe_ep_gather(const void* packed, const void* xq, const float* xs, int xs_ld,
                           const int32_t* row_src, const int32_t* total_rows, int row_capacity,
                           int H, void* xp, float* xps, int xps_ld, cwStream_t stream);

/* No counterpart in the reference.  moe_ep_pack_rows / moe_ep_gather for
 * two-term activations: a packed row is the hi plane's H bytes, the lo
 * plane's H bytes, then the scales (moe_ep_row_bytes(H) + H bytes); xq_lo /
 * xp_lo are the lo planes ([T][H] / [rows][H]; for the gather both given or
 * both NULL, NULL meaning one plane). */
moe_status_t moe_ep_pack_rows_x2(const void* xq, const void* xq_lo, const float* xs, int xs_ld,
                                 const int32_t* row_token, const int32_t* num_rows, int row_capacity,
                                 int H, void* packed, cwStream_t stream);
moe_status_t moe_ep_gather_x2(const void* packed, const void* xq, const void* xq_lo, const float* xs,
                              int xs_ld, const int32_t* row_src, const int32_t* total_rows,
                              int row_capacity, int H, void* xp, void* xp_lo, float* xps, int xps_ld,
                              cwStream_t stream);

/* vidx[p] = slot_of_expert[topk_idx[p]] for 0 <= topk_idx[p] < E, else -1
 * (num_pairs = T * k; device arrays). */
moe_status_t moe_ep_remap_experts(const int32_t* topk_idx, int num_pairs, int E,
                                  const int32_t* slot_of_expert, int32_t* vidx, cwStream_t stream);

/* The peer exchange's per-destination numbering (one packed row per token
 * and destination rank): for every rank d < ep_size, this rank's tokens with
 * at least one pair whose expert id v (vidx, [T][k], -1 = none) lives on d
 * (v / experts_per_rank == d), in token order.  Outputs (device):
 * uidx [ep_size][T] (the token's row number for d, -1 when none),
 * utok [ep_size][T] (the token of each row number; entries past ucount[d]
 * are left as they were), ucount [ep_size].  ep_size <= 64. */
moe_status_t moe_ep_token_rows(const int32_t* vidx, int T, int k, int ep_size, int experts_per_rank,
                               int32_t* uidx, int32_t* utok, int32_t* ucount, cwStream_t stream);

/* ysend[i] = y[recv_dst[i]] for i < n (bf16 rows of H). */
moe_status_t moe_ep_pack_y(const void* y_bf16, const int32_t* recv_dst, int n, int H,
                           void* ysend_bf16, cwStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_LAYER_H */
