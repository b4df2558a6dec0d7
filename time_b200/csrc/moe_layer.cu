// moe_layer.cu -- the MoE FFN block forward (include/moe_layer.h): owns the
// workspace layout and issues the stage kernels in stream order.  Replaces
// the MoE branch of src/terra/engine.t:1310-1369.
//
// Data layout in HBM for one call (T tokens, G = local experts + shared):
//   rms        [T] f32
//   n          [T][H] f32          RMSNorm output (the router's input)
//   logits     [T][E] f32          router logits
//   xq         [T][H] e4m3         token order, 1x128-quantised RMSNorm output
//   xs         [H/128][T_ld] f32   its scales (transposed: one K block's scales
//                                  of consecutive rows are contiguous, so the
//                                  GEMM fetches them with one bulk copy)
//   topk_idx   [T][k] i32, topk_w [T][k] f32
//   counts/seg_start [G] i32, total_rows [1] i32, pos [T*k] i32
//   row_token  [R_cap] i32         token of every expert-ordered row
//   xp         [R_cap][H] e4m3     rows grouped by expert, segments padded to 16
//   xps        [H/128][R_cap] f32
//   hq         [R_cap][I] e4m3     SwiGLU output, 1x128-quantised
//   hs         [I/128][R_cap] f32
//   y          [R_cap][H] bf16     expert outputs
// R_cap = T*k + S*T + 16*G rounded up to 16: every assignment plus the shared
// expert's T rows plus worst-case segment padding.
//
// With expert parallelism (ep_size > 1, the exchange is described in
// moe_ep.cu) the workspace also holds, for T_r = max_tokens own tokens and
// recv_cap = ep * T_r * min(k, E/ep) received rows (every peer's every token
// routed here as often as it can be):
//   ecounts/rcounts [E] + [E] i32  pairs sent per global expert / received
//                                  per (source, local expert); one D2H copy
//   estart [E], stotal, spos [T*k], stok [T*k]   the dense send order
//   psend  [T*k][rb] / precv [recv_cap][rb]      packed rows (rb bytes each)
//   row_src [R_cap], recv_dst [recv_cap]          received row <-> GEMM row
//   ysend  [recv_cap][H] bf16 / yrecv [T*k][H] bf16  combine exchange
//   row_out [R_cap] pointers        peer exchange: each GEMM row's output
//                                  address (the owner's yrecv slot or local y)
//   uidx/utok [ep][T] i32, ucount [ep]  peer exchange: this rank's tokens
//                                  with a pair for each destination rank
// and R_cap = recv_cap + S*T + 16*G (rounded to 16).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "cublas_wrappers.h"
#include "moe_layer.h"
#include "moe_ep_peer.h"

extern "C" moe_status_t moe_gather_rows_n(const void* xq, const float* xs, int xs_ld, const int32_t* row_token,
                                          const int32_t* total_rows, int row_capacity, int H, void* xp, float* xps,
                                          int xps_ld, cwStream_t stream);

struct moe_layer {
    moe_layer_config_t cfg;
    moe_layer_weights_t w;
    ncwComm_t comm;
    int e_begin, e_end, groups;
    int* error_word;      // device
    cudaEvent_t stage_ev[MOE_NUM_STAGES + 1];
    bool timing;
    // workspace layout (byte offsets)
    size_t off_bcounts, bcounts_bytes;
    size_t off_wrc = 0;   // router weight in the router column order (H % 256 == 0)
    size_t off_rms, off_n, off_logits, off_xq, off_xs, off_idx, off_w, off_counts, off_start, off_total, off_pos, off_rowtok,
        off_xp, off_xps, off_hq, off_hs, off_y, bytes;
    int xs_ld, rcap;
    // expert parallelism
    size_t off_ecounts, off_estart, off_stotal, off_stok, off_psend, off_precv, off_rdst, off_ysend, off_yrecv;
    size_t off_uidx, off_utok, off_ucount;   // peer exchange: tokens per destination rank
    size_t row_bytes, off_vidx;
    int recv_cap;
    int32_t* h_counts;    // pinned [2E]
    int sync_timeout_ms;
    // peer-memory exchange (moe_layer_set_peer_buffers)
    bool peer_mode;
    int32_t* slot_of_expert;   // device [E] or NULL (contiguous placement)
    tbep::Peers peers;
    uint32_t* epoch_dev;   // peer exchange: the forward counter, on the device
    size_t off_plan;
    // peer exchange, TIME_B200_EP_FUSED_RETURN=1: the down GEMM stores each
    // received row's output straight into its token owner's return buffer
    // instead of a copy kernel after the GEMM.  Off by default: at EP 2 (GLM
    // shape, 4096 tokens) the epilogue's stores over NVLink hold the GEMM's
    // TMEM buffers and the down GEMM takes 0.72 ms against 0.41 ms + a
    // 0.14 ms copy.
    bool fused_return = false;
    size_t off_rowout = 0;   // [rcap] output row addresses of the down GEMM
    int gemm_form;        // 0 = by the rule in gemm_form(), else a CBW_GEMM_*_TILES flag
    int act_planes = 1;   // 1: e4m3 activations; 2: two-term e4m3 (hi + lo residual)
    size_t off_xq_lo = 0;  // [T][H] lo plane of xq (act_planes == 2)
};

namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

void plan_workspace(moe_layer* L) {
    const moe_layer_config_t& c = L->cfg;
    const size_t T = static_cast<size_t>(c.max_tokens);
    const size_t H = c.hidden, I = c.intermediate, K = c.top_k;
    const bool ep = c.ep_size > 1;
    const size_t epr = static_cast<size_t>(c.num_experts / c.ep_size);
    L->xs_ld = static_cast<int>(align_up(T, 4));
    L->recv_cap = ep ? static_cast<int>(static_cast<size_t>(c.ep_size) * T * std::min(K, epr)) : 0;
    const size_t routed_rows = ep ? static_cast<size_t>(L->recv_cap) : T * K;
    L->rcap = static_cast<int>(align_up(routed_rows + static_cast<size_t>(c.num_shared) * T + 16 * static_cast<size_t>(L->groups), 16));
    L->row_bytes = moe_ep_row_bytes(c.hidden) + (L->act_planes == 2 ? static_cast<size_t>(c.hidden) : 0);
    const size_t R = L->rcap;
    size_t o = 0;
    auto take = [&o](size_t bytes) { size_t at = o; o = align_up(o + bytes, 256); return at; };
    L->off_rms = take(T * 4);
    L->bcounts_bytes = moe_permute_mb_scratch_bytes(static_cast<int>(T), c.top_k, 0, c.num_experts);
    L->off_bcounts = take(L->bcounts_bytes);
    L->off_n = take(T * H * 4);
    L->off_logits = take(T * static_cast<size_t>(c.num_experts) * 4);
    if (H % 256 == 0) L->off_wrc = take(static_cast<size_t>(c.num_experts) * H * 4);
    L->off_xq = take(T * H);
    if (L->act_planes == 2) L->off_xq_lo = take(T * H);
    L->off_xs = take((H / 128) * L->xs_ld * 4);
    L->off_idx = take(T * K * 4);
    L->off_w = take(T * K * 4);
    L->off_counts = take(L->groups * 4);
    L->off_start = take(L->groups * 4);
    L->off_total = take(16);
    L->off_pos = take(T * K * 4);
    L->off_rowtok = take(R * 4);
    L->off_xp = take(R * H * L->act_planes);     // [planes][R][H]: the lo plane R*H bytes on
    L->off_xps = take((H / 128) * R * 4);
    L->off_hq = take(R * I * L->act_planes);     // [planes][R][I]
    L->off_hs = take((I / 128) * R * 4);
    L->off_y = take(R * H * 2);
    if (ep) {
        const size_t E = c.num_experts, RC = L->recv_cap;
        L->off_ecounts = take(2 * E * 4);
        L->off_estart = take(E * 4);
        L->off_stotal = take(16);
        L->off_stok = take(T * K * 4);
        L->off_psend = take(T * K * L->row_bytes);
        L->off_precv = take(RC * L->row_bytes);
        L->off_rdst = take(RC * 4);
        L->off_ysend = take(RC * H * 2);
        L->off_yrecv = take(T * K * H * 2);
        L->off_plan = take(tbep::plan_ints(c.ep_size) * 4);
        L->off_vidx = take(T * K * 4);
        L->off_rowout = take(R * sizeof(void*));
        L->off_uidx = take(static_cast<size_t>(c.ep_size) * T * 4);
        L->off_utok = take(static_cast<size_t>(c.ep_size) * T * 4);
        L->off_ucount = take(static_cast<size_t>(c.ep_size) * 4);
    }
    L->bytes = o;
}

template <typename T>
T* at(void* ws, size_t off) { return reinterpret_cast<T*>(static_cast<char*>(ws) + off); }

inline void mark(moe_layer* L, int stage, cudaStream_t st) {
    if (L->timing) cudaEventRecord(L->stage_ev[stage], st);
}

moe_status_t cbw_to_moe(cbwStatus_t s) {
    return s == CBW_SUCCESS ? MOE_OK : (s == CBW_ERROR_INVALID_VALUE ? MOE_ERR_INVALID_ARGUMENT : MOE_ERR_CUDA);
}

#define MOE_TRY(expr)                      \
    do {                                   \
        moe_status_t _s = (expr);          \
        if (_s != MOE_OK) return _s;       \
    } while (0)

moe_status_t nccl_to_moe(ncwResult_t r) { return r == NCW_SUCCESS ? MOE_OK : MOE_ERR_NCCL; }

// The grouped GEMM's decode form (32-row tiles whose K blocks the promotion
// groups share) when a call averages at most 16 routed tokens per expert over
// all ranks (tokens x top_k <= 16 x E).  The two forms add a row's K blocks in
// different orders, so every rank of an expert-parallel call must make the
// same choice: with ep_size > 1 the rule counts max_tokens x ep_size tokens
// (max_tokens is the same on every rank), never the rank's own token count,
// which differs between ranks when the tokens do not split evenly.  A single
// GPU counts the call's tokens.  moe_layer_set_gemm_form overrides the rule.
// One expert (a dense FFN as one group) always takes the full form.  The down
// projection takes the token-major full form even at decode sizes when the
// hidden size allows it (N % 256 == 0): its 256 weight rows per tile stream
// W_down faster than 32-token tiles do (GLM shape, 256 tokens, two planes:
// 0.27 vs 0.41 ms), while the gate/up projection keeps the decode form there
// (0.57 vs 0.69 ms).
int gemm_form(const moe_layer* L, int T, bool down = false) {
    if (L->gemm_form) return L->gemm_form;
    const moe_layer_config_t& c = L->cfg;
    const long long tokens = c.ep_size > 1 ? static_cast<long long>(c.max_tokens) * c.ep_size : T;
    const bool small = c.num_experts > 1 && tokens * c.top_k <= 16ll * c.num_experts;
    if (small && down && c.hidden % 256 == 0) return CBW_GEMM_TOKEN_TILES;
    return small ? CBW_GEMM_SMALL_TILES : CBW_GEMM_FULL_TILES;
}

// True when the down projection runs the token-major form, the one form that
// takes per-row output addresses (cbwFp8BlockScaledGroupedGemmRowOut).
bool down_token_major(const moe_layer* L, int T) {
    const int f = gemm_form(L, T, true);
    return L->cfg.hidden % 256 == 0 && (f == CBW_GEMM_TOKEN_TILES || f == CBW_GEMM_FULL_TILES);
}

cbwGroupedGemmArgs gemm_args(const moe_layer* L, void* ws, bool down, int T) {
    const moe_layer_config_t& c = L->cfg;
    cbwGroupedGemmArgs g;
    std::memset(&g, 0, sizeof(g));
    g.num_groups = L->groups;
    g.rows = L->rcap;
    g.a_ld = L->rcap;
    g.count = at<int32_t>(ws, L->off_counts);
    g.start = at<int32_t>(ws, L->off_start);
    if (!down) {
        g.mode = CBW_GEMM_GATED_SWIGLU | gemm_form(L, T) | (L->act_planes == 2 ? CBW_GEMM_ACT_X2 : 0);
        g.K = c.hidden;
        g.N = c.intermediate;
        g.a = at<void>(ws, L->off_xp);
        g.a_scale = at<float>(ws, L->off_xps);
        g.w = L->w.w13;
        g.w_scale = L->w.s13;
        g.out = at<void>(ws, L->off_hq);
        g.out_scale = at<float>(ws, L->off_hs);
        g.out_ld = L->rcap;
    } else {
        g.mode = CBW_GEMM_DOWN_BF16 | gemm_form(L, T, true) | (L->act_planes == 2 ? CBW_GEMM_ACT_X2 : 0);
        g.K = c.intermediate;
        g.N = c.hidden;
        g.a = at<void>(ws, L->off_hq);
        g.a_scale = at<float>(ws, L->off_hs);
        g.w = L->w.w2;
        g.w_scale = L->w.s2;
        g.out = at<void>(ws, L->off_y);
    }
    return g;
}

moe_status_t run_experts(moe_layer* L, const void* x, const int32_t* idx, const float* wts, void* out, int T,
                         void* ws, cudaStream_t st) {
    const moe_layer_config_t& c = L->cfg;
    const int H = c.hidden, K = c.top_k, S = c.num_shared;
    int32_t* counts = at<int32_t>(ws, L->off_counts);
    int32_t* start = at<int32_t>(ws, L->off_start);
    int32_t* total = at<int32_t>(ws, L->off_total);
    int32_t* pos = at<int32_t>(ws, L->off_pos);
    int32_t* rowtok = at<int32_t>(ws, L->off_rowtok);
    mark(L, 2, st);
    MOE_TRY(moe_permute_mb(idx, T, K, L->e_begin, L->e_end, S, counts, start, pos, rowtok, total, L->rcap,
                           L->error_word, 16, at<void>(ws, L->off_bcounts), L->bcounts_bytes, st));
    mark(L, 3, st);
    const bool x2 = L->act_planes == 2;
    // token-major: each token's row is read once and stored to its k routed
    // rows and its shared-expert rows (the same bytes as the row-major gather)
    MOE_TRY(moe_scatter_rows_x2(at<void>(ws, L->off_xq), x2 ? at<void>(ws, L->off_xq_lo) : nullptr,
                                at<float>(ws, L->off_xs), L->xs_ld, pos, T, K, start + (L->e_end - L->e_begin), S,
                                rowtok, total, L->rcap, H, at<void>(ws, L->off_xp),
                                x2 ? at<void>(ws, L->off_xp + L->rcap * static_cast<size_t>(H)) : nullptr,
                                at<float>(ws, L->off_xps), L->rcap, st));
    cbwGroupedGemmArgs g1 = gemm_args(L, ws, false, T), g2 = gemm_args(L, ws, true, T);
    mark(L, 4, st);
    MOE_TRY(cbw_to_moe(cbwFp8BlockScaledGroupedGemm(&g1, L->error_word, st)));
    mark(L, 5, st);
    MOE_TRY(cbw_to_moe(cbwFp8BlockScaledGroupedGemm(&g2, L->error_word, st)));
    const int32_t* shared_rows = start + (L->e_end - L->e_begin);
    mark(L, 6, st);
    MOE_TRY(moe_combine(x, at<void>(ws, L->off_y), pos, wts, shared_rows, S, T, K, H, out, st));
    mark(L, MOE_NUM_STAGES, st);
    return MOE_OK;
}

// Expert-parallel expert stage (moe_ep.cu has the exchange protocol).  Every
// rank takes the same collective steps in the same order; a rank with no
// tokens still exchanges (empty) counts and rows.
moe_status_t run_experts_ep(moe_layer* L, const int32_t* idx, const float* wts, const void* x, void* out, int T,
                            void* ws, cudaStream_t st) {
    const moe_layer_config_t& c = L->cfg;
    const int H = c.hidden, K = c.top_k, S = c.num_shared, E = c.num_experts, ep = c.ep_size;
    const int epr = E / ep;
    int32_t* ecounts = at<int32_t>(ws, L->off_ecounts);
    int32_t* rcounts = ecounts + E;
    int32_t* spos = at<int32_t>(ws, L->off_pos);
    int32_t* stok = at<int32_t>(ws, L->off_stok);
    int32_t* stotal = at<int32_t>(ws, L->off_stotal);
    int32_t* counts = at<int32_t>(ws, L->off_counts);
    int32_t* start = at<int32_t>(ws, L->off_start);
    int32_t* total = at<int32_t>(ws, L->off_total);
    int32_t* row_src = at<int32_t>(ws, L->off_rowtok);
    int32_t* recv_dst = at<int32_t>(ws, L->off_rdst);
    const size_t rb = L->row_bytes;
    // expert placement: the send order sorts by virtual expert (rank-major)
    const int32_t* sort_ids = idx;
    if (L->slot_of_expert) {
        int32_t* vidx = at<int32_t>(ws, L->off_vidx);
        MOE_TRY(moe_ep_remap_experts(idx, T * K, E, L->slot_of_expert, vidx, st));
        sort_ids = vidx;
    }

    if (L->peer_mode) {
        // device-driven exchange over the symmetric peer buffers: no host synchronisation
        const tbep::Peers& P = L->peers;
        uint8_t* mine = static_cast<uint8_t*>(P.base[c.ep_rank]);
        int32_t* plan = at<int32_t>(ws, L->off_plan);
        uint32_t* epoch = L->epoch_dev;   // advanced on the device by the counts exchange
        const int y_cap = c.max_tokens * K;
        mark(L, 2, st);
        MOE_TRY(moe_permute_mb(sort_ids, T, K, 0, E, 0, ecounts, at<int32_t>(ws, L->off_estart), spos, stok, stotal,
                                   T * K, L->error_word, 1, at<void>(ws, L->off_bcounts), L->bcounts_bytes, st));
        // each token travels once per destination rank, however many of its experts live there
        int32_t* uidx = at<int32_t>(ws, L->off_uidx);
        int32_t* utok = at<int32_t>(ws, L->off_utok);
        int32_t* ucount = at<int32_t>(ws, L->off_ucount);
        MOE_TRY(tbep::unique_rows(P, sort_ids, T, K, uidx, utok, ucount, st));
        MOE_TRY(tbep::counts(P, ecounts, ucount, epoch, plan, rcounts, L->error_word, st));
        mark(L, 3, st);
        const bool x2 = L->act_planes == 2;
        void* xq_lo = x2 ? at<void>(ws, L->off_xq_lo) : nullptr;
        void* xp_lo = x2 ? at<void>(ws, L->off_xp + L->rcap * static_cast<size_t>(H)) : nullptr;
        MOE_TRY(tbep::dispatch(P, at<void>(ws, L->off_xq), xq_lo, at<float>(ws, L->off_xs), L->xs_ld, stok, uidx,
                               utok, T, plan, H, rb, L->recv_cap, T * K, st));
        MOE_TRY(tbep::signal_wait(P, tbep::kDispatch, epoch, L->error_word, st));
        MOE_TRY(moe_ep_recv_plan(rcounts, ep, epr, T, S, counts, start, total, row_src, recv_dst, L->rcap, L->recv_cap,
                                 L->error_word, st));
        MOE_TRY(tbep::gather(P, at<void>(ws, L->off_xq), xq_lo, at<float>(ws, L->off_xs), L->xs_ld, row_src, total,
                             L->rcap, H, rb, L->recv_cap, at<void>(ws, L->off_xp), xp_lo, at<float>(ws, L->off_xps),
                             L->rcap, st));
        // fused return: every received row's output address in its owner's
        // return buffer, for the down GEMM's epilogue
        const bool fused = L->fused_return && down_token_major(L, T);
        void** row_out = at<void*>(ws, L->off_rowout);
        if (fused) MOE_TRY(tbep::return_rows(P, row_src, total, plan, H, y_cap, L->rcap, row_out, st));
        cbwGroupedGemmArgs g1 = gemm_args(L, ws, false, T), g2 = gemm_args(L, ws, true, T);
        mark(L, 4, st);
        MOE_TRY(cbw_to_moe(cbwFp8BlockScaledGroupedGemm(&g1, L->error_word, st)));
        mark(L, 5, st);
        if (fused) {
            MOE_TRY(cbw_to_moe(cbwFp8BlockScaledGroupedGemmRowOut(&g2, row_out, L->error_word, st)));
        } else {
            MOE_TRY(cbw_to_moe(cbwFp8BlockScaledGroupedGemm(&g2, L->error_word, st)));
        }
        mark(L, 6, st);
        if (!fused)
            MOE_TRY(tbep::combine_send(P, at<void>(ws, L->off_y), recv_dst, plan, H, y_cap, L->rcap, L->recv_cap, st));
        MOE_TRY(tbep::signal_wait(P, tbep::kCombine, epoch, L->error_word, st));
        MOE_TRY(moe_combine_split(x, mine + P.lay.off_yrecv, spos, wts, at<void>(ws, L->off_y), start + epr, S, T, K,
                                  H, out, st));
        mark(L, MOE_NUM_STAGES, st);
        return MOE_OK;
    }

    const bool x2 = L->act_planes == 2;
    void* xq_lo = x2 ? at<void>(ws, L->off_xq_lo) : nullptr;
    void* xp_lo = x2 ? at<void>(ws, L->off_xp + L->rcap * static_cast<size_t>(H)) : nullptr;
    mark(L, 2, st);
    MOE_TRY(moe_permute_mb(sort_ids, T, K, 0, E, 0, ecounts, at<int32_t>(ws, L->off_estart), spos, stok, stotal,
                               T * K, L->error_word, 1, at<void>(ws, L->off_bcounts), L->bcounts_bytes, st));
    MOE_TRY(moe_ep_pack_rows_x2(at<void>(ws, L->off_xq), xq_lo, at<float>(ws, L->off_xs), L->xs_ld, stok, stotal,
                                T * K, H, at<void>(ws, L->off_psend), st));
    std::vector<size_t> cc(ep, static_cast<size_t>(epr)), co(ep);
    for (int p = 0; p < ep; ++p) co[p] = static_cast<size_t>(p) * epr;
    MOE_TRY(nccl_to_moe(ncwAllToAllv(ecounts, cc.data(), co.data(), rcounts, cc.data(), co.data(), NCW_INT32,
                                     L->comm, st)));
    if (cudaMemcpyAsync(L->h_counts, ecounts, 2 * static_cast<size_t>(E) * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return MOE_ERR_CUDA;
    MOE_TRY(nccl_to_moe(ncwStreamSynchronizeTimeout(L->comm, st, L->sync_timeout_ms)));
    std::vector<size_t> srows(ep), soff(ep), rrows(ep), roff(ep);
    size_t stot = 0, rtot = 0;
    MOE_TRY(moe_ep_plan_host(ep, epr, L->h_counts, L->h_counts + E, srows.data(), soff.data(), rrows.data(),
                             roff.data(), &stot, &rtot));
    // Cannot trigger while every rank keeps T <= max_tokens (recv_cap is the
    // worst case); a peer that broke that contract has already sent.
    if (rtot > static_cast<size_t>(L->recv_cap) || stot > static_cast<size_t>(T) * K) return MOE_ERR_WORKSPACE;

    mark(L, 3, st);
    {
        std::vector<size_t> sb(ep), sbo(ep), rbn(ep), rbo(ep);
        for (int p = 0; p < ep; ++p) { sb[p] = srows[p] * rb; sbo[p] = soff[p] * rb; rbn[p] = rrows[p] * rb; rbo[p] = roff[p] * rb; }
        MOE_TRY(nccl_to_moe(ncwAllToAllv(at<void>(ws, L->off_psend), sb.data(), sbo.data(), at<void>(ws, L->off_precv),
                                         rbn.data(), rbo.data(), NCW_UINT8, L->comm, st)));
    }
    MOE_TRY(moe_ep_recv_plan(rcounts, ep, epr, T, S, counts, start, total, row_src, recv_dst, L->rcap, L->recv_cap,
                             L->error_word, st));
    MOE_TRY(moe_ep_gather_x2(at<void>(ws, L->off_precv), at<void>(ws, L->off_xq), xq_lo, at<float>(ws, L->off_xs),
                             L->xs_ld, row_src, total, L->rcap, H, at<void>(ws, L->off_xp), xp_lo,
                             at<float>(ws, L->off_xps), L->rcap, st));
    cbwGroupedGemmArgs g1 = gemm_args(L, ws, false, T), g2 = gemm_args(L, ws, true, T);
    mark(L, 4, st);
    MOE_TRY(cbw_to_moe(cbwFp8BlockScaledGroupedGemm(&g1, L->error_word, st)));
    mark(L, 5, st);
    MOE_TRY(cbw_to_moe(cbwFp8BlockScaledGroupedGemm(&g2, L->error_word, st)));
    mark(L, 6, st);
    MOE_TRY(moe_ep_pack_y(at<void>(ws, L->off_y), recv_dst, static_cast<int>(rtot), H, at<void>(ws, L->off_ysend), st));
    {
        const size_t hw = static_cast<size_t>(H);
        std::vector<size_t> sn(ep), so(ep), rn(ep), ro(ep);
        for (int p = 0; p < ep; ++p) { sn[p] = rrows[p] * hw; so[p] = roff[p] * hw; rn[p] = srows[p] * hw; ro[p] = soff[p] * hw; }
        MOE_TRY(nccl_to_moe(ncwAllToAllv(at<void>(ws, L->off_ysend), sn.data(), so.data(), at<void>(ws, L->off_yrecv),
                                         rn.data(), ro.data(), NCW_BFLOAT16, L->comm, st)));
    }
    MOE_TRY(moe_combine_split(x, at<void>(ws, L->off_yrecv), spos, wts, at<void>(ws, L->off_y), start + epr, S, T, K,
                              H, out, st));
    mark(L, MOE_NUM_STAGES, st);
    return MOE_OK;
}

moe_status_t run_experts_any(moe_layer* L, const void* x, const int32_t* idx, const float* wts, void* out, int T,
                             void* ws, cudaStream_t st) {
    if (L->cfg.ep_size > 1) return run_experts_ep(L, idx, wts, x, out, T, ws, st);
    return run_experts(L, x, idx, wts, out, T, ws, st);
}

}  // namespace

extern "C" {

const char* moe_status_string(moe_status_t s) {
    switch (s) {
        case MOE_OK: return "ok";
        case MOE_ERR_INVALID_ARGUMENT: return "invalid argument";
        case MOE_ERR_CUDA: return "CUDA error";
        case MOE_ERR_UNSUPPORTED: return "unsupported configuration";
        case MOE_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        case MOE_ERR_NCCL: return "NCCL error";
        case MOE_ERR_WORKSPACE: return "workspace too small or row capacity exceeded";
        default: return "unknown status";
    }
}

moe_status_t moe_layer_create(const moe_layer_config_t* cfg, const moe_layer_weights_t* w, ncwComm_t comm,
                              moe_layer_t** out) {
    if (!cfg || !w || !out) return MOE_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    const moe_layer_config_t& c = *cfg;
    if (c.hidden <= 0 || c.hidden % 128 || c.intermediate <= 0 || c.intermediate % 128) return MOE_ERR_INVALID_ARGUMENT;
    if (c.num_experts <= 0 || c.num_experts > 256 || c.top_k <= 0 || c.top_k > 16 || c.top_k > c.num_experts)
        return MOE_ERR_INVALID_ARGUMENT;
    if (c.num_shared < 0 || c.num_shared > 1 || c.max_tokens <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (c.ep_size <= 0 || c.ep_rank < 0 || c.ep_rank >= c.ep_size || c.num_experts % c.ep_size) return MOE_ERR_INVALID_ARGUMENT;
    // ep_size > 1 without a communicator: the peer-memory exchange only (its
    // buffers must be set before the first forward)
    if (c.ep_size > 1 && c.num_experts > 1024) return MOE_ERR_UNSUPPORTED;
    if (!w->norm_gamma || !w->router_w || !w->w13 || !w->s13 || !w->w2 || !w->s2) return MOE_ERR_INVALID_ARGUMENT;
    moe_layer* L = new (std::nothrow) moe_layer;
    if (!L) return MOE_ERR_INVALID_ARGUMENT;
    std::memset(L, 0, sizeof(*L));
    L->act_planes = 1;
    L->cfg = c;
    L->w = *w;
    L->comm = comm;
    const int per = c.num_experts / c.ep_size;
    L->e_begin = c.ep_rank * per;
    L->e_end = L->e_begin + per;
    L->groups = per + c.num_shared;
    if (cudaMalloc(&L->error_word, sizeof(int)) != cudaSuccess) { delete L; return MOE_ERR_CUDA; }
    if (cudaMemset(L->error_word, 0, sizeof(int)) != cudaSuccess) { cudaFree(L->error_word); delete L; return MOE_ERR_CUDA; }
    if (c.ep_size > 1) {
        if (cudaMallocHost(&L->h_counts, 2 * static_cast<size_t>(c.num_experts) * sizeof(int32_t)) != cudaSuccess) {
            cudaFree(L->error_word);
            delete L;
            return MOE_ERR_CUDA;
        }
        const char* tm = std::getenv("TIME_B200_EP_TIMEOUT_MS");
        L->sync_timeout_ms = (tm && std::atoi(tm) > 0) ? std::atoi(tm) : 120000;
    }
    plan_workspace(L);
    *out = L;
    return MOE_OK;
}

moe_status_t moe_layer_destroy(moe_layer_t* L) {
    if (!L) return MOE_OK;
    if (L->slot_of_expert) cudaFree(L->slot_of_expert);
    if (L->h_counts) cudaFreeHost(L->h_counts);
    if (L->epoch_dev) cudaFree(L->epoch_dev);
    cudaFree(L->error_word);
    delete L;
    return MOE_OK;
}

size_t moe_layer_workspace_bytes(const moe_layer_t* L) { return L ? L->bytes : 0; }

moe_status_t moe_layer_forward_routed(moe_layer_t* L, const void* x, const int32_t* idx, const float* wts, void* out,
                                      int T, void* ws, size_t ws_bytes, cwStream_t stream) {
    if (!L || !ws || (T > 0 && (!x || !out || !idx || !wts))) return MOE_ERR_INVALID_ARGUMENT;
    if (L->cfg.ep_size > 1 && !L->peer_mode && !L->comm) return MOE_ERR_INVALID_ARGUMENT;
    if (T < 0 || T > L->cfg.max_tokens) return MOE_ERR_INVALID_ARGUMENT;
    if (ws_bytes < L->bytes) return MOE_ERR_WORKSPACE;
    if (T == 0 && L->cfg.ep_size == 1) return MOE_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const moe_layer_config_t& c = L->cfg;
    mark(L, 0, st);
    if (L->act_planes == 2)
        MOE_TRY(moe_rmsnorm_quant_x2(x, L->w.norm_gamma, T, c.hidden, c.rms_eps, at<float>(ws, L->off_rms), nullptr,
                                     0, at<void>(ws, L->off_xq), at<void>(ws, L->off_xq_lo), at<float>(ws, L->off_xs),
                                     L->xs_ld, stream));
    else
        MOE_TRY(moe_rmsnorm_quant(x, L->w.norm_gamma, T, c.hidden, c.rms_eps, at<float>(ws, L->off_rms),
                                  at<void>(ws, L->off_xq), at<float>(ws, L->off_xs), L->xs_ld, stream));
    mark(L, 1, st);
    return run_experts_any(L, x, idx, wts, out, T, ws, st);
}

moe_status_t moe_layer_forward(moe_layer_t* L, const void* x, void* out, int T, void* ws, size_t ws_bytes,
                               cwStream_t stream) {
    if (!L || !ws || (T > 0 && (!x || !out))) return MOE_ERR_INVALID_ARGUMENT;
    if (L->cfg.ep_size > 1 && !L->peer_mode && !L->comm) return MOE_ERR_INVALID_ARGUMENT;
    if (T < 0 || T > L->cfg.max_tokens) return MOE_ERR_INVALID_ARGUMENT;
    if (ws_bytes < L->bytes) return MOE_ERR_WORKSPACE;
    if (T == 0 && L->cfg.ep_size == 1) return MOE_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const moe_layer_config_t& c = L->cfg;
    float* rms = at<float>(ws, L->off_rms);
    float* n = at<float>(ws, L->off_n);
    float* logits = at<float>(ws, L->off_logits);
    mark(L, 0, st);
    // hidden sizes that are multiples of 256 (every real model) take the
    // column-ordered router: n is written in that order by the RMSNorm and
    // the router weight is reordered into the workspace (E x H floats)
    const bool rc = c.hidden % 256 == 0;
    if (L->act_planes == 2)
        MOE_TRY(moe_rmsnorm_quant_x2(x, L->w.norm_gamma, T, c.hidden, c.rms_eps, rms, n, rc ? 1 : 0,
                                     at<void>(ws, L->off_xq), at<void>(ws, L->off_xq_lo), at<float>(ws, L->off_xs),
                                     L->xs_ld, stream));
    else if (rc)
        MOE_TRY(moe_rmsnorm_quant_rc(x, L->w.norm_gamma, T, c.hidden, c.rms_eps, rms, n, at<void>(ws, L->off_xq),
                                     at<float>(ws, L->off_xs), L->xs_ld, stream));
    else
        MOE_TRY(moe_rmsnorm_quant_n(x, L->w.norm_gamma, T, c.hidden, c.rms_eps, rms, n, at<void>(ws, L->off_xq),
                                    at<float>(ws, L->off_xs), L->xs_ld, stream));
    int32_t* idx = at<int32_t>(ws, L->off_idx);
    float* wts = at<float>(ws, L->off_w);
    mark(L, 1, st);
    if (rc) {
        float* wrc = at<float>(ws, L->off_wrc);
        MOE_TRY(moe_router_columns(L->w.router_w, wrc, c.num_experts, c.hidden, stream));
        MOE_TRY(moe_router_logits_rc(n, wrc, L->w.router_bias, T, c.hidden, c.num_experts, logits, stream));
    } else {
        MOE_TRY(moe_router_logits(n, L->w.router_w, L->w.router_bias, T, c.hidden, c.num_experts, logits, stream));
    }
    MOE_TRY(moe_topk_softmax(logits, T, c.num_experts, c.top_k, idx, wts, stream));
    return run_experts_any(L, x, idx, wts, out, T, ws, st);
}

moe_status_t moe_layer_last_routing(const moe_layer_t* L, const void* ws, const int32_t** idx, const float** wts,
                                    const int32_t** counts) {
    if (!L || !ws) return MOE_ERR_INVALID_ARGUMENT;
    void* w = const_cast<void*>(ws);
    if (idx) *idx = at<int32_t>(w, L->off_idx);
    if (wts) *wts = at<float>(w, L->off_w);
    if (counts) *counts = at<int32_t>(w, L->off_counts);
    return MOE_OK;
}

moe_status_t moe_layer_set_stage_events(moe_layer_t* L, cwEvent_t* events) {
    if (!L) return MOE_ERR_INVALID_ARGUMENT;
    L->timing = events != nullptr;
    for (int i = 0; i <= MOE_NUM_STAGES; ++i)
        L->stage_ev[i] = events ? static_cast<cudaEvent_t>(events[i]) : nullptr;
    return MOE_OK;
}

moe_status_t moe_layer_set_act_planes(moe_layer_t* L, int planes) {
    if (!L || (planes != 1 && planes != 2)) return MOE_ERR_INVALID_ARGUMENT;
    // the exchange's packed rows and the peer buffers are sized for the format:
    // choose it before the peer buffers are set
    if (L->peer_mode && planes != L->act_planes) return MOE_ERR_INVALID_ARGUMENT;
    L->act_planes = planes;
    plan_workspace(L);
    return MOE_OK;
}

moe_status_t moe_layer_get_act_planes(const moe_layer_t* L, int* planes) {
    if (!L || !planes) return MOE_ERR_INVALID_ARGUMENT;
    *planes = L->act_planes;
    return MOE_OK;
}

moe_status_t moe_layer_set_gemm_form(moe_layer_t* L, int form) {
    if (!L) return MOE_ERR_INVALID_ARGUMENT;
    if (form != 0 && form != CBW_GEMM_SMALL_TILES && form != CBW_GEMM_FULL_TILES && form != CBW_GEMM_ONE_SM_TILES &&
        form != CBW_GEMM_PAIR_TILES && form != CBW_GEMM_TOKEN_TILES)
        return MOE_ERR_INVALID_ARGUMENT;
    L->gemm_form = form;
    return MOE_OK;
}

moe_status_t moe_layer_set_expert_placement(moe_layer_t* L, const int32_t* slot_of_expert) {
    if (!L) return MOE_ERR_INVALID_ARGUMENT;
    const int E = L->cfg.num_experts;
    if (!slot_of_expert) {
        if (L->slot_of_expert) cudaFree(L->slot_of_expert);
        L->slot_of_expert = nullptr;
        return MOE_OK;
    }
    if (L->cfg.ep_size <= 1) return MOE_ERR_INVALID_ARGUMENT;
    std::vector<char> seen(E, 0);
    for (int e = 0; e < E; ++e) {
        const int v = slot_of_expert[e];
        if (v < 0 || v >= E || seen[v]) return MOE_ERR_INVALID_ARGUMENT;   // must be a permutation
        seen[v] = 1;
    }
    if (!L->slot_of_expert && cudaMalloc(&L->slot_of_expert, E * sizeof(int32_t)) != cudaSuccess) {
        L->slot_of_expert = nullptr;
        return MOE_ERR_CUDA;
    }
    if (cudaMemcpy(L->slot_of_expert, slot_of_expert, E * sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess)
        return MOE_ERR_CUDA;
    return MOE_OK;
}

size_t moe_layer_peer_bytes(const moe_layer_t* L) {
    if (!L || L->cfg.ep_size <= 1) return 0;
    const moe_layer_config_t& c = L->cfg;
    return tbep::layout(c.ep_size, c.num_experts, L->recv_cap, L->row_bytes,
                        static_cast<size_t>(c.max_tokens) * c.top_k, c.hidden).bytes;
}

moe_status_t moe_layer_set_peer_buffers(moe_layer_t* L, void* const* peer_bufs, int n) {
    if (!L) return MOE_ERR_INVALID_ARGUMENT;
    const moe_layer_config_t& c = L->cfg;
    if (!peer_bufs) { L->peer_mode = false; return MOE_OK; }
    if (c.ep_size <= 1 || n != c.ep_size || n > tbep::kMaxRanks) return MOE_ERR_INVALID_ARGUMENT;
    for (int r = 0; r < n; ++r)
        if (!peer_bufs[r] || (reinterpret_cast<uintptr_t>(peer_bufs[r]) & 255)) return MOE_ERR_INVALID_ARGUMENT;
    std::memset(&L->peers, 0, sizeof(L->peers));
    for (int r = 0; r < n; ++r) L->peers.base[r] = peer_bufs[r];
    L->peers.ep = c.ep_size;
    L->peers.me = c.ep_rank;
    L->peers.E = c.num_experts;
    L->peers.epr = c.num_experts / c.ep_size;
    L->peers.lay = tbep::layout(c.ep_size, c.num_experts, L->recv_cap, L->row_bytes,
                                static_cast<size_t>(c.max_tokens) * c.top_k, c.hidden);
    const int ms = L->sync_timeout_ms < 20000 ? L->sync_timeout_ms : 20000;   // device waits: at most 20 s
    L->peers.timeout_ns = static_cast<unsigned long long>(ms) * 1000000ull;
    if (!L->epoch_dev && cudaMalloc(&L->epoch_dev, sizeof(uint32_t)) != cudaSuccess) {
        L->epoch_dev = nullptr;
        return MOE_ERR_CUDA;
    }
    if (cudaMemset(L->epoch_dev, 0, sizeof(uint32_t)) != cudaSuccess) return MOE_ERR_CUDA;
    {
        const char* f = std::getenv("TIME_B200_EP_FUSED_RETURN");
        L->fused_return = f && f[0] == '1';
    }
    L->peer_mode = true;
    return MOE_OK;
}

moe_status_t moe_layer_check_error(moe_layer_t* L, cwStream_t stream) {
    if (!L) return MOE_ERR_INVALID_ARGUMENT;
    int h = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&h, L->error_word, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return MOE_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return MOE_ERR_CUDA;
    if (h == 0) return MOE_OK;
    cudaMemsetAsync(L->error_word, 0, sizeof(int), st);
    cudaStreamSynchronize(st);
    return h == 2 ? MOE_ERR_WORKSPACE : MOE_ERR_DEVICE_TIMEOUT;   // 1: GEMM wait, 3: peer exchange wait
}

}  // extern "C"
