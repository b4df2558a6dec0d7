// attn_block.cu -- the tensor-parallel decode attention block of the decoder
// layer, one call per decode step (one new token per sequence), per TP rank:
//
//   rmsnorm + e4m3 1x128   moe_rmsnorm_quant
//   QKV projection         bf16 out: the tcgen05 grouped GEMM with one group, or
//                          for a small batch on a small weight (a TP rank's
//                          slice) fp8_gemm_small (split-K mma.sync), which
//                          spreads the few weight rows over every SM
//   partial RoPE + pages   attn_rope_kv_write (also seq_lens = pos + 1)
//   decode attention       attn_decode_paged (bf16 + e4m3 rows for o_proj)
//   o_proj (row parallel)  the same, bf16 partial
//   TP sum + residual      ranks summed in fp32 in rank order
//
// The reference's layer runs the same sequence in fp32 through cbwSgemm and
// its launch_* attention kernels (src/terra/engine.t:1269-1310) with the
// all-reduce of the spec after o_proj (kernels.fut:605-607, ncclAllReduce).
// Here, for tp > 1, each rank's partial goes into its peer-visible buffer,
// one thread raises the rank's ready flag on every rank (system-scope
// release), the reduce kernel waits for every flag and reads all partials over
// NVLink, and a one-thread kernel then raises the rank's done flag; the next
// call waits for every done flag before overwriting its partial.  The epoch
// lives in device memory, so a decode step can be captured in a CUDA graph
// and replayed.  Every wait is bounded (error word 3 on timeout).
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "attn_block.h"
#include "cublas_wrappers.h"
#include "sm100.cuh"

namespace {

using namespace tb;

constexpr int kD = 128;
constexpr int kMaxTp = 64;
constexpr size_t kFlagBytes = 512;   // ready[kMaxTp] at 0, done[kMaxTp] at 256, partial after
constexpr int kSmallGemmMaxT = 64;    // batches up to this may run the projections on fp8_gemm_small
constexpr long long kSmallGemmMaxW = 32ll << 20;   // ... when the weight has fewer bytes than this

inline moe_status_t launch_status() {
    return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

// Measured on B200 (one GPU's GLM shapes, bf16 out): QKV 14336 x 5120 at 16 /
// 64 / 256 tokens 31 / 33 / 52 us grouped vs 59 / 58 / 181 us split-K;
// o_proj 5120 x 12288 57 / 64 / 102 vs 64 / 65 / 216 us.  The split-K kernel
// wins only where the grouped GEMM's 128-row tiles leave most SMs idle (a TP
// rank's 1792 x 5120 or 5120 x 1536 at a decode batch).
bool use_small_gemm(int B, int N, int K) {
    return B <= kSmallGemmMaxT && static_cast<long long>(N) * K < kSmallGemmMaxW;
}

// out = bf16(residual + (0 + part)): the tp == 1 form of the rank-ordered sum
__global__ void __launch_bounds__(256)
residual_add_kernel(const __nv_bfloat16* __restrict__ part, const __nv_bfloat16* __restrict__ residual, size_t n,
                    __nv_bfloat16* __restrict__ out) {
    const size_t i8 = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (i8 >= n) return;
    const uint4 rv = *reinterpret_cast<const uint4*>(residual + i8);
    const uint4 pv = *reinterpret_cast<const uint4*>(part + i8);
    const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
    const __nv_bfloat16* pb = reinterpret_cast<const __nv_bfloat16*>(&pv);
    uint4 ov;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int j = 0; j < 8; ++j) ob[j] = __float2bfloat16_rn(__bfloat162float(rb[j]) + (0.0f + __bfloat162float(pb[j])));
    *reinterpret_cast<uint4*>(out + i8) = ov;
}

__global__ void set_group_kernel(int32_t* cs, int B) {
    cs[0] = B;   // count of the one group
    cs[1] = 0;   // its first row
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct PeerSet {
    uint8_t* base[kMaxTp];   // rank r's buffer as mapped here
    int tp, me;
};

__device__ __forceinline__ uint32_t* ready_flag(const PeerSet& P, int rank, int src) {
    return reinterpret_cast<uint32_t*>(P.base[rank]) + src;
}
__device__ __forceinline__ uint32_t* done_flag(const PeerSet& P, int rank, int src) {
    return reinterpret_cast<uint32_t*>(P.base[rank] + 256) + src;
}

// One thread: wait (bounded) until every rank's flag here equals `value`.
__device__ bool wait_all(const PeerSet& P, bool done, uint32_t value, unsigned long long timeout_ns) {
    const uint64_t t0 = globaltimer_ns();
    for (int s = 0; s < P.tp; ++s) {
        const uint32_t* f = done ? done_flag(P, P.me, s) : ready_flag(P, P.me, s);
        while (ld_acquire_sys_u32(f) != value) {
            if (globaltimer_ns() - t0 > timeout_ns) return false;
            __nanosleep(64);
        }
    }
    return true;
}

// Before this rank overwrites its partial: every rank has finished reading
// the previous one (done[s] == current epoch).
__global__ void tp_wait_done_kernel(const PeerSet P, const uint32_t* __restrict__ epoch, unsigned long long timeout_ns,
                                    int* __restrict__ error_word) {
    if (threadIdx.x != 0) return;
    if (!wait_all(P, true, *epoch, timeout_ns) && error_word) atomicExch(error_word, 3);
}

// The partial is written: epoch += 1, raise ready[me] = epoch on every rank.
__global__ void tp_signal_kernel(const PeerSet P, uint32_t* __restrict__ epoch) {
    if (threadIdx.x != 0) return;
    const uint32_t e = *epoch + 1u;
    *epoch = e;
    __threadfence_system();
    for (int d = 0; d < P.tp; ++d) st_release_sys_u32(ready_flag(P, d, P.me), e);
}

// The reduce is done reading: raise done[me] = epoch on every rank.
__global__ void tp_done_kernel(const PeerSet P, const uint32_t* __restrict__ epoch) {
    if (threadIdx.x != 0) return;
    const uint32_t e = *epoch;
    __threadfence_system();
    for (int d = 0; d < P.tp; ++d) st_release_sys_u32(done_flag(P, d, P.me), e);
}

// Each block: one thread waits (bounded) for every rank's ready flag, then
// the block sums its slice of the partials in rank order.
__global__ void __launch_bounds__(256)
tp_peer_reduce_kernel(const PeerSet P, const uint32_t* __restrict__ epoch,
                      const __nv_bfloat16* __restrict__ residual, size_t n, __nv_bfloat16* __restrict__ out,
                      unsigned long long timeout_ns, int* __restrict__ error_word) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = wait_all(P, false, *epoch, timeout_ns) ? 1 : 0;
        if (!ok && error_word) atomicExch(error_word, 3);
    }
    __syncthreads();
    if (!ok) return;
    const size_t i8 = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
    if (i8 >= n) return;
    float acc[8];
    {
        const uint4 rv = *reinterpret_cast<const uint4*>(residual + i8);
        const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __bfloat162float(rb[j]);
    }
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < P.tp; ++r) {
        const __nv_bfloat16* part = reinterpret_cast<const __nv_bfloat16*>(P.base[r] + kFlagBytes);
        const uint4 pv = *reinterpret_cast<const uint4*>(part + i8);
        const __nv_bfloat16* pb = reinterpret_cast<const __nv_bfloat16*>(&pv);
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] += __bfloat162float(pb[j]);
    }
    uint4 ov;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&ov);
#pragma unroll
    for (int j = 0; j < 8; ++j) ob[j] = __float2bfloat16_rn(acc[j] + s[j]);
    *reinterpret_cast<uint4*>(out + i8) = ov;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct attn_block {
    attn_block_config_t cfg;
    attn_block_weights_t w;
    int nqkv;              // (nq + 2 nkv) * 128
    int rows_pad;          // max_batch rounded up to 16, at least 32 (the GEMM's token tiles)
    int ld;                // scale-row stride (= rows_pad)
    int split_tokens, max_splits;
    float* inv_freq;       // device [rot / 2]
    int* error_word;       // device
    // workspace plan
    size_t off_xq, off_xs, off_rms, off_group, off_qkv, off_q, off_lens, off_out, off_aq, off_as, off_dec, off_part,
        off_gsplit, dec_bytes, gsplit_bytes, bytes;
    // peer buffers (tp > 1)
    bool peer_mode;
    PeerSet peers;
    uint32_t* epoch_dev;   // device: calls so far (tp > 1)
    unsigned long long timeout_ns;
};

namespace {

template <typename T>
T* at(void* ws, size_t off) { return reinterpret_cast<T*>(static_cast<uint8_t*>(ws) + off); }

void plan(attn_block* L) {
    const attn_block_config_t& c = L->cfg;
    size_t o = 0;
    auto take = [&](size_t n) { const size_t r = o; o = align_up(o + n, 256); return r; };
    const size_t R = L->rows_pad, H = c.hidden;
    L->off_xq = take(R * H);
    L->off_xs = take(H / 128 * L->ld * 4);
    L->off_rms = take(R * 4);
    L->off_group = take(16);
    L->off_qkv = take(R * L->nqkv * 2);
    L->off_q = take(R * c.num_q_heads * kD * 2);
    L->off_lens = take(R * 4);
    L->off_out = take(R * c.num_q_heads * kD * 2);
    L->off_aq = take(R * c.num_q_heads * kD);
    L->off_as = take(static_cast<size_t>(c.num_q_heads) * L->ld * 4);
    L->dec_bytes = attn_decode_workspace_bytes(c.max_batch, c.num_q_heads, L->max_splits);
    L->off_dec = take(L->dec_bytes);
    L->off_part = take(R * H * 2);
    // split-K partials of the small-batch projections, for any B <= max_batch
    size_t g = 0;
    for (int t = 1; t <= c.max_batch && t <= kSmallGemmMaxT; ++t) {
        const size_t a = use_small_gemm(t, L->nqkv, H) ? fp8_gemm_small_workspace_bytes(t, L->nqkv, H) : 0;
        const size_t b = use_small_gemm(t, H, c.num_q_heads * kD)
                             ? fp8_gemm_small_workspace_bytes(t, H, c.num_q_heads * kD)
                             : 0;
        g = a > g ? a : g;
        g = b > g ? b : g;
    }
    L->gsplit_bytes = g;
    L->off_gsplit = take(g > 0 ? g : 16);
    L->bytes = o;
}

moe_status_t gemm(const attn_block* L, int mode, int B, int K, int N, const void* a, const float* as, const void* w,
                  const float* ws, void* ws_base, void* out, cudaStream_t st) {
    if (use_small_gemm(B, N, K))
        return fp8_gemm_small(a, as, L->ld, B, w, ws, N, K, out, at<void>(ws_base, L->off_gsplit), L->gsplit_bytes, st);
    cbwGroupedGemmArgs g;
    std::memset(&g, 0, sizeof(g));
    g.mode = mode;
    g.num_groups = 1;
    g.K = K;
    g.N = N;
    g.rows = L->rows_pad;
    g.a = a;
    g.a_scale = as;
    g.a_ld = L->ld;
    g.w = w;
    g.w_scale = ws;
    g.count = at<int32_t>(ws_base, L->off_group);
    g.start = at<int32_t>(ws_base, L->off_group) + 1;
    g.out = out;
    g.out_scale = nullptr;
    g.out_ld = 0;
    const cbwStatus_t s = cbwFp8BlockScaledGroupedGemm(&g, L->error_word, st);
    return s == CBW_SUCCESS ? MOE_OK : (s == CBW_ERROR_INVALID_VALUE ? MOE_ERR_INVALID_ARGUMENT : MOE_ERR_CUDA);
}

#define ATT_TRY(x)                          \
    do {                                    \
        const moe_status_t s_ = (x);        \
        if (s_ != MOE_OK) return s_;        \
    } while (0)

// Context split for a call of B rows: about two CTAs per SM at half the
// longest context (256..4096 tokens), the same rule as at creation for
// max_batch rows, then widened until the split partials of B rows fit the
// workspace sized at creation.
int split_for_rows(const attn_block* L, int B, int* max_splits) {
    const attn_block_config_t& c = L->cfg;
    const long long work = static_cast<long long>(B) * c.num_kv_heads * (c.max_context / 2 + 1);
    int split = 256;
    while (split < 4096 && work / split > 2 * 2 * 148) split *= 2;
    const long long cap = static_cast<long long>(c.max_batch) * L->max_splits;
    while (split < 8192 && static_cast<long long>(B) * ((c.max_context + split - 1) / split) > cap) split *= 2;
    *max_splits = (c.max_context + split - 1) / split;
    return split;
}

// Steps 1-5: the rank's o_proj partial (bf16 [B][H]) into `partial`.
moe_status_t run_partial(attn_block* L, const void* x, int B, const int32_t* positions, const int32_t* row_seq,
                         int num_seqs, int prefill_rows, const int32_t* page_table, int num_cache_pages, void* k_cache,
                         void* v_cache, void* partial, void* ws, cudaStream_t st) {
    const attn_block_config_t& c = L->cfg;
    const int H = c.hidden, nq = c.num_q_heads, nkv = c.num_kv_heads;
    ATT_TRY(moe_rmsnorm_quant(x, L->w.gamma, B, H, c.eps, at<float>(ws, L->off_rms), at<void>(ws, L->off_xq),
                              at<float>(ws, L->off_xs), L->ld, st));
    if (!use_small_gemm(B, L->nqkv, H) || !use_small_gemm(B, H, nq * kD)) {
        set_group_kernel<<<1, 1, 0, st>>>(at<int32_t>(ws, L->off_group), B);
        ATT_TRY(launch_status());
    }
    ATT_TRY(gemm(L, CBW_GEMM_DOWN_BF16, B, H, L->nqkv, at<void>(ws, L->off_xq), at<float>(ws, L->off_xs), L->w.w_qkv,
                 L->w.s_qkv, ws, at<void>(ws, L->off_qkv), st));
    ATT_TRY(attn_rope_kv_write_rows(at<void>(ws, L->off_qkv), B, nq, nkv, kD, c.rotary_dim, L->inv_freq, positions,
                                    row_seq, num_seqs, page_table, c.max_pages_per_seq, 16, num_cache_pages,
                                    at<void>(ws, L->off_q), k_cache, v_cache, at<int32_t>(ws, L->off_lens),
                                    L->error_word, st));
    int max_splits = 0;
    const int split = split_for_rows(L, B, &max_splits);
    ATT_TRY(attn_paged_rows(at<void>(ws, L->off_q), k_cache, v_cache, num_cache_pages, page_table,
                                   c.max_pages_per_seq, row_seq, num_seqs, at<int32_t>(ws, L->off_lens), B,
                                   prefill_rows, nq, nkv,
                                   kD, 16, 1.0f / std::sqrt(static_cast<float>(kD)), split, max_splits,
                                   at<void>(ws, L->off_dec), L->dec_bytes, at<void>(ws, L->off_out),
                                   at<void>(ws, L->off_aq), at<float>(ws, L->off_as), L->ld, L->error_word, st));
    ATT_TRY(gemm(L, CBW_GEMM_DOWN_BF16, B, nq * kD, H, at<void>(ws, L->off_aq), at<float>(ws, L->off_as), L->w.w_o,
                 L->w.s_o, ws, partial, st));
    return MOE_OK;
}

}  // namespace

extern "C" {

moe_status_t attn_block_create(const attn_block_config_t* cfg, const attn_block_weights_t* w, attn_block_t** out) {
    if (!cfg || !w || !out) return MOE_ERR_INVALID_ARGUMENT;
    const attn_block_config_t& c = *cfg;
    if (c.hidden <= 0 || c.hidden % 128 || c.num_q_heads <= 0 || c.num_kv_heads <= 0 ||
        c.num_q_heads % c.num_kv_heads || c.num_q_heads / c.num_kv_heads > 16 || c.head_dim != kD)
        return MOE_ERR_INVALID_ARGUMENT;
    if (c.rotary_dim < 0 || c.rotary_dim > kD || c.rotary_dim % 2 || !(c.rope_theta > 0.0f)) return MOE_ERR_INVALID_ARGUMENT;
    if (c.max_batch <= 0 || c.max_pages_per_seq <= 0 || c.max_context <= 0 || c.max_context > c.max_pages_per_seq * 16)
        return MOE_ERR_INVALID_ARGUMENT;
    if (c.tp_size <= 0 || c.tp_size > kMaxTp || c.tp_rank < 0 || c.tp_rank >= c.tp_size) return MOE_ERR_INVALID_ARGUMENT;
    if (!w->gamma || !w->w_qkv || !w->s_qkv || !w->w_o || !w->s_o) return MOE_ERR_INVALID_ARGUMENT;
    attn_block* L = new (std::nothrow) attn_block();
    if (!L) return MOE_ERR_INVALID_ARGUMENT;
    L->cfg = c;
    L->w = *w;
    L->nqkv = (c.num_q_heads + 2 * c.num_kv_heads) * kD;
    // rows of the GEMMs' activation tensors: a multiple of 16, at least the
    // grouped GEMM's 32-row token box
    L->rows_pad = std::max(32, (c.max_batch + 15) / 16 * 16);
    L->ld = L->rows_pad;   // the GEMM wants a scale stride of at least its row extent
    // splits: about two CTAs per SM for a full batch at half the longest context
    const long long work = static_cast<long long>(c.max_batch) * c.num_kv_heads * (c.max_context / 2 + 1);
    int split = 256;
    while (split < 4096 && work / split > 2 * 2 * 148) split *= 2;
    L->split_tokens = split;
    L->max_splits = (c.max_context + split - 1) / split;
    plan(L);
    std::vector<float> f(c.rotary_dim / 2 > 0 ? c.rotary_dim / 2 : 1, 0.0f);
    for (int i = 0; i < c.rotary_dim / 2; ++i)
        f[i] = static_cast<float>(std::pow(static_cast<double>(c.rope_theta), -2.0 * i / c.rotary_dim));
    if (cudaMalloc(&L->inv_freq, f.size() * sizeof(float)) != cudaSuccess ||
        cudaMemcpy(L->inv_freq, f.data(), f.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMalloc(&L->error_word, sizeof(int)) != cudaSuccess || cudaMemset(L->error_word, 0, sizeof(int)) != cudaSuccess) {
        attn_block_destroy(L);
        return MOE_ERR_CUDA;
    }
    const char* tm = std::getenv("TIME_B200_EP_TIMEOUT_MS");
    const long long ms = (tm && std::atoi(tm) > 0) ? std::atoi(tm) : 20000;
    L->timeout_ns = static_cast<unsigned long long>(ms < 20000 ? ms : 20000) * 1000000ull;
    *out = L;
    return MOE_OK;
}

moe_status_t attn_block_destroy(attn_block_t* L) {
    if (!L) return MOE_OK;
    if (L->inv_freq) cudaFree(L->inv_freq);
    if (L->epoch_dev) cudaFree(L->epoch_dev);
    if (L->error_word) cudaFree(L->error_word);
    delete L;
    return MOE_OK;
}

size_t attn_block_workspace_bytes(const attn_block_t* L) { return L ? L->bytes : 0; }

int attn_block_split_tokens(const attn_block_t* L) { return L ? L->split_tokens : 0; }

size_t attn_block_peer_bytes(const attn_block_t* L) {
    if (!L || L->cfg.tp_size <= 1) return 0;
    return kFlagBytes + static_cast<size_t>(L->rows_pad) * L->cfg.hidden * 2;
}

moe_status_t attn_block_set_peer_buffers(attn_block_t* L, void* const* bufs, int n) {
    if (!L || !bufs || n != L->cfg.tp_size || n <= 1) return MOE_ERR_INVALID_ARGUMENT;
    if (L->peer_mode) return MOE_ERR_INVALID_ARGUMENT;   // once: the flags in the buffers pair up with the epoch
    for (int r = 0; r < n; ++r) {
        if (!bufs[r] || (reinterpret_cast<uintptr_t>(bufs[r]) & 255)) return MOE_ERR_INVALID_ARGUMENT;
        L->peers.base[r] = static_cast<uint8_t*>(bufs[r]);
    }
    L->peers.tp = n;
    L->peers.me = L->cfg.tp_rank;
    if (!L->epoch_dev && cudaMalloc(&L->epoch_dev, sizeof(uint32_t)) != cudaSuccess) {
        L->epoch_dev = nullptr;
        return MOE_ERR_CUDA;
    }
    if (cudaMemset(L->epoch_dev, 0, sizeof(uint32_t)) != cudaSuccess) return MOE_ERR_CUDA;
    L->peer_mode = true;
    return MOE_OK;
}

moe_status_t attn_block_prefill_partial(attn_block_t* L, const void* x_bf16, int B, const int32_t* positions,
                                        const int32_t* row_seq, int num_seqs, int prefill_rows,
                                        const int32_t* page_table, int num_cache_pages, void* k_cache, void* v_cache,
                                        void* partial_bf16, void* workspace, size_t workspace_bytes,
                                        cwStream_t stream) {
    if (!L || B < 0 || B > L->cfg.max_batch || num_seqs <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (prefill_rows < 0 || prefill_rows > B) return MOE_ERR_INVALID_ARGUMENT;
    if (B == 0) return MOE_OK;
    if (!x_bf16 || !positions || !page_table || !k_cache || !v_cache || !partial_bf16 || !workspace)
        return MOE_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < L->bytes) return MOE_ERR_WORKSPACE;
    return run_partial(L, x_bf16, B, positions, row_seq, num_seqs, prefill_rows, page_table, num_cache_pages, k_cache,
                       v_cache, partial_bf16, workspace, static_cast<cudaStream_t>(stream));
}

moe_status_t attn_block_forward_partial(attn_block_t* L, const void* x_bf16, int B, const int32_t* positions,
                                        const int32_t* row_seq, int num_seqs, const int32_t* page_table,
                                        int num_cache_pages, void* k_cache, void* v_cache, void* partial_bf16,
                                        void* workspace, size_t workspace_bytes, cwStream_t stream) {
    return attn_block_prefill_partial(L, x_bf16, B, positions, row_seq, num_seqs, 0, page_table, num_cache_pages,
                                      k_cache, v_cache, partial_bf16, workspace, workspace_bytes, stream);
}

moe_status_t attn_block_decode_partial(attn_block_t* L, const void* x_bf16, int B, const int32_t* positions,
                                       const int32_t* page_table, int num_cache_pages, void* k_cache, void* v_cache,
                                       void* partial_bf16, void* workspace, size_t workspace_bytes, cwStream_t stream) {
    return attn_block_forward_partial(L, x_bf16, B, positions, nullptr, B > 0 ? B : 1, page_table, num_cache_pages,
                                      k_cache, v_cache, partial_bf16, workspace, workspace_bytes, stream);
}

moe_status_t attn_block_prefill(attn_block_t* L, const void* x_bf16, int B, const int32_t* positions,
                                const int32_t* row_seq, int num_seqs, int prefill_rows, const int32_t* page_table,
                                int num_cache_pages, void* k_cache, void* v_cache, void* out_bf16, void* workspace,
                                size_t workspace_bytes, cwStream_t stream) {
    if (!L || B < 0 || B > L->cfg.max_batch || num_seqs <= 0) return MOE_ERR_INVALID_ARGUMENT;
    if (prefill_rows < 0 || prefill_rows > B) return MOE_ERR_INVALID_ARGUMENT;
    if (!x_bf16 || !positions || !page_table || !k_cache || !v_cache || !out_bf16 || !workspace)
        return MOE_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < L->bytes) return MOE_ERR_WORKSPACE;
    if (L->cfg.tp_size > 1 && !L->peer_mode) return MOE_ERR_UNSUPPORTED;   // peer buffers not set
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t n = static_cast<size_t>(B) * L->cfg.hidden;
    const int blocks = static_cast<int>((n / 8 + 255) / 256);
    if (L->cfg.tp_size == 1) {
        if (B == 0) return MOE_OK;
        void* part = at<void>(workspace, L->off_part);
        ATT_TRY(run_partial(L, x_bf16, B, positions, row_seq, num_seqs, prefill_rows, page_table, num_cache_pages,
                            k_cache, v_cache, part, workspace, st));
        residual_add_kernel<<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(part),
                                                    static_cast<const __nv_bfloat16*>(x_bf16), n,
                                                    static_cast<__nv_bfloat16*>(out_bf16));
        return launch_status();
    }
    // every rank takes every step (even with B == 0): the flags pair up calls
    void* part = L->peers.base[L->peers.me] + kFlagBytes;
    tp_wait_done_kernel<<<1, 32, 0, st>>>(L->peers, L->epoch_dev, L->timeout_ns, L->error_word);
    ATT_TRY(launch_status());
    if (B > 0)
        ATT_TRY(run_partial(L, x_bf16, B, positions, row_seq, num_seqs, prefill_rows, page_table, num_cache_pages,
                            k_cache, v_cache, part, workspace, st));
    tp_signal_kernel<<<1, 32, 0, st>>>(L->peers, L->epoch_dev);
    ATT_TRY(launch_status());
    if (B > 0) {
        tp_peer_reduce_kernel<<<blocks, 256, 0, st>>>(L->peers, L->epoch_dev, static_cast<const __nv_bfloat16*>(x_bf16),
                                                      n, static_cast<__nv_bfloat16*>(out_bf16), L->timeout_ns,
                                                      L->error_word);
        ATT_TRY(launch_status());
    }
    tp_done_kernel<<<1, 32, 0, st>>>(L->peers, L->epoch_dev);
    return launch_status();
}

moe_status_t attn_block_forward(attn_block_t* L, const void* x_bf16, int B, const int32_t* positions,
                                const int32_t* row_seq, int num_seqs, const int32_t* page_table, int num_cache_pages,
                                void* k_cache, void* v_cache, void* out_bf16, void* workspace, size_t workspace_bytes,
                                cwStream_t stream) {
    return attn_block_prefill(L, x_bf16, B, positions, row_seq, num_seqs, 0, page_table, num_cache_pages, k_cache,
                              v_cache, out_bf16, workspace, workspace_bytes, stream);
}

moe_status_t attn_block_decode(attn_block_t* L, const void* x_bf16, int B, const int32_t* positions,
                               const int32_t* page_table, int num_cache_pages, void* k_cache, void* v_cache,
                               void* out_bf16, void* workspace, size_t workspace_bytes, cwStream_t stream) {
    return attn_block_forward(L, x_bf16, B, positions, nullptr, B > 0 ? B : 1, page_table, num_cache_pages, k_cache,
                              v_cache, out_bf16, workspace, workspace_bytes, stream);
}

moe_status_t attn_block_check_error(attn_block_t* L, cwStream_t stream) {
    if (!L) return MOE_ERR_INVALID_ARGUMENT;
    int h = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&h, L->error_word, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return MOE_ERR_CUDA;
    cudaMemsetAsync(L->error_word, 0, sizeof(int), st);
    if (h == 0) return MOE_OK;
    // 1: a GEMM wait gave up, 3: a peer flag wait gave up; 4-7: positions,
    // lengths, page ids or sequence rows outside the given tables
    return (h == 1 || h == 3) ? MOE_ERR_DEVICE_TIMEOUT : MOE_ERR_INVALID_ARGUMENT;
}

}  // extern "C"
