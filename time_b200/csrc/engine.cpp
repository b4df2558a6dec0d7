// engine.cpp -- the decoder serving engine (include/engine.h): requests, the
// KV page pool and the batched forward over all layers.  Host code; the
// device work is the attention block (attn_block.cu), the MoE layer
// (moe_layer.cu), cuBLAS for the bf16 lm_head and engine_kernels.cu.
//
// The reference keeps the same pieces in src/terra/engine.t: the request
// state (create_request_state, engine.t:974-1030), the page allocator
// (allocate_kv_pages / free_kv_pages, engine.t:793-856), prefill and decode
// (run_prefill / run_decode_step, engine.t:1373-1512) and the opaque entry
// points (engine.t:1833-1903).  Here prefill_opaque only admits a request;
// a decode step runs every request in flight together -- the positions of
// admitted prompts that have no K/V yet, request by request, in forwards of
// at most rows_cap rows, the last forward ending with each request's newest
// position (the sampled rows).  One forward:
//
//   stage (pinned)   token, position, page-table row of every row, and seed,
//                    temperature, top_p of every sampled row -> one copy
//   embed            bf16 rows
//   per layer        attn_block_prefill (RoPE + K/V page write; prompt rows
//                    through the prefill attention kernel, sampled rows through
//                    split decode; o_proj + residual), then the FFN: moe_layer_forward
//                    (routed experts + shared expert + residual) or, for the
//                    first dense layers, the same layer with one expert
//   final norm       bf16, the sampled rows only
//   lm_head          cuBLAS bf16 GEMM, fp32 logits [sampled rows][vocab]
//   sample           one warp per row; the tokens come back in one copy
//
// row_seq maps every row to its request's page-table row, and every row's K/V
// is written before any row attends, so prompt rows in one forward are causal.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <unordered_set>
#include <vector>

#include "engine.h"
#include "cublas_wrappers.h"
#include "engine_kernels.h"
#include "json_lite.h"
#include "st_loader.h"

namespace {

constexpr int kPage = 16;
constexpr int kHeadDim = 128;

struct Request {
    int64_t id = 0;
    int slot = -1;
    std::vector<int64_t> tokens;   // prompt then generated tokens
    int generated = 0;
    int max_tokens = 0;
    float temperature = 1.0f, top_p = 1.0f, rep_penalty = 1.0f;
    std::vector<int32_t> pages;
    int kv_len = 0;                // positions whose K/V are in the pages
    bool finished = false;
};

struct Layer {
    attn_block_t* attn = nullptr;
    moe_layer_t* ffn = nullptr;
    bool dense = false;
    void* k_cache = nullptr;
    void* v_cache = nullptr;
};

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Staging layout of one forward's per-row inputs (pinned host and device
// copies; R = rows_cap, a multiple of 16).
struct StageLayout {
    size_t tokens, seeds, pos, row_seq, temp, top_p, bytes;
    explicit StageLayout(size_t R = 0) {
        tokens = 0;
        seeds = tokens + R * 8;
        pos = seeds + R * 8;
        row_seq = pos + R * 4;
        temp = row_seq + R * 4;
        top_p = temp + R * 4;
        bytes = top_p + R * 4;
    }
};

}  // namespace

struct glm_engine {
    glm_engine_config_t cfg{};
    int rows_cap = 0;            // max(max_batch, prefill_chunk), rounded to 16
    int max_pages_per_seq = 0;
    int num_pages = 0;
    int device = 0;
    int num_gpus_requested = 1;
    int num_tensors = 0;
    cudaStream_t stream = nullptr;
    cublasHandle_t cublas = nullptr;
    std::vector<Layer> layers;
    const void* embed = nullptr;
    const float* final_norm = nullptr;
    const void* lm_head = nullptr;
    std::vector<void*> owned;    // weights loaded by init_engine
    // engine buffers (device)
    void* kv = nullptr;
    size_t kv_layer_bytes = 0;   // one of k / v for one layer
    void* x0 = nullptr;
    void* x1 = nullptr;
    void* xn = nullptr;
    float* logits = nullptr;
    int64_t* tokens_out = nullptr;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int32_t* page_table = nullptr;
    int32_t* dense_idx = nullptr;
    float* dense_w = nullptr;
    float* dummy_router = nullptr;
    int* error_word = nullptr;
    uint8_t* stage_dev = nullptr;
    // pinned host
    int32_t* page_table_host = nullptr;
    uint8_t* stage_host = nullptr;
    int64_t* tokens_host = nullptr;
    StageLayout stage;
    // pool
    std::vector<int32_t> free_pages;
    std::vector<int> free_slots;
    std::unordered_set<Request*> requests;
    std::mutex mu;
    int last_rows = 0;
    bool timing = false;
    std::vector<cudaEvent_t> events;
    float stage_ms[4] = {0, 0, 0, 0};
    // routing capture (tests): [layer][rows_cap][top_k] of the last forward
    int32_t* cap_idx = nullptr;
    float* cap_w = nullptr;
    int cap_rows = 0;
    // ... gathered on the host over all forwards of the last step: [layer][row][top_k]
    std::vector<std::vector<int32_t>> cap_step_idx;
    std::vector<std::vector<float>> cap_step_w;
    // several GPUs (cfg.num_gpus > 1): this object is rank `rank` of `world`,
    // one per device; rank 0 holds the requests, the host buffers and the
    // head, and owns the other ranks' objects (ranks[0] == rank 0 itself)
    int rank = 0, world = 1;
    std::vector<glm_engine*> ranks;
    glm_engine* root = nullptr;
    void* x2 = nullptr;              // the other residual-stream buffer: layers alternate x0 / x2
    uint32_t* gather_flags = nullptr;   // [kMaxGatherRanks] epochs raised by every rank
    uint32_t* gather_epoch = nullptr;   // this rank's all-gather epoch (device)
    unsigned int* gather_done = nullptr;
    std::vector<void*> peer_bufs;    // attention / FFN peer buffers this rank allocated
    moe_status_t thread_status = MOE_OK;
    // one GPU: a pure decode step of R rows replays a CUDA graph of the whole
    // forward (stage copy, 92 layers, head, token copy), captured the second
    // time R occurs; off with TIME_B200_ENGINE_GRAPHS=0, timing or routing capture
    bool graphs_ok = true;
    std::map<int, cudaGraphExec_t> graph_exec;
    std::map<int, int> graph_seen;
};

namespace {

#define ENG_TRY(x)                          \
    do {                                    \
        const moe_status_t s_ = (x);        \
        if (s_ != MOE_OK) return s_;        \
    } while (0)
#define ENG_CUDA(x)                                      \
    do {                                                 \
        if ((x) != cudaSuccess) return MOE_ERR_CUDA;     \
    } while (0)

bool config_ok(const glm_engine_config_t& c) {
    return c.hidden > 0 && c.hidden % 128 == 0 && c.num_layers > 0 && c.first_dense >= 0 &&
           c.first_dense <= c.num_layers && c.num_q_heads > 0 && c.num_kv_heads > 0 &&
           c.num_q_heads % c.num_kv_heads == 0 && c.head_dim == kHeadDim && c.rotary_dim >= 0 &&
           c.rotary_dim <= kHeadDim && c.rotary_dim % 2 == 0 && c.vocab_size > 0 &&
           (c.first_dense == c.num_layers ||
            (c.num_experts > 0 && c.top_k > 0 && c.top_k <= c.num_experts && c.moe_intermediate > 0 &&
             c.moe_intermediate % 128 == 0 && (c.num_shared == 0 || c.num_shared == 1))) &&
           (c.first_dense == 0 || (c.dense_intermediate > 0 && c.dense_intermediate % 128 == 0)) &&
           c.rope_theta > 0.0f && c.rms_eps > 0.0f && c.max_batch > 0 && c.max_seq > 0 && c.prefill_chunk >= 0 &&
           c.num_cache_pages >= 0;
}

struct Plan {
    int rows_cap, max_pages_per_seq, num_pages;
    size_t kv_layer_bytes, kv_bytes, act_bytes, logits_bytes, small_bytes;
};

Plan make_plan(const glm_engine_config_t& c) {
    Plan p{};
    const int chunk = c.prefill_chunk > 0 ? c.prefill_chunk : 2048;
    p.rows_cap = static_cast<int>(align_up(static_cast<size_t>(std::max(c.max_batch, chunk)), 16));
    p.max_pages_per_seq = (c.max_seq + kPage - 1) / kPage;
    p.num_pages = c.num_cache_pages > 0 ? c.num_cache_pages : c.max_batch * p.max_pages_per_seq;
    const int world = c.num_gpus > 1 ? c.num_gpus : 1;
    p.kv_layer_bytes =
        align_up(static_cast<size_t>(p.num_pages) * kPage * (c.num_kv_heads / world) * kHeadDim * 2, 256);
    p.kv_bytes = p.kv_layer_bytes * 2 * c.num_layers;
    p.act_bytes = static_cast<size_t>(p.rows_cap) * c.hidden * 2;
    p.logits_bytes = static_cast<size_t>(c.max_batch) * c.vocab_size * 4;
    p.small_bytes = static_cast<size_t>(c.max_batch) * p.max_pages_per_seq * 4 + p.rows_cap * (8 + 4 + 4) +
                    c.hidden * 4 + StageLayout(p.rows_cap).bytes;
    return p;
}

template <typename T>
cudaError_t dev_alloc(T** p, size_t bytes) {
    void* v = nullptr;
    const cudaError_t e = cudaMalloc(&v, bytes);
    *p = static_cast<T*>(v);
    return e;
}

void destroy_one(glm_engine* E) {
    if (!E) return;
    if (E->stream) cudaStreamSynchronize(E->stream);
    for (auto& kv : E->graph_exec) cudaGraphExecDestroy(kv.second);
    E->graph_exec.clear();
    for (Request* r : E->requests) delete r;
    E->requests.clear();
    for (Layer& L : E->layers) {
        if (L.attn) attn_block_destroy(L.attn);
        if (L.ffn) moe_layer_destroy(L.ffn);
    }
    for (void* p : E->owned) cudaFree(p);
    void* dev[] = {E->kv, E->x0, E->x1, E->xn, E->logits, E->tokens_out, E->ws, E->page_table, E->dense_idx,
                   E->dense_w, E->dummy_router, E->error_word, E->stage_dev, E->cap_idx, E->cap_w, E->x2,
                   E->gather_flags, E->gather_epoch, E->gather_done};
    for (void* p : dev)
        if (p) cudaFree(p);
    for (void* p : E->peer_bufs) cudaFree(p);
    void* host[] = {E->page_table_host, E->stage_host, E->tokens_host};
    for (void* p : host)
        if (p) cudaFreeHost(p);
    for (cudaEvent_t ev : E->events) cudaEventDestroy(ev);
    if (E->cublas) cublasDestroy(E->cublas);
    if (E->stream) cudaStreamDestroy(E->stream);
    delete E;
}

// Every rank (each on its own device), then rank 0.
void destroy(glm_engine* E) {
    if (!E) return;
    for (size_t r = 1; r < E->ranks.size(); ++r) {
        cudaSetDevice(E->ranks[r]->device);
        destroy_one(E->ranks[r]);
    }
    cudaSetDevice(E->device);
    destroy_one(E);
}

// One rank's device state on the current device.
moe_status_t create_one(const glm_engine_config_t* cfg, int rank, int world, glm_engine** out) {
    if (!cfg || !out || !config_ok(*cfg)) return MOE_ERR_INVALID_ARGUMENT;
    glm_engine* E = new (std::nothrow) glm_engine();
    if (!E) return MOE_ERR_INVALID_ARGUMENT;
    E->cfg = *cfg;
    E->rank = rank;
    E->world = world;
    E->root = E;
    {
        const char* g = std::getenv("TIME_B200_ENGINE_GRAPHS");
        E->graphs_ok = !(g && g[0] == '0');
    }
    if (E->cfg.prefill_chunk <= 0) E->cfg.prefill_chunk = 2048;
    const Plan p = make_plan(E->cfg);
    E->rows_cap = p.rows_cap;
    E->max_pages_per_seq = p.max_pages_per_seq;
    E->num_pages = p.num_pages;
    E->kv_layer_bytes = p.kv_layer_bytes;
    E->stage = StageLayout(p.rows_cap);
    E->layers.resize(cfg->num_layers);
    const size_t H = cfg->hidden;
    bool ok = cudaGetDevice(&E->device) == cudaSuccess &&
              cudaStreamCreateWithFlags(&E->stream, cudaStreamNonBlocking) == cudaSuccess &&
              cublasCreate(&E->cublas) == CUBLAS_STATUS_SUCCESS &&
              cublasSetStream(E->cublas, E->stream) == CUBLAS_STATUS_SUCCESS &&
              dev_alloc(&E->kv, p.kv_bytes) == cudaSuccess && dev_alloc(&E->x0, p.act_bytes) == cudaSuccess &&
              dev_alloc(&E->x1, p.act_bytes) == cudaSuccess &&
              dev_alloc(&E->xn, static_cast<size_t>(cfg->max_batch) * H * 2) == cudaSuccess &&
              dev_alloc(&E->logits, p.logits_bytes) == cudaSuccess &&
              dev_alloc(&E->tokens_out, static_cast<size_t>(p.rows_cap) * 8) == cudaSuccess &&
              dev_alloc(&E->page_table, static_cast<size_t>(cfg->max_batch) * p.max_pages_per_seq * 4) == cudaSuccess &&
              dev_alloc(&E->dense_idx, static_cast<size_t>(p.rows_cap) * 4) == cudaSuccess &&
              dev_alloc(&E->dense_w, static_cast<size_t>(p.rows_cap) * 4) == cudaSuccess &&
              dev_alloc(&E->dummy_router, H * 4) == cudaSuccess && dev_alloc(&E->error_word, 4) == cudaSuccess &&
              dev_alloc(&E->stage_dev, E->stage.bytes) == cudaSuccess &&
              cudaHostAlloc(reinterpret_cast<void**>(&E->page_table_host),
                            static_cast<size_t>(cfg->max_batch) * p.max_pages_per_seq * 4, 0) == cudaSuccess &&
              cudaHostAlloc(reinterpret_cast<void**>(&E->stage_host), E->stage.bytes, 0) == cudaSuccess &&
              cudaHostAlloc(reinterpret_cast<void**>(&E->tokens_host), static_cast<size_t>(p.rows_cap) * 8, 0) ==
                  cudaSuccess &&
              (world == 1 || (dev_alloc(&E->x2, p.act_bytes) == cudaSuccess &&
                              dev_alloc(&E->gather_flags, tb_engine::kMaxGatherRanks * 4) == cudaSuccess &&
                              dev_alloc(&E->gather_epoch, 4) == cudaSuccess &&
                              dev_alloc(&E->gather_done, 4) == cudaSuccess &&
                              cudaMemset(E->gather_flags, 0, tb_engine::kMaxGatherRanks * 4) == cudaSuccess &&
                              cudaMemset(E->gather_epoch, 0, 4) == cudaSuccess &&
                              cudaMemset(E->gather_done, 0, 4) == cudaSuccess));
    if (ok) {
        // K/V pages are zero until written (a page id is never read before
        // its slot is written, but the pool starts clean); the dense layers'
        // routing is expert 0 with weight 1.0
        std::vector<float> ones(p.rows_cap, 1.0f);
        ok = cudaMemset(E->kv, 0, p.kv_bytes) == cudaSuccess &&
             cudaMemset(E->dense_idx, 0, static_cast<size_t>(p.rows_cap) * 4) == cudaSuccess &&
             cudaMemcpy(E->dense_w, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemset(E->dummy_router, 0, H * 4) == cudaSuccess && cudaMemset(E->error_word, 0, 4) == cudaSuccess &&
             cudaMemset(E->page_table, 0, static_cast<size_t>(cfg->max_batch) * p.max_pages_per_seq * 4) ==
                 cudaSuccess;
    }
    if (!ok) {
        cudaGetLastError();
        destroy(E);
        return MOE_ERR_CUDA;
    }
    std::memset(E->page_table_host, 0, static_cast<size_t>(cfg->max_batch) * p.max_pages_per_seq * 4);
    for (int l = 0; l < cfg->num_layers; ++l) {
        E->layers[l].k_cache = static_cast<uint8_t*>(E->kv) + (2 * static_cast<size_t>(l)) * p.kv_layer_bytes;
        E->layers[l].v_cache = static_cast<uint8_t*>(E->kv) + (2 * static_cast<size_t>(l) + 1) * p.kv_layer_bytes;
        E->layers[l].dense = l < cfg->first_dense;
    }
    E->free_pages.reserve(E->num_pages);
    for (int i = E->num_pages - 1; i >= 0; --i) E->free_pages.push_back(i);
    for (int s = cfg->max_batch - 1; s >= 0; --s) E->free_slots.push_back(s);
    *out = E;
    return MOE_OK;
}

// The engine: one rank, or cfg->num_gpus ranks on the devices from the
// current one on, with peer access between every pair.
moe_status_t create(const glm_engine_config_t* cfg, glm_engine** out) {
    if (!cfg || !out) return MOE_ERR_INVALID_ARGUMENT;
    const int N = cfg->num_gpus > 1 ? cfg->num_gpus : 1;
    if (N == 1) return create_one(cfg, 0, 1, out);
    const glm_engine_config_t& c = *cfg;
    if (N > tb_engine::kMaxGatherRanks || c.num_q_heads % N || c.num_kv_heads % N ||
        (c.first_dense < c.num_layers && c.num_experts % N))
        return MOE_ERR_INVALID_ARGUMENT;
    int dev0 = 0, count = 0;
    if (cudaGetDevice(&dev0) != cudaSuccess || cudaGetDeviceCount(&count) != cudaSuccess) return MOE_ERR_CUDA;
    if (dev0 + N > count) return MOE_ERR_INVALID_ARGUMENT;
    for (int a = 0; a < N; ++a) {
        if (cudaSetDevice(dev0 + a) != cudaSuccess) return MOE_ERR_CUDA;
        for (int b = 0; b < N; ++b) {
            if (a == b) continue;
            int can = 0;
            if (cudaDeviceCanAccessPeer(&can, dev0 + a, dev0 + b) != cudaSuccess || !can) {
                cudaSetDevice(dev0);
                return MOE_ERR_UNSUPPORTED;
            }
            const cudaError_t e = cudaDeviceEnablePeerAccess(dev0 + b, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (e != cudaSuccess) {
                cudaSetDevice(dev0);
                return MOE_ERR_CUDA;
            }
        }
    }
    std::vector<glm_engine*> ranks(N, nullptr);
    moe_status_t st = MOE_OK;
    for (int r = 0; r < N && st == MOE_OK; ++r) {
        if (cudaSetDevice(dev0 + r) != cudaSuccess) st = MOE_ERR_CUDA;
        else st = create_one(cfg, r, N, &ranks[r]);
    }
    cudaSetDevice(dev0);
    if (st != MOE_OK) {
        for (int r = N - 1; r >= 0; --r)
            if (ranks[r]) {
                cudaSetDevice(dev0 + r);
                destroy_one(ranks[r]);
            }
        cudaSetDevice(dev0);
        return st;
    }
    for (glm_engine* R : ranks) R->root = ranks[0];
    ranks[0]->ranks = ranks;
    *out = ranks[0];
    return MOE_OK;
}

// Layer l of one rank (the rank's device current): attention with the
// rank's heads (tp = world), the FFN for the rank's slice of the rows (EP =
// world for a MoE layer, the whole dense FFN).
moe_status_t set_layer_one(glm_engine* E, int l, const attn_block_weights_t* aw, const moe_layer_weights_t* fw) {
    if (!E || l < 0 || l >= E->cfg.num_layers || !aw || !fw) return MOE_ERR_INVALID_ARGUMENT;
    const glm_engine_config_t& c = E->cfg;
    Layer& L = E->layers[l];
    if (L.attn || L.ffn) return MOE_ERR_INVALID_ARGUMENT;   // once per layer
    attn_block_config_t ac{};
    ac.hidden = c.hidden;
    ac.num_q_heads = c.num_q_heads / E->world;
    ac.num_kv_heads = c.num_kv_heads / E->world;
    ac.head_dim = c.head_dim;
    ac.rotary_dim = c.rotary_dim;
    ac.rope_theta = c.rope_theta;
    ac.eps = c.rms_eps;
    ac.max_batch = E->rows_cap;
    ac.max_pages_per_seq = E->max_pages_per_seq;
    ac.max_context = E->max_pages_per_seq * kPage;
    ac.tp_size = E->world;
    ac.tp_rank = E->rank;
    ENG_TRY(attn_block_create(&ac, aw, &L.attn));
    moe_layer_config_t mc{};
    mc.hidden = c.hidden;
    mc.rms_eps = c.rms_eps;
    mc.max_tokens = (E->rows_cap + E->world - 1) / E->world;   // this rank's slice of a forward's rows
    mc.ep_size = L.dense ? 1 : E->world;
    mc.ep_rank = L.dense ? 0 : E->rank;
    moe_layer_weights_t w = *fw;
    if (L.dense) {
        mc.num_experts = 1;
        mc.top_k = 1;
        mc.intermediate = c.dense_intermediate;
        mc.num_shared = 0;
        w.router_w = E->dummy_router;
        w.router_bias = nullptr;
    } else {
        mc.num_experts = c.num_experts;
        mc.top_k = c.top_k;
        mc.intermediate = c.moe_intermediate;
        mc.num_shared = c.num_shared;
    }
    const moe_status_t s = moe_layer_create(&mc, &w, nullptr, &L.ffn);
    if (s != MOE_OK) {
        attn_block_destroy(L.attn);
        L.attn = nullptr;
        L.ffn = nullptr;
        return s;
    }
    return MOE_OK;
}

// Layer l is set on every rank: one zero-filled peer buffer per rank for its
// attention sum and its expert exchange, every rank given all of them.
moe_status_t setup_layer_peers(glm_engine* root, int l) {
    const int N = root->world;
    std::vector<void*> ab(N, nullptr), fb(N, nullptr);
    const size_t abytes = attn_block_peer_bytes(root->layers[l].attn);
    const size_t fbytes = moe_layer_peer_bytes(root->layers[l].ffn);
    moe_status_t st = MOE_OK;
    for (int r = 0; r < N && st == MOE_OK; ++r) {
        glm_engine* R = root->ranks[r];
        if (cudaSetDevice(R->device) != cudaSuccess) st = MOE_ERR_CUDA;
        if (st == MOE_OK && abytes) {
            if (dev_alloc(&ab[r], abytes) != cudaSuccess || cudaMemset(ab[r], 0, abytes) != cudaSuccess) st = MOE_ERR_CUDA;
            if (ab[r]) R->peer_bufs.push_back(ab[r]);
        }
        if (st == MOE_OK && fbytes) {
            if (dev_alloc(&fb[r], fbytes) != cudaSuccess || cudaMemset(fb[r], 0, fbytes) != cudaSuccess) st = MOE_ERR_CUDA;
            if (fb[r]) R->peer_bufs.push_back(fb[r]);
        }
        if (st == MOE_OK && cudaDeviceSynchronize() != cudaSuccess) st = MOE_ERR_CUDA;
    }
    for (int r = 0; r < N && st == MOE_OK; ++r) {
        glm_engine* R = root->ranks[r];
        cudaSetDevice(R->device);
        if (abytes) st = attn_block_set_peer_buffers(R->layers[l].attn, ab.data(), N);
        if (st == MOE_OK && fbytes) st = moe_layer_set_peer_buffers(R->layers[l].ffn, fb.data(), N);
    }
    cudaSetDevice(root->device);
    return st;
}

// Rank `rank`'s layer l; once every rank has it, the peer buffers.
moe_status_t set_layer(glm_engine* E, int rank, int l, const attn_block_weights_t* aw, const moe_layer_weights_t* fw) {
    if (!E || rank < 0 || rank >= E->world || l < 0 || l >= E->cfg.num_layers) return MOE_ERR_INVALID_ARGUMENT;
    glm_engine* R = E->world > 1 ? E->ranks[rank] : E;
    if (cudaSetDevice(R->device) != cudaSuccess) return MOE_ERR_CUDA;
    moe_status_t st = set_layer_one(R, l, aw, fw);
    if (st == MOE_OK && E->world > 1) {
        bool all = true;
        for (glm_engine* P : E->ranks) all = all && P->layers[l].attn && P->layers[l].ffn;
        if (all) st = setup_layer_peers(E, l);
    }
    cudaSetDevice(E->device);
    return st;
}

// Every layer and the embedding are set: size and allocate the workspace.
// The first call also waits for the whole device once, so that weights the
// caller wrote on any stream are complete before the engine's stream reads them.
moe_status_t ensure_ready_one(glm_engine* E) {
    if (E->ws) return MOE_OK;
    if (!E->embed || (E->rank == 0 && (!E->final_norm || !E->lm_head))) return MOE_ERR_INVALID_ARGUMENT;
    size_t need = 0;
    for (const Layer& L : E->layers) {
        if (!L.attn || !L.ffn) return MOE_ERR_INVALID_ARGUMENT;
        need = std::max(need, attn_block_workspace_bytes(L.attn));
        need = std::max(need, moe_layer_workspace_bytes(L.ffn));
    }
    ENG_CUDA(cudaDeviceSynchronize());
    ENG_CUDA(dev_alloc(&E->ws, need));
    E->ws_bytes = need;
    return MOE_OK;
}

moe_status_t ensure_ready(glm_engine* E) {
    if (E->world == 1) return ensure_ready_one(E);
    moe_status_t st = MOE_OK;
    for (glm_engine* R : E->ranks) {
        if (st != MOE_OK) break;
        if (cudaSetDevice(R->device) != cudaSuccess) st = MOE_ERR_CUDA;
        else st = ensure_ready_one(R);
    }
    cudaSetDevice(E->device);
    return st;
}

void set_events(glm_engine* E, bool on) {
    for (cudaEvent_t ev : E->events) cudaEventDestroy(ev);
    E->events.clear();
    E->timing = false;
    if (!on) return;
    const size_t n = 2 * E->layers.size() + 3;
    for (size_t i = 0; i < n; ++i) {
        cudaEvent_t ev;
        if (cudaEventCreate(&ev) != cudaSuccess) {
            set_events(E, false);
            return;
        }
        E->events.push_back(ev);
    }
    E->timing = true;
}

// One forward over R staged rows (already copied to the device).  With
// head > 0: rows [R - head, R) also go through the final norm, the lm_head
// and the sampler (per-row parameters at stage indices 0..head-1), and the
// tokens come back to tokens_host.
moe_status_t forward_one(glm_engine* E, int R, int head, bool sync = true) {
    const bool sample = head > 0;
    const glm_engine_config_t& c = E->cfg;
    cudaStream_t st = E->stream;
    const int64_t* tokens = reinterpret_cast<const int64_t*>(E->stage_dev + E->stage.tokens);
    const int32_t* pos = reinterpret_cast<const int32_t*>(E->stage_dev + E->stage.pos);
    const int32_t* row_seq = reinterpret_cast<const int32_t*>(E->stage_dev + E->stage.row_seq);
    const bool tm = E->timing && sample;
    if (tm) cudaEventRecord(E->events[0], st);
    ENG_CUDA(tb_engine::embed_rows(E->embed, tokens, R, c.vocab_size, c.hidden, E->x0, E->error_word, st));
    for (size_t l = 0; l < E->layers.size(); ++l) {
        Layer& L = E->layers[l];
        if (tm) cudaEventRecord(E->events[1 + 2 * l], st);
        // rows [0, R - head) are prompt positions (the prefill kernel), the last `head` the sampled rows
        ENG_TRY(attn_block_prefill(L.attn, E->x0, R, pos, row_seq, c.max_batch, R - head, E->page_table, E->num_pages,
                                   L.k_cache, L.v_cache, E->x1, E->ws, E->ws_bytes, st));
        if (tm) cudaEventRecord(E->events[2 + 2 * l], st);
        if (L.dense)
            ENG_TRY(moe_layer_forward_routed(L.ffn, E->x1, E->dense_idx, E->dense_w, E->x0, R, E->ws, E->ws_bytes, st));
        else
            ENG_TRY(moe_layer_forward(L.ffn, E->x1, E->x0, R, E->ws, E->ws_bytes, st));
        if (E->cap_idx && !L.dense) {
            const int32_t* idx;
            const float* w;
            const int32_t* cnt;
            ENG_TRY(moe_layer_last_routing(L.ffn, E->ws, &idx, &w, &cnt));
            const size_t n = static_cast<size_t>(R) * c.top_k, off = l * static_cast<size_t>(E->rows_cap) * c.top_k;
            ENG_CUDA(cudaMemcpyAsync(E->cap_idx + off, idx, n * 4, cudaMemcpyDeviceToDevice, st));
            ENG_CUDA(cudaMemcpyAsync(E->cap_w + off, w, n * 4, cudaMemcpyDeviceToDevice, st));
        }
    }
    E->cap_rows = R;
    if (E->cap_idx) {   // keep this forward's routing with the step's (tests only: synchronises)
        ENG_CUDA(cudaStreamSynchronize(st));
        for (size_t l = 0; l < E->layers.size(); ++l) {
            if (E->layers[l].dense) continue;
            const size_t n = static_cast<size_t>(R) * c.top_k, off = l * static_cast<size_t>(E->rows_cap) * c.top_k;
            std::vector<int32_t>& vi = E->cap_step_idx[l];
            std::vector<float>& vw = E->cap_step_w[l];
            const size_t o = vi.size();
            vi.resize(o + n);
            vw.resize(o + n);
            ENG_CUDA(cudaMemcpy(vi.data() + o, E->cap_idx + off, n * 4, cudaMemcpyDeviceToHost));
            ENG_CUDA(cudaMemcpy(vw.data() + o, E->cap_w + off, n * 4, cudaMemcpyDeviceToHost));
        }
    }
    if (!sample) return cudaStreamSynchronize(st) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
    const size_t nl = E->layers.size();
    if (tm) cudaEventRecord(E->events[1 + 2 * nl], st);
    const void* head_x = static_cast<const uint8_t*>(E->x0) + static_cast<size_t>(R - head) * c.hidden * 2;
    ENG_CUDA(tb_engine::final_norm_rows(head_x, E->final_norm, head, c.hidden, c.rms_eps, E->xn, st));
    // logits [R][V] (row-major) = xn [R][H] . lm_head [V][H]^T: column-major
    // C [V][R] = A^T B with A = lm_head as [H][V], B = xn as [H][R]
    const float one = 1.0f, zero = 0.0f;
    if (cublasGemmEx(E->cublas, CUBLAS_OP_T, CUBLAS_OP_N, c.vocab_size, head, c.hidden, &one, E->lm_head, CUDA_R_16BF,
                     c.hidden, E->xn, CUDA_R_16BF, c.hidden, &zero, E->logits, CUDA_R_32F, c.vocab_size,
                     CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS)
        return MOE_ERR_CUDA;
    ENG_CUDA(tb_engine::sample_rows(E->logits, head, c.vocab_size,
                                    reinterpret_cast<const float*>(E->stage_dev + E->stage.temp),
                                    reinterpret_cast<const float*>(E->stage_dev + E->stage.top_p),
                                    reinterpret_cast<const uint64_t*>(E->stage_dev + E->stage.seeds), E->tokens_out,
                                    st));
    if (tm) cudaEventRecord(E->events[2 + 2 * nl], st);
    ENG_CUDA(cudaMemcpyAsync(E->tokens_host, E->tokens_out, static_cast<size_t>(head) * 8, cudaMemcpyDeviceToHost, st));
    if (!sync) return MOE_OK;   // being captured into a graph
    ENG_CUDA(cudaStreamSynchronize(st));
    if (tm) {
        float ms = 0.0f, attn = 0.0f, ffn = 0.0f;
        cudaEventElapsedTime(&ms, E->events[0], E->events[1]);
        E->stage_ms[0] = ms;
        for (size_t l = 0; l < nl; ++l) {
            cudaEventElapsedTime(&ms, E->events[1 + 2 * l], E->events[2 + 2 * l]);
            attn += ms;
            cudaEventElapsedTime(&ms, E->events[2 + 2 * l], E->events[3 + 2 * l]);
            ffn += ms;
        }
        E->stage_ms[1] = attn;
        E->stage_ms[2] = ffn;
        cudaEventElapsedTime(&ms, E->events[1 + 2 * nl], E->events[2 + 2 * nl]);
        E->stage_ms[3] = ms;
    }
    return MOE_OK;
}

// Rank P's part of a forward over R staged rows (several GPUs): the
// attention of every layer on all rows (tensor parallel), the FFN on the
// rank's rows [lo, hi), then those rows stored into every rank's buffer
// before the next layer; the layers alternate between x0 and x2 so that a
// rank that is ahead never overwrites rows another rank still reads.  Rank 0
// then runs the head on the sampled rows.
moe_status_t forward_rank(glm_engine* P, int R, int head, bool sync = true) {
    glm_engine* E = P->root;
    const glm_engine_config_t& c = P->cfg;
    ENG_CUDA(cudaSetDevice(P->device));
    cudaStream_t st = P->stream;
    const bool sample = head > 0;
    const bool tm = P->rank == 0 && E->timing && sample;
    ENG_CUDA(cudaMemcpyAsync(P->stage_dev, E->stage_host, E->stage.bytes, cudaMemcpyHostToDevice, st));
    const int64_t* tokens = reinterpret_cast<const int64_t*>(P->stage_dev + P->stage.tokens);
    const int32_t* pos = reinterpret_cast<const int32_t*>(P->stage_dev + P->stage.pos);
    const int32_t* row_seq = reinterpret_cast<const int32_t*>(P->stage_dev + P->stage.row_seq);
    if (tm) cudaEventRecord(E->events[0], st);
    ENG_CUDA(tb_engine::embed_rows(P->embed, tokens, R, c.vocab_size, c.hidden, P->x0, P->error_word, st));
    tb_engine::GatherSet G{};
    G.world = P->world;
    G.me = P->rank;
    for (int r = 0; r < P->world; ++r) G.flags[r] = E->ranks[r]->gather_flags;
    const int lo = static_cast<int>(static_cast<long long>(R) * P->rank / P->world);
    const int hi = static_cast<int>(static_cast<long long>(R) * (P->rank + 1) / P->world);
    const size_t row_bytes = static_cast<size_t>(c.hidden) * 2;
    const size_t nl = P->layers.size();
    void* xfinal = P->x0;
    // the grouped-GEMM form from the forward's rows, which every rank knows (the
    // one-GPU rule on R): all ranks of an expert-parallel layer take the same one
    const int form = c.num_experts > 1 && static_cast<long long>(R) * c.top_k <= 16ll * c.num_experts
                         ? CBW_GEMM_SMALL_TILES
                         : CBW_GEMM_FULL_TILES;
    for (size_t l = 0; l < nl; ++l) {
        Layer& L = P->layers[l];
        void* xin = (l & 1) ? P->x2 : P->x0;
        void* xout = (l & 1) ? P->x0 : P->x2;
        if (tm) cudaEventRecord(E->events[1 + 2 * l], st);
        ENG_TRY(attn_block_prefill(L.attn, xin, R, pos, row_seq, c.max_batch, R - head, P->page_table, P->num_pages,
                                   L.k_cache, L.v_cache, P->x1, P->ws, P->ws_bytes, st));
        if (tm) cudaEventRecord(E->events[2 + 2 * l], st);
        const void* fin = static_cast<const uint8_t*>(P->x1) + lo * row_bytes;
        void* fout = static_cast<uint8_t*>(xout) + lo * row_bytes;
        if (L.dense)
            ENG_TRY(moe_layer_forward_routed(L.ffn, fin, P->dense_idx, P->dense_w, fout, hi - lo, P->ws, P->ws_bytes,
                                             st));
        else {
            ENG_TRY(moe_layer_set_gemm_form(L.ffn, form));
            ENG_TRY(moe_layer_forward(L.ffn, fin, fout, hi - lo, P->ws, P->ws_bytes, st));
        }
        for (int r = 0; r < P->world; ++r) G.x[r] = (l & 1) ? E->ranks[r]->x0 : E->ranks[r]->x2;
        ENG_CUDA(tb_engine::rows_allgather(G, xout, lo, hi - lo, c.hidden, P->gather_epoch, P->gather_done,
                                           20000000000ull, P->error_word, st));
        xfinal = xout;
    }
    if (P->rank != 0 || !sample) {
        if (!sync) return MOE_OK;
        return cudaStreamSynchronize(st) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
    }
    if (tm) cudaEventRecord(E->events[1 + 2 * nl], st);
    const void* head_x = static_cast<const uint8_t*>(xfinal) + static_cast<size_t>(R - head) * row_bytes;
    ENG_CUDA(tb_engine::final_norm_rows(head_x, P->final_norm, head, c.hidden, c.rms_eps, P->xn, st));
    const float one = 1.0f, zero = 0.0f;
    if (cublasGemmEx(P->cublas, CUBLAS_OP_T, CUBLAS_OP_N, c.vocab_size, head, c.hidden, &one, P->lm_head, CUDA_R_16BF,
                     c.hidden, P->xn, CUDA_R_16BF, c.hidden, &zero, P->logits, CUDA_R_32F, c.vocab_size,
                     CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS)
        return MOE_ERR_CUDA;
    ENG_CUDA(tb_engine::sample_rows(P->logits, head, c.vocab_size,
                                    reinterpret_cast<const float*>(P->stage_dev + P->stage.temp),
                                    reinterpret_cast<const float*>(P->stage_dev + P->stage.top_p),
                                    reinterpret_cast<const uint64_t*>(P->stage_dev + P->stage.seeds), P->tokens_out,
                                    st));
    if (tm) cudaEventRecord(E->events[2 + 2 * nl], st);
    ENG_CUDA(cudaMemcpyAsync(E->tokens_host, P->tokens_out, static_cast<size_t>(head) * 8, cudaMemcpyDeviceToHost, st));
    if (!sync) return MOE_OK;   // being captured into a graph
    ENG_CUDA(cudaStreamSynchronize(st));
    if (tm) {
        float ms = 0.0f, attn = 0.0f, ffn = 0.0f;
        cudaEventElapsedTime(&ms, E->events[0], E->events[1]);
        E->stage_ms[0] = ms;
        for (size_t l = 0; l < nl; ++l) {
            cudaEventElapsedTime(&ms, E->events[1 + 2 * l], E->events[2 + 2 * l]);
            attn += ms;
            cudaEventElapsedTime(&ms, E->events[2 + 2 * l], E->events[3 + 2 * l]);
            ffn += ms;
        }
        E->stage_ms[1] = attn;
        E->stage_ms[2] = ffn;
        cudaEventElapsedTime(&ms, E->events[1 + 2 * nl], E->events[2 + 2 * nl]);
        E->stage_ms[3] = ms;
    }
    return MOE_OK;
}

// Rank P's pure decode step of R rows from a CUDA graph of its part of the
// forward, as forward_graph on one GPU (every rank sees the same sequence of
// row counts, so all ranks replay, capture or run eagerly in the same step;
// the exchanges keep their epochs on the device, so a replay pairs up with
// the other ranks' eager or replayed kernels).
moe_status_t forward_rank_graph(glm_engine* P, int R) {
    ENG_CUDA(cudaSetDevice(P->device));
    auto it = P->graph_exec.find(R);
    if (it == P->graph_exec.end()) {
        if (++P->graph_seen[R] < 2 || !P->graphs_ok) return forward_rank(P, R, R);
        cudaStream_t st = P->stream;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            cudaGetLastError();
            P->graphs_ok = false;
            return forward_rank(P, R, R);
        }
        const moe_status_t s = forward_rank(P, R, R, false);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(st, &g);
        cudaGraphExec_t x = nullptr;
        if (s != MOE_OK || e != cudaSuccess || !g || cudaGraphInstantiate(&x, g, 0) != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            P->graphs_ok = false;
            return forward_rank(P, R, R);
        }
        cudaGraphDestroy(g);
        it = P->graph_exec.emplace(R, x).first;
    }
    ENG_CUDA(cudaGraphLaunch(it->second, P->stream));
    ENG_CUDA(cudaStreamSynchronize(P->stream));
    return MOE_OK;
}

// One forward: on one GPU, or every rank on its own host thread.
// A pure decode step of R rows on one GPU from a CUDA graph of the whole
// forward: the first time R occurs it runs eagerly (every lazy setup --
// shared-memory opt-ins, library handles -- happens outside the capture), the
// second time it is captured (stage copy from the pinned staging buffer
// included, so every replay reads the step's own rows), then replayed.  A
// capture that fails leaves the engine eager for good.
moe_status_t forward_graph(glm_engine* E, int R) {
    auto it = E->graph_exec.find(R);
    if (it == E->graph_exec.end()) {
        if (++E->graph_seen[R] < 2) return forward_one(E, R, R);
        cudaStream_t st = E->stream;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            cudaGetLastError();
            E->graphs_ok = false;
            return forward_one(E, R, R);
        }
        moe_status_t s = cudaMemcpyAsync(E->stage_dev, E->stage_host, E->stage.bytes, cudaMemcpyHostToDevice, st) ==
                                 cudaSuccess
                             ? MOE_OK
                             : MOE_ERR_CUDA;
        if (s == MOE_OK) s = forward_one(E, R, R, false);
        cudaGraph_t g = nullptr;
        const cudaError_t e = cudaStreamEndCapture(st, &g);
        cudaGraphExec_t x = nullptr;
        if (s != MOE_OK || e != cudaSuccess || !g || cudaGraphInstantiate(&x, g, 0) != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            E->graphs_ok = false;
            return forward_one(E, R, R);
        }
        cudaGraphDestroy(g);
        it = E->graph_exec.emplace(R, x).first;
    }
    ENG_CUDA(cudaGraphLaunch(it->second, E->stream));
    ENG_CUDA(cudaStreamSynchronize(E->stream));
    return MOE_OK;
}

moe_status_t forward(glm_engine* E, int R, int head) {
    if (E->world == 1) {
        if (head == R && head > 0 && E->graphs_ok && !E->timing && !E->cap_idx) return forward_graph(E, R);
        return forward_one(E, R, head);
    }
    const bool graph = head == R && head > 0 && E->graphs_ok && !E->timing;
    std::vector<std::thread> th;
    th.reserve(E->world - 1);
    for (int r = 1; r < E->world; ++r) {
        glm_engine* P = E->ranks[r];
        th.emplace_back([P, R, head, graph]() {
            P->thread_status = graph ? forward_rank_graph(P, R) : forward_rank(P, R, head);
        });
    }
    const moe_status_t s0 = graph ? forward_rank_graph(E, R) : forward_rank(E, R, head);
    for (std::thread& t : th) t.join();
    cudaSetDevice(E->device);
    if (s0 != MOE_OK) return s0;
    for (int r = 1; r < E->world; ++r)
        if (E->ranks[r]->thread_status != MOE_OK) return E->ranks[r]->thread_status;
    return MOE_OK;
}

moe_status_t upload_stage(glm_engine* E) {
    if (E->world > 1) return MOE_OK;   // every rank copies the stage itself (forward_rank)
    return cudaMemcpyAsync(E->stage_dev, E->stage_host, E->stage.bytes, cudaMemcpyHostToDevice, E->stream) ==
                   cudaSuccess
               ? MOE_OK
               : MOE_ERR_CUDA;
}

// Page-table entries [i0, i1) of a request's row, host mirror -> device.
moe_status_t upload_pages(glm_engine* E, const Request* r, int i0, int i1) {
    if (i1 <= i0) return MOE_OK;
    const size_t off = static_cast<size_t>(r->slot) * E->max_pages_per_seq + i0;
    for (int i = i0; i < i1; ++i) E->page_table_host[off + (i - i0)] = r->pages[i];
    if (E->world == 1)
        return cudaMemcpyAsync(E->page_table + off, E->page_table_host + off, static_cast<size_t>(i1 - i0) * 4,
                               cudaMemcpyHostToDevice, E->stream) == cudaSuccess
                   ? MOE_OK
                   : MOE_ERR_CUDA;
    // every rank holds the page table; the copies finish before the next forward reads it
    bool ok = true;
    for (glm_engine* P : E->ranks) {
        ok = ok && cudaSetDevice(P->device) == cudaSuccess &&
             cudaMemcpyAsync(P->page_table + off, E->page_table_host + off, static_cast<size_t>(i1 - i0) * 4,
                             cudaMemcpyHostToDevice, P->stream) == cudaSuccess;
    }
    cudaSetDevice(E->device);
    return ok ? MOE_OK : MOE_ERR_CUDA;
}

void release(glm_engine* E, Request* r) {
    for (int32_t p : r->pages) E->free_pages.push_back(p);
    r->pages.clear();
    if (r->slot >= 0) E->free_slots.push_back(r->slot);
    r->slot = -1;
}

uint64_t reference_seed(int64_t request_id, int64_t past_len) {
    uint64_t s = static_cast<uint64_t>(request_id * 31 + past_len * 17);
    return s * 6364136223846793005ull + 1442695040888963407ull;
}

// Admits a request: checks, a request slot, KV pages for its prompt and its
// page-table row.  Its prompt runs with the next decode step.
Request* prefill(glm_engine* E, int64_t id, const int64_t* ids, int L, float temperature, float top_p,
                 float rep_penalty, int max_tokens) {
    if (L <= 0 || L > E->cfg.max_seq || !ids) return nullptr;
    for (int i = 0; i < L; ++i)
        if (ids[i] < 0 || ids[i] >= E->cfg.vocab_size) return nullptr;
    if (ensure_ready(E) != MOE_OK) return nullptr;
    const int need = (L + kPage - 1) / kPage;
    if (E->free_slots.empty() || static_cast<int>(E->free_pages.size()) < need) return nullptr;
    Request* r = new (std::nothrow) Request();
    if (!r) return nullptr;
    r->id = id;
    r->tokens.assign(ids, ids + L);
    r->max_tokens = max_tokens;
    r->temperature = temperature;
    r->top_p = top_p;
    r->rep_penalty = rep_penalty;
    r->slot = E->free_slots.back();
    E->free_slots.pop_back();
    for (int i = 0; i < need; ++i) {
        r->pages.push_back(E->free_pages.back());
        E->free_pages.pop_back();
    }
    if (upload_pages(E, r, 0, need) != MOE_OK || cudaStreamSynchronize(E->stream) != cudaSuccess) {
        release(E, r);
        delete r;
        return nullptr;
    }
    E->requests.insert(r);
    return r;
}

// One batched decode step over `n` states.  Per state: out token, done flag.
int32_t batch_decode(glm_engine* E, void* const* states, int n, int64_t* out_tokens, int32_t* out_done) {
    std::vector<int> row_of(n, -1);
    std::vector<Request*> rows;
    for (int i = 0; i < n; ++i) {
        out_tokens[i] = 0;
        out_done[i] = 1;
        Request* r = static_cast<Request*>(states[i]);
        if (!r || !E->requests.count(r) || r->finished) continue;
        const int pos = static_cast<int>(r->tokens.size()) - 1;
        const int pidx = pos / kPage;
        if (pidx >= E->max_pages_per_seq) {
            r->finished = true;
            continue;
        }
        if (pidx >= static_cast<int>(r->pages.size())) {
            if (E->free_pages.empty()) {   // out of KV pages: the request ends here
                r->finished = true;
                continue;
            }
            r->pages.push_back(E->free_pages.back());
            E->free_pages.pop_back();
            if (upload_pages(E, r, pidx, pidx + 1) != MOE_OK) return -4;
        }
        if (std::find(rows.begin(), rows.end(), r) != rows.end()) continue;   // a state passed twice
        row_of[i] = static_cast<int>(rows.size());
        rows.push_back(r);
    }
    const int B = static_cast<int>(rows.size());
    E->last_rows = B;
    for (auto& v : E->cap_step_idx) v.clear();
    for (auto& v : E->cap_step_w) v.clear();
    if (B == 0) return 0;
    int64_t* tok = reinterpret_cast<int64_t*>(E->stage_host + E->stage.tokens);
    uint64_t* seeds = reinterpret_cast<uint64_t*>(E->stage_host + E->stage.seeds);
    int32_t* pos = reinterpret_cast<int32_t*>(E->stage_host + E->stage.pos);
    int32_t* rs = reinterpret_cast<int32_t*>(E->stage_host + E->stage.row_seq);
    float* temp = reinterpret_cast<float*>(E->stage_host + E->stage.temp);
    float* topp = reinterpret_cast<float*>(E->stage_host + E->stage.top_p);
    // Rows: every position whose K/V is not yet written (admitted prompts,
    // chunked), request by request, in forwards of at most rows_cap rows;
    // the last forward ends with each request's newest position, the rows
    // that are sampled.
    moe_status_t s = MOE_OK;
    int fill = 0;
    auto flush = [&](int head) {
        if (s == MOE_OK) s = upload_stage(E);
        if (s == MOE_OK) s = forward(E, fill, head);
        fill = 0;
    };
    for (Request* r : rows) {
        const int last = static_cast<int>(r->tokens.size()) - 1;
        for (int p = r->kv_len; p < last && s == MOE_OK; ++p) {
            tok[fill] = r->tokens[p];
            pos[fill] = p;
            rs[fill] = r->slot;
            if (++fill == E->rows_cap) flush(0);
        }
    }
    if (s == MOE_OK && fill + B > E->rows_cap) flush(0);
    for (int b = 0; b < B && s == MOE_OK; ++b) {
        const Request* r = rows[b];
        const int64_t past_len = static_cast<int64_t>(r->tokens.size());
        tok[fill + b] = r->tokens.back();
        pos[fill + b] = static_cast<int32_t>(past_len - 1);
        rs[fill + b] = r->slot;
        seeds[b] = reference_seed(r->id, past_len);
        temp[b] = r->temperature;
        topp[b] = r->top_p;
    }
    if (s == MOE_OK) {
        fill += B;
        flush(B);
    }
    if (s != MOE_OK) {
        for (Request* r : rows) r->finished = true;
        return -4;
    }
    for (int i = 0; i < n; ++i) {
        if (row_of[i] < 0) continue;
        Request* r = rows[row_of[i]];
        const int64_t t = E->tokens_host[row_of[i]];
        r->kv_len = static_cast<int>(r->tokens.size());
        r->tokens.push_back(t);
        r->generated += 1;
        if (r->generated >= r->max_tokens || static_cast<int>(r->tokens.size()) >= E->cfg.max_seq) r->finished = true;
        out_tokens[i] = t;
        out_done[i] = r->finished ? 1 : 0;
    }
    return 0;
}

// ---------------------------------------------------------------- init_engine

struct HostBuf {
    std::vector<uint8_t> b;
    template <typename T>
    T* as() { return reinterpret_cast<T*>(b.data()); }
};

uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);   // NaN stays NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
}

// A [rows][cols] table (BF16 / F16 / F32) into device bf16.
bool upload_bf16_table(glm_engine* E, const st_model_t* M, const char* name, int64_t rows, int64_t cols,
                       void** out) {
    st_tensor_t t;
    if (st_get(M, name, &t) != MOE_OK || t.ndim != 2 || t.shape[0] != rows || t.shape[1] != cols) return false;
    const size_t n = static_cast<size_t>(rows) * cols;
    void* d = nullptr;
    if (cudaMalloc(&d, n * 2) != cudaSuccess) return false;
    E->owned.push_back(d);
    *out = d;
    if (t.dtype == ST_BF16) return cudaMemcpy(d, t.data, n * 2, cudaMemcpyHostToDevice) == cudaSuccess;
    if (t.dtype != ST_F16 && t.dtype != ST_F32) return false;
    std::vector<uint16_t> h(n);
    for (size_t i = 0; i < n; ++i) {
        float v;
        if (t.dtype == ST_F32) {
            std::memcpy(&v, static_cast<const uint8_t*>(t.data) + 4 * i, 4);
        } else {
            uint16_t x;
            std::memcpy(&x, static_cast<const uint8_t*>(t.data) + 2 * i, 2);
            const uint32_t sign = (x >> 15) & 1u, ex = (x >> 10) & 0x1fu, man = x & 0x3ffu;
            if (ex == 0) v = std::ldexp(static_cast<float>(man), -24);
            else if (ex == 31) v = man ? NAN : INFINITY;
            else v = std::ldexp(static_cast<float>(man | 0x400u), static_cast<int>(ex) - 25);
            if (sign) v = -v;
        }
        h[i] = f32_to_bf16_rne(v);
    }
    return cudaMemcpy(d, h.data(), n * 2, cudaMemcpyHostToDevice) == cudaSuccess;
}

bool upload_owned(glm_engine* E, const void* host, size_t bytes, void** out) {
    void* d = nullptr;
    if (bytes == 0) {
        *out = nullptr;
        return true;
    }
    if (cudaMalloc(&d, bytes) != cudaSuccess) return false;
    E->owned.push_back(d);
    *out = d;
    return cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
}

int64_t jint(const tb_json::JVal& root, const char* key, int64_t dflt) {
    const tb_json::JVal* v = root.get(key);
    if (!v || v->kind != tb_json::JVal::kNum) return dflt;
    return static_cast<int64_t>(v->d);
}
double jnum(const tb_json::JVal& root, const char* key, double dflt) {
    const tb_json::JVal* v = root.get(key);
    return (v && v->kind == tb_json::JVal::kNum) ? v->d : dflt;
}
bool jbool(const tb_json::JVal& root, const char* key, bool dflt) {
    const tb_json::JVal* v = root.get(key);
    return (v && v->kind == tb_json::JVal::kBool) ? v->b : dflt;
}

// config.json -> engine config: the HF GLM-4.x keys, with the reference's
// keys and defaults where those are absent (engine.t:380-408).
bool read_config(const std::string& dir, int max_batch, int max_seq, glm_engine_config_t* c, bool* tied) {
    std::string text;
    {
        FILE* f = std::fopen((dir + "/config.json").c_str(), "rb");
        if (!f) return false;
        char buf[65536];
        size_t n;
        while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) text.append(buf, n);
        std::fclose(f);
    }
    tb_json::JVal root;
    tb_json::JsonParser parser(text.data(), text.size());
    if (!parser.parse(&root) || root.kind != tb_json::JVal::kObj) return false;
    std::memset(c, 0, sizeof(*c));
    c->hidden = static_cast<int>(jint(root, "hidden_size", 4096));
    c->num_layers = static_cast<int>(jint(root, "num_hidden_layers", 92));
    c->num_q_heads = static_cast<int>(jint(root, "num_attention_heads", 32));
    c->num_kv_heads = static_cast<int>(jint(root, "num_key_value_heads", c->num_q_heads));
    c->head_dim = static_cast<int>(jint(root, "head_dim", c->num_q_heads > 0 ? c->hidden / c->num_q_heads : 0));
    c->rotary_dim = static_cast<int>(std::lround(c->head_dim * jnum(root, "partial_rotary_factor", 1.0)));
    c->vocab_size = static_cast<int>(jint(root, "vocab_size", 151552));
    c->num_experts = static_cast<int>(jint(root, "n_routed_experts", jint(root, "num_local_experts", 160)));
    c->top_k = static_cast<int>(jint(root, "num_experts_per_tok", 8));
    c->dense_intermediate = static_cast<int>(jint(root, "intermediate_size", 13696));
    c->moe_intermediate = static_cast<int>(jint(root, "moe_intermediate_size", c->dense_intermediate));
    c->num_shared = static_cast<int>(jint(root, "n_shared_experts", 0));
    c->first_dense = static_cast<int>(jint(root, "first_k_dense_replace", 0));
    if (c->first_dense > c->num_layers) c->first_dense = c->num_layers;
    c->rope_theta = static_cast<float>(jnum(root, "rope_theta", 10000.0));
    c->rms_eps = static_cast<float>(jnum(root, "rms_norm_eps", 1e-5));
    c->max_batch = max_batch;
    c->max_seq = max_seq;
    *tied = jbool(root, "tie_word_embeddings", false);
    return true;
}

// One layer's attention (the rank's heads) and FFN (the rank's experts, or
// the whole dense FFN) from the checkpoint into the rank's device memory.
bool load_layer_rank(glm_engine* E, glm_engine* R, const st_model_t* M, int l, int rank) {
    const glm_engine_config_t& c = E->cfg;
    const std::string prefix = "model.layers." + std::to_string(l) + ".";
    if (cudaSetDevice(R->device) != cudaSuccess) return false;
    st_attn_spec_t as{c.hidden, c.num_q_heads, c.num_kv_heads, c.head_dim, E->world, rank};
    st_attn_sizes_t asz;
    if (st_attn_rank_sizes(&as, &asz) != MOE_OK) return false;
    HostBuf ag, aqkv, asqkv, ao, aso;
    ag.b.resize(asz.gamma);
    aqkv.b.resize(asz.w_qkv);
    asqkv.b.resize(asz.s_qkv);
    ao.b.resize(asz.w_o);
    aso.b.resize(asz.s_o);
    if (st_attn_rank_host(M, prefix.c_str(), &as, ag.as<float>(), aqkv.as<uint8_t>(), asqkv.as<float>(),
                          ao.as<uint8_t>(), aso.as<float>()) != MOE_OK) {
        std::fprintf(stderr, "init_engine: layer %d attention tensors missing or malformed\n", l);
        return false;
    }
    void *d0, *d1, *d2, *d3, *d4;
    if (!(upload_owned(R, ag.b.data(), asz.gamma, &d0) && upload_owned(R, aqkv.b.data(), asz.w_qkv, &d1) &&
          upload_owned(R, asqkv.b.data(), asz.s_qkv, &d2) && upload_owned(R, ao.b.data(), asz.w_o, &d3) &&
          upload_owned(R, aso.b.data(), asz.s_o, &d4))) {
        std::fprintf(stderr, "init_engine: layer %d attention upload failed (%s)\n", l,
                     cudaGetErrorString(cudaGetLastError()));
        return false;
    }
    attn_block_weights_t aw{};
    aw.gamma = static_cast<const float*>(d0);
    aw.w_qkv = d1;
    aw.s_qkv = static_cast<const float*>(d2);
    aw.w_o = d3;
    aw.s_o = static_cast<const float*>(d4);
    st_moe_sizes_t fs;
    HostBuf fg, frw, frb, fw13, fs13, fw2, fs2;
    int has_bias = 0;
    moe_status_t s;
    const bool dense = l < c.first_dense;
    st_moe_spec_t ms{c.hidden, c.num_experts, c.moe_intermediate, c.num_shared, E->world, rank, nullptr};
    s = dense ? st_dense_ffn_sizes(c.hidden, c.dense_intermediate, &fs) : st_moe_layer_sizes(&ms, &fs);
    if (s == MOE_OK) {
        fg.b.resize(fs.gamma);
        frw.b.resize(fs.router_w);
        frb.b.resize(fs.router_bias);
        fw13.b.resize(fs.w13);
        fs13.b.resize(fs.s13);
        fw2.b.resize(fs.w2);
        fs2.b.resize(fs.s2);
        if (dense)
            s = st_dense_ffn_host(M, prefix.c_str(), c.hidden, c.dense_intermediate, fg.as<float>(), fw13.as<uint8_t>(),
                                  fs13.as<float>(), fw2.as<uint8_t>(), fs2.as<float>());
        else
            s = st_moe_layer_host(M, prefix.c_str(), &ms, fg.as<float>(), frw.as<float>(), frb.as<float>(), &has_bias,
                                  fw13.as<uint8_t>(), fs13.as<float>(), fw2.as<uint8_t>(), fs2.as<float>());
    }
    if (s != MOE_OK) {
        std::fprintf(stderr, "init_engine: layer %d FFN tensors missing or malformed\n", l);
        return false;
    }
    void *e0, *e1 = nullptr, *e2 = nullptr, *e3, *e4, *e5, *e6;
    if (!(upload_owned(R, fg.b.data(), fs.gamma, &e0) && upload_owned(R, frw.b.data(), fs.router_w, &e1) &&
          (has_bias ? upload_owned(R, frb.b.data(), fs.router_bias, &e2) : true) &&
          upload_owned(R, fw13.b.data(), fs.w13, &e3) && upload_owned(R, fs13.b.data(), fs.s13, &e4) &&
          upload_owned(R, fw2.b.data(), fs.w2, &e5) && upload_owned(R, fs2.b.data(), fs.s2, &e6))) {
        std::fprintf(stderr, "init_engine: layer %d FFN upload failed (%s)\n", l,
                     cudaGetErrorString(cudaGetLastError()));
        return false;
    }
    moe_layer_weights_t fw{};
    fw.norm_gamma = static_cast<const float*>(e0);
    fw.router_w = static_cast<const float*>(e1);
    fw.router_bias = has_bias ? static_cast<const float*>(e2) : nullptr;
    fw.w13 = e3;
    fw.s13 = static_cast<const float*>(e4);
    fw.w2 = e5;
    fw.s2 = static_cast<const float*>(e6);
    if (set_layer(E, rank, l, &aw, &fw) != MOE_OK) {
        std::fprintf(stderr, "init_engine: layer %d rejected by the layer kernels\n", l);
        return false;
    }
    return true;
}

glm_engine* init_from_dir(const char* model_dir, int max_batch, int max_seq, int num_gpus) {
    if (!model_dir || max_batch <= 0 || max_seq <= 0) return nullptr;
    const std::string dir(model_dir);
    glm_engine_config_t c;
    bool tied = false;
    if (!read_config(dir, max_batch, max_seq, &c, &tied)) {
        std::fprintf(stderr, "init_engine: cannot read %s/config.json\n", model_dir);
        return nullptr;
    }
    if (!config_ok(c)) {
        std::fprintf(stderr, "init_engine: unsupported model shape in %s/config.json\n", model_dir);
        return nullptr;
    }
    c.num_gpus = num_gpus > 1 ? num_gpus : 1;
    st_model_t* M = nullptr;
    if (st_open(model_dir, &M) != MOE_OK) {
        std::fprintf(stderr, "init_engine: cannot open the safetensors checkpoint in %s\n", model_dir);
        return nullptr;
    }
    glm_engine* E = nullptr;
    if (create(&c, &E) != MOE_OK) {
        st_close(M);
        std::fprintf(stderr, "init_engine: device allocation failed (or %d GPUs with peer access not available)\n",
                     c.num_gpus);
        return nullptr;
    }
    E->num_gpus_requested = num_gpus;
    E->num_tensors = st_num_tensors(M);
    bool ok = true;
    const int64_t H = c.hidden, V = c.vocab_size;
    for (int rank = 0; ok && rank < E->world; ++rank) {
        glm_engine* R = E->world > 1 ? E->ranks[rank] : E;
        ok = cudaSetDevice(R->device) == cudaSuccess;
        void *embed = nullptr, *lm = nullptr, *fnorm = nullptr;
        ok = ok && upload_bf16_table(R, M, "model.embed_tokens.weight", V, H, &embed);
        if (ok && rank == 0) {
            st_tensor_t t;
            if (st_get(M, "lm_head.weight", &t) == MOE_OK) ok = upload_bf16_table(R, M, "lm_head.weight", V, H, &lm);
            else if (tied) lm = embed;
            else ok = false;
            std::vector<float> g(H);
            ok = ok && st_get(M, "model.norm.weight", &t) == MOE_OK && t.ndim == 1 && t.shape[0] == H;
            if (ok && t.dtype == ST_F32) std::memcpy(g.data(), t.data, H * 4);
            else if (ok && t.dtype == ST_BF16)
                for (int64_t i = 0; i < H; ++i) {
                    uint16_t x;
                    std::memcpy(&x, static_cast<const uint8_t*>(t.data) + 2 * i, 2);
                    const uint32_t u = static_cast<uint32_t>(x) << 16;
                    std::memcpy(&g[i], &u, 4);
                }
            else ok = false;
            ok = ok && upload_owned(R, g.data(), H * 4, &fnorm);
        }
        if (!ok) std::fprintf(stderr, "init_engine: embedding, lm_head or final norm missing or malformed\n");
        if (ok) {
            R->embed = embed;
            R->final_norm = static_cast<const float*>(fnorm);
            R->lm_head = lm;
        }
    }
    for (int l = 0; ok && l < c.num_layers; ++l)
        for (int rank = 0; ok && rank < E->world; ++rank)
            ok = load_layer_rank(E, E->world > 1 ? E->ranks[rank] : E, M, l, rank);
    st_close(M);
    cudaSetDevice(E->device);
    if (ok && ensure_ready(E) != MOE_OK) {
        std::fprintf(stderr, "init_engine: workspace allocation failed\n");
        ok = false;
    }
    if (!ok) {
        destroy(E);
        return nullptr;
    }
    return E;
}

}  // namespace

extern "C" {

glm_engine_t* init_engine(const char* model_dir, int32_t max_batch, int32_t max_seq, int32_t num_gpus) {
    return init_from_dir(model_dir, max_batch, max_seq, num_gpus);
}

void* prefill_opaque(glm_engine_t* E, int64_t request_id, const int64_t* token_ids, int32_t seq_len,
                     float temperature, float top_p, float rep_penalty, int32_t max_tokens) {
    if (!E) return nullptr;
    std::lock_guard<std::mutex> g(E->mu);
    cudaSetDevice(E->device);
    return prefill(E, request_id, token_ids, seq_len, temperature, top_p, rep_penalty, max_tokens);
}

int32_t decode_step_opaque(glm_engine_t* E, void* state, int64_t* next_token_out, int32_t* is_done_out) {
    if (!E) return -1;
    if (!state) return -2;
    std::lock_guard<std::mutex> g(E->mu);
    cudaSetDevice(E->device);
    Request* r = static_cast<Request*>(state);
    if (!E->requests.count(r)) return -2;
    if (ensure_ready(E) != MOE_OK) return -1;
    const bool was_finished = r->finished;
    int64_t tok = 0;
    int32_t done = 1;
    const int32_t s = batch_decode(E, &state, 1, &tok, &done);
    if (s < 0) return s;
    if (!was_finished && E->last_rows == 0) return -3;   // no KV page for the next position
    if (next_token_out) *next_token_out = tok;
    if (is_done_out) *is_done_out = done;
    return 0;
}

void free_request_opaque(glm_engine_t* E, void* state) {
    if (!E || !state) return;
    std::lock_guard<std::mutex> g(E->mu);
    Request* r = static_cast<Request*>(state);
    if (!E->requests.erase(r)) return;
    release(E, r);
    delete r;
}

void free_engine(glm_engine_t* E) {
    if (!E) return;
    cudaSetDevice(E->device);
    destroy(E);
}

int64_t get_engine_info(glm_engine_t* E, int32_t info_type) {
    if (!E) return -1;
    std::lock_guard<std::mutex> g(E->mu);
    const glm_engine_config_t& c = E->cfg;
    switch (info_type) {
        case 0: return c.hidden;
        case 1: return c.num_layers;
        case 2: return c.num_q_heads;
        case 3: return c.vocab_size;
        case 4: return c.num_experts;
        case 5: return c.top_k;
        case 6: return E->world;
        case 7: return c.max_batch;
        case 8: return c.max_seq;
        case 9: return E->num_pages - static_cast<int64_t>(E->free_pages.size());
        case 10: return E->num_pages;
        case 11: return static_cast<int64_t>(E->requests.size());
        case 12: return E->num_tensors;
        case 13: return 1;
        default: return -1;
    }
}

int32_t run_batch_decode_ext(glm_engine_t* E, void* const* states, int32_t num_states, int64_t* out_tokens,
                             int32_t* out_done) {
    if (!E) return -1;
    if (num_states <= 0) return 0;
    if (!states || !out_tokens || !out_done) return -1;
    std::lock_guard<std::mutex> g(E->mu);
    cudaSetDevice(E->device);
    if (ensure_ready(E) != MOE_OK) return -1;
    return batch_decode(E, states, num_states, out_tokens, out_done);
}

moe_status_t glm_engine_create(const glm_engine_config_t* cfg, glm_engine_t** out) { return create(cfg, out); }

moe_status_t glm_engine_set_embedding(glm_engine_t* E, const void* embed_bf16, const float* final_norm,
                                      const void* lm_head_bf16) {
    if (!E || !embed_bf16 || !final_norm || !lm_head_bf16) return MOE_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(embed_bf16) & 15) || (reinterpret_cast<uintptr_t>(lm_head_bf16) & 15))
        return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    E->embed = embed_bf16;
    E->final_norm = final_norm;
    E->lm_head = lm_head_bf16;
    return MOE_OK;
}

moe_status_t glm_engine_set_layer(glm_engine_t* E, int layer, const attn_block_weights_t* attn,
                                  const moe_layer_weights_t* ffn) {
    if (!E || E->world > 1) return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    cudaSetDevice(E->device);
    return set_layer(E, 0, layer, attn, ffn);
}

moe_status_t glm_engine_set_layer_rank(glm_engine_t* E, int rank, int layer, const attn_block_weights_t* attn,
                                       const moe_layer_weights_t* ffn) {
    if (!E) return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    return set_layer(E, rank, layer, attn, ffn);
}

moe_status_t glm_engine_set_embedding_rank(glm_engine_t* E, int rank, const void* embed_bf16, const float* final_norm,
                                           const void* lm_head_bf16) {
    if (!E || rank < 0 || rank >= E->world || !embed_bf16 || (reinterpret_cast<uintptr_t>(embed_bf16) & 15))
        return MOE_ERR_INVALID_ARGUMENT;
    if (rank == 0 && (!final_norm || !lm_head_bf16 || (reinterpret_cast<uintptr_t>(lm_head_bf16) & 15)))
        return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    glm_engine* P = E->world > 1 ? E->ranks[rank] : E;
    P->embed = embed_bf16;
    P->final_norm = final_norm;
    P->lm_head = lm_head_bf16;
    return MOE_OK;
}

moe_status_t glm_engine_copy_logits(glm_engine_t* E, float* host_out, int rows) {
    if (!E || !host_out || rows < 0) return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    if (rows > E->last_rows) return MOE_ERR_INVALID_ARGUMENT;
    cudaSetDevice(E->device);
    return cudaMemcpy(host_out, E->logits, static_cast<size_t>(rows) * E->cfg.vocab_size * 4,
                      cudaMemcpyDeviceToHost) == cudaSuccess
               ? MOE_OK
               : MOE_ERR_CUDA;
}

moe_status_t glm_engine_set_capture(glm_engine_t* E, int on) {
    if (!E) return MOE_ERR_INVALID_ARGUMENT;
    if (E->world > 1) return on ? MOE_ERR_UNSUPPORTED : MOE_OK;   // routing is spread over the ranks
    std::lock_guard<std::mutex> g(E->mu);
    cudaSetDevice(E->device);
    if (!on) {
        if (E->cap_idx) cudaFree(E->cap_idx);
        if (E->cap_w) cudaFree(E->cap_w);
        E->cap_idx = nullptr;
        E->cap_w = nullptr;
        return MOE_OK;
    }
    if (E->cap_idx || E->cfg.first_dense == E->cfg.num_layers) return MOE_OK;
    E->cap_step_idx.assign(E->cfg.num_layers, {});
    E->cap_step_w.assign(E->cfg.num_layers, {});
    const size_t n = static_cast<size_t>(E->cfg.num_layers) * E->rows_cap * E->cfg.top_k;
    if (dev_alloc(&E->cap_idx, n * 4) != cudaSuccess || dev_alloc(&E->cap_w, n * 4) != cudaSuccess) {
        if (E->cap_idx) cudaFree(E->cap_idx);
        E->cap_idx = nullptr;
        E->cap_w = nullptr;
        return MOE_ERR_CUDA;
    }
    return MOE_OK;
}

moe_status_t glm_engine_copy_routing(glm_engine_t* E, int layer, int rows, int32_t* idx_host, float* w_host) {
    if (!E || !idx_host || !w_host || layer < 0 || rows < 0) return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    if (!E->cap_idx || layer >= E->cfg.num_layers || E->layers[layer].dense) return MOE_ERR_INVALID_ARGUMENT;
    const size_t n = static_cast<size_t>(rows) * E->cfg.top_k;
    if (n > E->cap_step_idx[layer].size()) return MOE_ERR_INVALID_ARGUMENT;
    std::memcpy(idx_host, E->cap_step_idx[layer].data(), n * 4);
    std::memcpy(w_host, E->cap_step_w[layer].data(), n * 4);
    return MOE_OK;
}

int glm_engine_request_pages(glm_engine_t* E, const void* state, int32_t* out, int max_pages) {
    if (!E || !state) return -1;
    std::lock_guard<std::mutex> g(E->mu);
    Request* r = static_cast<Request*>(const_cast<void*>(state));
    if (!E->requests.count(r)) return -1;
    const int n = static_cast<int>(r->pages.size());
    for (int i = 0; i < n && i < max_pages && out; ++i) out[i] = r->pages[i];
    return n;
}

moe_status_t glm_engine_copy_kv(glm_engine_t* E, int layer, int page, int npages, void* k_host, void* v_host) {
    if (!E || layer < 0 || layer >= E->cfg.num_layers || page < 0 || npages < 0 || page + npages > E->num_pages ||
        !k_host || !v_host)
        return MOE_ERR_INVALID_ARGUMENT;
    if (E->world > 1) return MOE_ERR_UNSUPPORTED;   // each rank holds its own KV heads
    std::lock_guard<std::mutex> g(E->mu);
    cudaSetDevice(E->device);
    const size_t pb = static_cast<size_t>(kPage) * E->cfg.num_kv_heads * kHeadDim * 2;
    const Layer& L = E->layers[layer];
    return cudaMemcpy(k_host, static_cast<const uint8_t*>(L.k_cache) + page * pb, npages * pb,
                      cudaMemcpyDeviceToHost) == cudaSuccess &&
                   cudaMemcpy(v_host, static_cast<const uint8_t*>(L.v_cache) + page * pb, npages * pb,
                              cudaMemcpyDeviceToHost) == cudaSuccess
               ? MOE_OK
               : MOE_ERR_CUDA;
}

static moe_status_t check_error_one(glm_engine* E) {
    cudaSetDevice(E->device);
    moe_status_t worst = MOE_OK;
    for (Layer& L : E->layers) {
        if (L.attn) {
            const moe_status_t s = attn_block_check_error(L.attn, E->stream);
            if (s != MOE_OK && worst == MOE_OK) worst = s;
        }
        if (L.ffn) {
            const moe_status_t s = moe_layer_check_error(L.ffn, E->stream);
            if (s != MOE_OK && worst == MOE_OK) worst = s;
        }
    }
    int h = 0;
    if (cudaMemcpy(&h, E->error_word, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return MOE_ERR_CUDA;
    if (h) {
        cudaMemset(E->error_word, 0, 4);
        // 3: a rows all-gather wait gave up (another rank stopped); else a token id outside the vocabulary
        if (worst == MOE_OK) worst = h == 3 ? MOE_ERR_DEVICE_TIMEOUT : MOE_ERR_INVALID_ARGUMENT;
    }
    return worst;
}

moe_status_t glm_engine_check_error(glm_engine_t* E) {
    if (!E) return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    moe_status_t worst = check_error_one(E);
    for (int r = 1; r < E->world; ++r) {
        const moe_status_t s = check_error_one(E->ranks[r]);
        if (s != MOE_OK && worst == MOE_OK) worst = s;
    }
    cudaSetDevice(E->device);
    return worst;
}

moe_status_t glm_engine_set_timing(glm_engine_t* E, int on) {
    if (!E) return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    set_events(E, on != 0);
    return (on != 0) == E->timing ? MOE_OK : MOE_ERR_CUDA;
}

moe_status_t glm_engine_stage_ms(glm_engine_t* E, float* out4) {
    if (!E || !out4) return MOE_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> g(E->mu);
    for (int i = 0; i < 4; ++i) out4[i] = E->stage_ms[i];
    return MOE_OK;
}

size_t glm_engine_device_bytes(const glm_engine_config_t* cfg) {
    if (!cfg || !config_ok(*cfg)) return 0;
    glm_engine_config_t c = *cfg;
    if (c.prefill_chunk <= 0) c.prefill_chunk = 2048;
    const Plan p = make_plan(c);
    return p.kv_bytes + 2 * p.act_bytes + static_cast<size_t>(c.max_batch) * c.hidden * 2 + p.logits_bytes +
           p.small_bytes;
}

}  // extern "C"
