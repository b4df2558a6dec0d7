// st_loader.cpp -- safetensors checkpoints into this library's weight layouts
// (declared in include/st_loader.h).  Host code only.
//
// A safetensors file is an 8-byte little-endian header length, a JSON object
// {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}
// and the tensor bytes, offsets relative to the end of the header.  A sharded
// checkpoint adds model.safetensors.index.json whose "weight_map" names the
// shard of each tensor (the reference reads the same files in
// src/terra/engine.t:412-720 with string scanning; this reads them with a
// small validating JSON parser and checks every range against the file).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <utility>
#include <vector>

#include "json_lite.h"
#include "st_loader.h"

namespace {

using tb_json::JVal;
using tb_json::JsonParser;

// ---------------------------------------------------------------- files

struct Mapped {
    const uint8_t* base = nullptr;
    size_t size = 0;
    bool map(const std::string& path) {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) return false;
        struct stat st;
        if (::fstat(fd, &st) != 0 || st.st_size <= 0) {
            ::close(fd);
            return false;
        }
        void* p = ::mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (p == MAP_FAILED) return false;
        base = static_cast<const uint8_t*>(p);
        size = static_cast<size_t>(st.st_size);
        return true;
    }
    void unmap() {
        if (base) ::munmap(const_cast<uint8_t*>(base), size);
        base = nullptr;
        size = 0;
    }
};

bool read_file(const std::string& path, std::string* out) {
    Mapped m;
    if (!m.map(path)) return false;
    out->assign(reinterpret_cast<const char*>(m.base), m.size);
    m.unmap();
    return true;
}

bool is_dir(const std::string& p) {
    struct stat st;
    return ::stat(p.c_str(), &st) == 0 && S_ISDIR(st.st_mode);
}
bool is_file(const std::string& p) {
    struct stat st;
    return ::stat(p.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

int dtype_code(const std::string& s, size_t* elem) {
    struct D { const char* n; int c; size_t sz; };
    static const D table[] = {{"F8_E4M3", ST_F8_E4M3, 1}, {"F16", ST_F16, 2}, {"BF16", ST_BF16, 2},
                              {"F32", ST_F32, 4}, {"I8", ST_I8, 1}, {"I16", ST_I16, 2}, {"I32", ST_I32, 4},
                              {"I64", ST_I64, 8}, {"U8", ST_U8, 1}, {"BOOL", ST_BOOL, 1}, {"F64", ST_F64, 8},
                              {"F8_E5M2", ST_F8_E5M2, 1}};
    for (const D& d : table)
        if (s == d.n) { *elem = d.sz; return d.c; }
    *elem = 0;
    return ST_UNKNOWN;
}

}  // namespace

struct st_model {
    std::vector<Mapped> shards;
    std::vector<std::string> names;
    std::unordered_map<std::string, st_tensor_t> tensors;
    ~st_model() {
        for (Mapped& m : shards) m.unmap();
    }
};

namespace {

// Maps one shard and records its tensors; false on any malformed part.
moe_status_t add_shard(st_model* M, const std::string& path) {
    Mapped m;
    if (!m.map(path)) return MOE_ERR_UNSUPPORTED;
    M->shards.push_back(m);
    if (m.size < 8) return MOE_ERR_INVALID_ARGUMENT;
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | m.base[i];
    if (hlen > 100ull * 1024 * 1024 || hlen > m.size - 8) return MOE_ERR_INVALID_ARGUMENT;
    JVal root;
    JsonParser jp(reinterpret_cast<const char*>(m.base + 8), static_cast<size_t>(hlen));
    if (!jp.parse(&root) || root.kind != JVal::kObj) return MOE_ERR_INVALID_ARGUMENT;
    const uint8_t* data = m.base + 8 + hlen;
    const uint64_t data_size = m.size - 8 - hlen;
    for (const auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const JVal& t = kv.second;
        if (t.kind != JVal::kObj) return MOE_ERR_INVALID_ARGUMENT;
        const JVal* dt = t.get("dtype");
        const JVal* sh = t.get("shape");
        const JVal* of = t.get("data_offsets");
        if (!dt || dt->kind != JVal::kStr || !sh || sh->kind != JVal::kArr || !of || of->kind != JVal::kArr ||
            of->arr.size() != 2 || sh->arr.size() > 8)
            return MOE_ERR_INVALID_ARGUMENT;
        st_tensor_t x;
        std::memset(&x, 0, sizeof(x));
        size_t elem = 0;
        x.dtype = dtype_code(dt->s, &elem);
        if (x.dtype == ST_UNKNOWN) return MOE_ERR_INVALID_ARGUMENT;
        x.ndim = static_cast<int>(sh->arr.size());
        uint64_t count = 1;
        for (int i = 0; i < x.ndim; ++i) {
            const JVal& d = sh->arr[i];
            if (d.kind != JVal::kNum || !d.is_uint || d.u > (1ull << 40)) return MOE_ERR_INVALID_ARGUMENT;
            x.shape[i] = static_cast<int64_t>(d.u);
            if (d.u != 0 && count > UINT64_MAX / d.u) return MOE_ERR_INVALID_ARGUMENT;
            count *= d.u;
        }
        const JVal& b0 = of->arr[0];
        const JVal& b1 = of->arr[1];
        if (b0.kind != JVal::kNum || b1.kind != JVal::kNum || !b0.is_uint || !b1.is_uint || b1.u < b0.u ||
            b1.u > data_size)
            return MOE_ERR_INVALID_ARGUMENT;
        if (count > UINT64_MAX / elem || count * elem != b1.u - b0.u) return MOE_ERR_INVALID_ARGUMENT;
        x.data = data + b0.u;
        x.nbytes = b1.u - b0.u;
        if (!M->tensors.emplace(kv.first, x).second) return MOE_ERR_INVALID_ARGUMENT;   // duplicate name
        M->names.push_back(kv.first);
    }
    return MOE_OK;
}

moe_status_t open_model(st_model* M, const std::string& path) {
    if (is_file(path)) return add_shard(M, path);
    if (!is_dir(path)) return MOE_ERR_UNSUPPORTED;
    const std::string index = path + "/model.safetensors.index.json";
    if (!is_file(index)) {
        const std::string single = path + "/model.safetensors";
        return is_file(single) ? add_shard(M, single) : MOE_ERR_UNSUPPORTED;
    }
    std::string text;
    if (!read_file(index, &text)) return MOE_ERR_UNSUPPORTED;
    JVal root;
    JsonParser jp(text.data(), text.size());
    if (!jp.parse(&root) || root.kind != JVal::kObj) return MOE_ERR_INVALID_ARGUMENT;
    const JVal* wm = root.get("weight_map");
    if (!wm || wm->kind != JVal::kObj) return MOE_ERR_INVALID_ARGUMENT;
    std::vector<std::string> files;
    std::unordered_set<std::string> seen;
    for (const auto& kv : wm->obj) {
        if (kv.second.kind != JVal::kStr) return MOE_ERR_INVALID_ARGUMENT;
        const std::string& f = kv.second.s;
        // shard names stay inside the checkpoint directory
        if (f.empty() || f.find('/') != std::string::npos || f == "." || f == "..") return MOE_ERR_INVALID_ARGUMENT;
        if (seen.insert(f).second) files.push_back(f);
    }
    for (const std::string& f : files) {
        const moe_status_t s = add_shard(M, path + "/" + f);
        if (s != MOE_OK) return s;
    }
    for (const auto& kv : wm->obj)
        if (!M->tensors.count(kv.first)) return MOE_ERR_INVALID_ARGUMENT;   // the map names a tensor no shard holds
    return MOE_OK;
}

// ---------------------------------------------------------------- conversions

float bf16_to_f32(uint16_t h) {
    const uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h >> 15) << 31;
    const int ex = (h >> 10) & 0x1F;
    const uint32_t man = h & 0x3FF;
    float f;
    if (ex == 0) {
        f = std::ldexp(static_cast<float>(man), -24);    // zero or subnormal
        if (sign) f = -f;
        return f;
    }
    uint32_t u;
    if (ex == 0x1F) u = sign | 0x7F800000u | (man << 13);   // inf / nan
    else u = sign | (static_cast<uint32_t>(ex + 112) << 23) | (man << 13);
    std::memcpy(&f, &u, 4);
    return f;
}

const st_tensor_t* find(const st_model* M, const std::string& name) {
    auto it = M->tensors.find(name);
    return it == M->tensors.end() ? nullptr : &it->second;
}

bool shape_is(const st_tensor_t* t, std::initializer_list<int64_t> dims) {
    if (t->ndim != static_cast<int>(dims.size())) return false;
    int i = 0;
    for (int64_t d : dims)
        if (t->shape[i++] != d) return false;
    return true;
}

// n floats from an F32 / BF16 / F16 tensor of exactly n elements
moe_status_t to_f32(const st_tensor_t* t, size_t n, float* out) {
    size_t count = 1;
    for (int i = 0; i < t->ndim; ++i) count *= static_cast<size_t>(t->shape[i]);
    if (count != n) return MOE_ERR_INVALID_ARGUMENT;
    if (t->dtype == ST_F32) {
        std::memcpy(out, t->data, n * 4);
    } else if (t->dtype == ST_BF16 || t->dtype == ST_F16) {
        const uint8_t* b = static_cast<const uint8_t*>(t->data);
        for (size_t i = 0; i < n; ++i) {
            uint16_t h;
            std::memcpy(&h, b + 2 * i, 2);
            out[i] = t->dtype == ST_BF16 ? bf16_to_f32(h) : f16_to_f32(h);
        }
    } else {
        return MOE_ERR_INVALID_ARGUMENT;
    }
    return MOE_OK;
}

// An FP8 projection [rows][cols] with its [rows/128][cols/128] fp32 scales.
moe_status_t fp8_pair(const st_model* M, const std::string& w_name, int64_t rows, int64_t cols, const st_tensor_t** w,
                      const st_tensor_t** s) {
    *w = find(M, w_name);
    *s = find(M, w_name + "_scale_inv");
    if (!*w || !*s) return MOE_ERR_INVALID_ARGUMENT;
    if ((*w)->dtype != ST_F8_E4M3 || !shape_is(*w, {rows, cols})) return MOE_ERR_INVALID_ARGUMENT;
    if ((*s)->dtype != ST_F32 || !shape_is(*s, {rows / 128, cols / 128})) return MOE_ERR_INVALID_ARGUMENT;
    return MOE_OK;
}

// The routed experts a rank holds, in its local-slot order.
bool local_experts(const st_moe_spec_t& sp, std::vector<int>* out) {
    const int epr = sp.num_experts / sp.ep_size;
    out->clear();
    if (!sp.slot_of_expert) {
        for (int j = 0; j < epr; ++j) out->push_back(sp.ep_rank * epr + j);
        return true;
    }
    std::vector<int> expert_of_slot(sp.num_experts, -1);
    for (int e = 0; e < sp.num_experts; ++e) {
        const int s = sp.slot_of_expert[e];
        if (s < 0 || s >= sp.num_experts || expert_of_slot[s] >= 0) return false;   // not a permutation
        expert_of_slot[s] = e;
    }
    for (int j = 0; j < epr; ++j) out->push_back(expert_of_slot[sp.ep_rank * epr + j]);
    return true;
}

bool moe_spec_ok(const st_moe_spec_t* sp) {
    return sp && sp->hidden > 0 && sp->hidden % 128 == 0 && sp->intermediate > 0 && sp->intermediate % 128 == 0 &&
           sp->num_experts > 0 && sp->ep_size > 0 && sp->num_experts % sp->ep_size == 0 && sp->ep_rank >= 0 &&
           sp->ep_rank < sp->ep_size && (sp->num_shared == 0 || sp->num_shared == 1);
}

bool attn_spec_ok(const st_attn_spec_t* sp) {
    return sp && sp->hidden > 0 && sp->hidden % 128 == 0 && sp->head_dim == 128 && sp->num_q_heads > 0 &&
           sp->num_kv_heads > 0 && sp->tp_size > 0 && sp->num_q_heads % sp->tp_size == 0 &&
           sp->num_kv_heads % sp->tp_size == 0 && sp->tp_rank >= 0 && sp->tp_rank < sp->tp_size;
}

}  // namespace

extern "C" {

moe_status_t st_open(const char* path, st_model_t** out) {
    if (!path || !out) return MOE_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    st_model* M = new (std::nothrow) st_model();
    if (!M) return MOE_ERR_UNSUPPORTED;
    const moe_status_t s = open_model(M, path);
    if (s != MOE_OK) {
        delete M;
        return s;
    }
    *out = M;
    return MOE_OK;
}

void st_close(st_model_t* M) { delete M; }

int st_num_tensors(const st_model_t* M) { return M ? static_cast<int>(M->names.size()) : 0; }

const char* st_tensor_name(const st_model_t* M, int i) {
    if (!M || i < 0 || i >= static_cast<int>(M->names.size())) return nullptr;
    return M->names[i].c_str();
}

moe_status_t st_get(const st_model_t* M, const char* name, st_tensor_t* out) {
    if (!M || !name || !out) return MOE_ERR_INVALID_ARGUMENT;
    const st_tensor_t* t = find(M, name);
    if (!t) return MOE_ERR_INVALID_ARGUMENT;
    *out = *t;
    return MOE_OK;
}

moe_status_t st_moe_layer_sizes(const st_moe_spec_t* sp, st_moe_sizes_t* out) {
    if (!moe_spec_ok(sp) || !out) return MOE_ERR_INVALID_ARGUMENT;
    const size_t H = sp->hidden, I = sp->intermediate, E = sp->num_experts;
    const size_t G = E / sp->ep_size + sp->num_shared;
    out->gamma = H * 4;
    out->router_w = E * H * 4;
    out->router_bias = E * 4;
    out->w13 = G * 2 * I * H;
    out->s13 = G * (2 * I / 128) * (H / 128) * 4;
    out->w2 = G * H * I;
    out->s2 = G * (H / 128) * (I / 128) * 4;
    return MOE_OK;
}

moe_status_t st_moe_layer_host(const st_model_t* M, const char* prefix, const st_moe_spec_t* sp, float* gamma,
                               float* router_w, float* router_bias, int* has_bias, uint8_t* w13, float* s13,
                               uint8_t* w2, float* s2) {
    if (!M || !prefix || !moe_spec_ok(sp) || !gamma || !router_w || !has_bias || !w13 || !s13 || !w2 || !s2)
        return MOE_ERR_INVALID_ARGUMENT;
    const std::string P(prefix);
    const int64_t H = sp->hidden, I = sp->intermediate, E = sp->num_experts;
    std::vector<int> experts;
    if (!local_experts(*sp, &experts)) return MOE_ERR_INVALID_ARGUMENT;
    const st_tensor_t* t = find(M, P + "post_attention_layernorm.weight");
    if (!t) return MOE_ERR_INVALID_ARGUMENT;
    moe_status_t s = to_f32(t, static_cast<size_t>(H), gamma);
    if (s != MOE_OK) return s;
    t = find(M, P + "mlp.gate.weight");
    if (!t || !shape_is(t, {E, H})) return MOE_ERR_INVALID_ARGUMENT;
    if ((s = to_f32(t, static_cast<size_t>(E * H), router_w)) != MOE_OK) return s;
    t = find(M, P + "mlp.gate.e_score_correction_bias");
    *has_bias = 0;
    if (t) {
        if (!router_bias) return MOE_ERR_INVALID_ARGUMENT;
        if ((s = to_f32(t, static_cast<size_t>(E), router_bias)) != MOE_OK) return s;
        *has_bias = 1;
    }
    const size_t wg = static_cast<size_t>(2 * I * H), sg = static_cast<size_t>((2 * I / 128) * (H / 128));
    const size_t w2g = static_cast<size_t>(H * I), s2g = static_cast<size_t>((H / 128) * (I / 128));
    const int groups = static_cast<int>(experts.size()) + sp->num_shared;
    for (int j = 0; j < groups; ++j) {
        const std::string base = j < static_cast<int>(experts.size())
                                     ? P + "mlp.experts." + std::to_string(experts[j]) + "."
                                     : P + "mlp.shared_experts.";
        const st_tensor_t *gw, *gs, *uw, *us, *dw, *ds;
        if ((s = fp8_pair(M, base + "gate_proj.weight", I, H, &gw, &gs)) != MOE_OK) return s;
        if ((s = fp8_pair(M, base + "up_proj.weight", I, H, &uw, &us)) != MOE_OK) return s;
        if ((s = fp8_pair(M, base + "down_proj.weight", H, I, &dw, &ds)) != MOE_OK) return s;
        // gate rows then up rows
        std::memcpy(w13 + j * wg, gw->data, gw->nbytes);
        std::memcpy(w13 + j * wg + gw->nbytes, uw->data, uw->nbytes);
        std::memcpy(s13 + j * sg, gs->data, gs->nbytes);
        std::memcpy(reinterpret_cast<uint8_t*>(s13 + j * sg) + gs->nbytes, us->data, us->nbytes);
        std::memcpy(w2 + j * w2g, dw->data, dw->nbytes);
        std::memcpy(s2 + j * s2g, ds->data, ds->nbytes);
    }
    return MOE_OK;
}

moe_status_t st_dense_ffn_sizes(int hidden, int intermediate, st_moe_sizes_t* out) {
    if (hidden <= 0 || hidden % 128 || intermediate <= 0 || intermediate % 128 || !out) return MOE_ERR_INVALID_ARGUMENT;
    const size_t H = hidden, I = intermediate;
    out->gamma = H * 4;
    out->router_w = 0;
    out->router_bias = 0;
    out->w13 = 2 * I * H;
    out->s13 = (2 * I / 128) * (H / 128) * 4;
    out->w2 = H * I;
    out->s2 = (H / 128) * (I / 128) * 4;
    return MOE_OK;
}

moe_status_t st_dense_ffn_host(const st_model_t* M, const char* prefix, int hidden, int intermediate, float* gamma,
                               uint8_t* w13, float* s13, uint8_t* w2, float* s2) {
    if (!M || !prefix || hidden <= 0 || hidden % 128 || intermediate <= 0 || intermediate % 128 || !gamma || !w13 ||
        !s13 || !w2 || !s2)
        return MOE_ERR_INVALID_ARGUMENT;
    const std::string P(prefix);
    const int64_t H = hidden, I = intermediate;
    const st_tensor_t* t = find(M, P + "post_attention_layernorm.weight");
    if (!t) return MOE_ERR_INVALID_ARGUMENT;
    moe_status_t s = to_f32(t, static_cast<size_t>(H), gamma);
    if (s != MOE_OK) return s;
    const st_tensor_t *gw, *gs, *uw, *us, *dw, *ds;
    if ((s = fp8_pair(M, P + "mlp.gate_proj.weight", I, H, &gw, &gs)) != MOE_OK) return s;
    if ((s = fp8_pair(M, P + "mlp.up_proj.weight", I, H, &uw, &us)) != MOE_OK) return s;
    if ((s = fp8_pair(M, P + "mlp.down_proj.weight", H, I, &dw, &ds)) != MOE_OK) return s;
    std::memcpy(w13, gw->data, gw->nbytes);
    std::memcpy(w13 + gw->nbytes, uw->data, uw->nbytes);
    std::memcpy(s13, gs->data, gs->nbytes);
    std::memcpy(reinterpret_cast<uint8_t*>(s13) + gs->nbytes, us->data, us->nbytes);
    std::memcpy(w2, dw->data, dw->nbytes);
    std::memcpy(s2, ds->data, ds->nbytes);
    return MOE_OK;
}

moe_status_t st_attn_rank_sizes(const st_attn_spec_t* sp, st_attn_sizes_t* out) {
    if (!attn_spec_ok(sp) || !out) return MOE_ERR_INVALID_ARGUMENT;
    const size_t H = sp->hidden, d = sp->head_dim;
    const size_t nq = sp->num_q_heads / sp->tp_size, nkv = sp->num_kv_heads / sp->tp_size;
    out->gamma = H * 4;
    out->w_qkv = (nq + 2 * nkv) * d * H;
    out->s_qkv = (nq + 2 * nkv) * (d / 128) * (H / 128) * 4;
    out->w_o = H * nq * d;
    out->s_o = (H / 128) * (nq * d / 128) * 4;
    return MOE_OK;
}

moe_status_t st_attn_rank_host(const st_model_t* M, const char* prefix, const st_attn_spec_t* sp, float* gamma,
                               uint8_t* w_qkv, float* s_qkv, uint8_t* w_o, float* s_o) {
    if (!M || !prefix || !attn_spec_ok(sp) || !gamma || !w_qkv || !s_qkv || !w_o || !s_o) return MOE_ERR_INVALID_ARGUMENT;
    const std::string P(prefix);
    const int64_t H = sp->hidden, d = sp->head_dim;
    const int64_t NQ = sp->num_q_heads, NKV = sp->num_kv_heads;
    const int64_t nq = NQ / sp->tp_size, nkv = NKV / sp->tp_size, r = sp->tp_rank;
    const st_tensor_t* t = find(M, P + "input_layernorm.weight");
    if (!t) return MOE_ERR_INVALID_ARGUMENT;
    moe_status_t s = to_f32(t, static_cast<size_t>(H), gamma);
    if (s != MOE_OK) return s;
    const st_tensor_t *qw, *qs, *kw, *ks, *vw, *vs, *ow, *os;
    if ((s = fp8_pair(M, P + "self_attn.q_proj.weight", NQ * d, H, &qw, &qs)) != MOE_OK) return s;
    if ((s = fp8_pair(M, P + "self_attn.k_proj.weight", NKV * d, H, &kw, &ks)) != MOE_OK) return s;
    if ((s = fp8_pair(M, P + "self_attn.v_proj.weight", NKV * d, H, &vw, &vs)) != MOE_OK) return s;
    if ((s = fp8_pair(M, P + "self_attn.o_proj.weight", H, NQ * d, &ow, &os)) != MOE_OK) return s;
    const size_t row = static_cast<size_t>(H), srow = static_cast<size_t>(H / 128) * 4;
    // stacked rows: this rank's q heads, k heads, v heads (d / 128 scale rows per head)
    uint8_t* wp = w_qkv;
    uint8_t* sp8 = reinterpret_cast<uint8_t*>(s_qkv);
    auto take_rows = [&](const st_tensor_t* w, const st_tensor_t* sc, int64_t first, int64_t rows) {
        std::memcpy(wp, static_cast<const uint8_t*>(w->data) + first * row, rows * row);
        wp += rows * row;
        std::memcpy(sp8, static_cast<const uint8_t*>(sc->data) + (first / 128) * srow, (rows / 128) * srow);
        sp8 += (rows / 128) * srow;
    };
    take_rows(qw, qs, r * nq * d, nq * d);
    take_rows(kw, ks, r * nkv * d, nkv * d);
    take_rows(vw, vs, r * nkv * d, nkv * d);
    // o_proj: the matching input columns of every row
    const int64_t cols = nq * d, c0 = r * nq * d, full = NQ * d;
    for (int64_t i = 0; i < H; ++i)
        std::memcpy(w_o + i * cols, static_cast<const uint8_t*>(ow->data) + i * full + c0, static_cast<size_t>(cols));
    const int64_t scols = cols / 128, sc0 = c0 / 128, sfull = full / 128;
    for (int64_t i = 0; i < H / 128; ++i)
        std::memcpy(s_o + i * scols, static_cast<const float*>(os->data) + i * sfull + sc0, static_cast<size_t>(scols) * 4);
    return MOE_OK;
}

}  // extern "C"
