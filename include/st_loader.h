/* st_loader.h -- safetensors checkpoints (the engine's FP8 GLM-4.x format)
 * into this library's weight layouts (libkernels.so, host code only).
 *
 * Replaces the reference's loader (src/terra/engine.t:412-720: the
 * model.safetensors.index.json weight map, mmapped shards, per-shard JSON
 * headers, get_tensor_data_ptr) and fills what its load_weights_to_gpu
 * (engine.t:872-926) leaves empty: the per-layer MoE and attention weights,
 * assembled from the FP8 tensors and their 128x128 `weight_scale_inv` blocks
 * into the layouts of moe_layer_weights_t (include/moe_layer.h) and
 * attn_block_weights_t (include/attn_block.h).  The assembled buffers are
 * host memory of the caller's; uploading them is one copy each.
 *
 * dtype codes 1-7 are the reference's TensorDescriptor codes (engine.t:583-599).
 */
#ifndef TIME_B200_ST_LOADER_H
#define TIME_B200_ST_LOADER_H

#include <stddef.h>
#include <stdint.h>

#include "moe_layer.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ST_UNKNOWN = 0, ST_F8_E4M3 = 1, ST_F16 = 2, ST_BF16 = 3, ST_F32 = 4, ST_I8 = 5, ST_I16 = 6, ST_I32 = 7,
    ST_I64 = 8, ST_U8 = 9, ST_BOOL = 10, ST_F64 = 11, ST_F8_E5M2 = 12
};

typedef struct st_model st_model_t;

typedef struct {
    int dtype;            /* ST_* */
    int ndim;
    int64_t shape[8];
    const void* data;     /* read-only, valid until st_close */
    uint64_t nbytes;
} st_tensor_t;

/* `path`: a directory holding model.safetensors.index.json (+ its shards) or
 * model.safetensors, or one .safetensors file.  Every shard is mapped
 * read-only and its header checked: dtype known, shape product x dtype size
 * == the byte range, ranges inside the file, names unique.  A malformed file
 * gives MOE_ERR_INVALID_ARGUMENT, an unreadable one MOE_ERR_UNSUPPORTED. */
moe_status_t st_open(const char* path, st_model_t** out);
void st_close(st_model_t* model);
int st_num_tensors(const st_model_t* model);
const char* st_tensor_name(const st_model_t* model, int i);
/* MOE_ERR_INVALID_ARGUMENT when the tensor is absent. */
moe_status_t st_get(const st_model_t* model, const char* name, st_tensor_t* out);

/* One MoE layer, tensors under `prefix` (e.g. "model.layers.3."):
 *   post_attention_layernorm.weight           [H]      bf16/f16/f32
 *   mlp.gate.weight                           [E][H]   bf16/f16/f32 (router)
 *   mlp.gate.e_score_correction_bias          [E]      optional
 *   mlp.experts.{e}.{gate,up,down}_proj.weight          F8_E4M3
 *   mlp.experts.{e}.{gate,up,down}_proj.weight_scale_inv F32 [rows/128][cols/128]
 *   mlp.shared_experts.{gate,up,down}_proj.*           (num_shared == 1)
 * assembled for expert-parallel rank ep_rank of ep_size: its experts (global
 * order, or local-slot order of slot_of_expert when given, as
 * moe_layer_set_expert_placement) then the shared expert; gate rows then up
 * rows in w13. */
typedef struct {
    int hidden, num_experts, intermediate, num_shared, ep_size, ep_rank;
    const int32_t* slot_of_expert;   /* host [E] or NULL */
} st_moe_spec_t;

typedef struct {
    size_t gamma, router_w, router_bias, w13, s13, w2, s2;   /* bytes */
} st_moe_sizes_t;

moe_status_t st_moe_layer_sizes(const st_moe_spec_t* spec, st_moe_sizes_t* out);
/* Host buffers sized by st_moe_layer_sizes; *has_bias = 0 when the checkpoint
 * has no router bias (router_bias left untouched). */
moe_status_t st_moe_layer_host(const st_model_t* model, const char* prefix, const st_moe_spec_t* spec, float* gamma,
                               float* router_w, float* router_bias, int* has_bias, uint8_t* w13, float* s13,
                               uint8_t* w2, float* s2);

/* A dense FFN layer (GLM's first layers), tensors under `prefix`:
 *   post_attention_layernorm.weight, mlp.{gate,up,down}_proj.weight (+ _scale_inv)
 * in the layout of a one-expert moe_layer_weights_t: w13 = gate rows then up
 * rows [2I][H], w2 [H][I] (router sizes 0). */
moe_status_t st_dense_ffn_sizes(int hidden, int intermediate, st_moe_sizes_t* out);
moe_status_t st_dense_ffn_host(const st_model_t* model, const char* prefix, int hidden, int intermediate, float* gamma,
                               uint8_t* w13, float* s13, uint8_t* w2, float* s2);

/* One tensor-parallel rank of an attention layer, tensors under `prefix`:
 *   input_layernorm.weight                     [H]
 *   self_attn.{q,k,v,o}_proj.weight            F8_E4M3 (q [nq*d][H], k/v [nkv*d][H], o [H][nq*d])
 *   self_attn.{q,k,v,o}_proj.weight_scale_inv  F32
 * into attn_block_weights_t's layout: w_qkv = the rank's q heads, k heads, v
 * heads stacked ([(nq/tp + 2 nkv/tp) * d][H] + scales), w_o = the matching
 * input columns of o_proj ([H][nq/tp * d] + scales); head_dim d = 128. */
typedef struct {
    int hidden, num_q_heads, num_kv_heads, head_dim, tp_size, tp_rank;
} st_attn_spec_t;

typedef struct {
    size_t gamma, w_qkv, s_qkv, w_o, s_o;   /* bytes */
} st_attn_sizes_t;

moe_status_t st_attn_rank_sizes(const st_attn_spec_t* spec, st_attn_sizes_t* out);
moe_status_t st_attn_rank_host(const st_model_t* model, const char* prefix, const st_attn_spec_t* spec, float* gamma,
                               uint8_t* w_qkv, float* s_qkv, uint8_t* w_o, float* s_o);

#ifdef __cplusplus
}
#endif

#endif /* TIME_B200_ST_LOADER_H */
