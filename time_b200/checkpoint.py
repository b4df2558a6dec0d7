"""Safetensors checkpoints (the engine's FP8 GLM-4.x format) into this
library's weight layouts, through the C loader of libkernels.so
(include/st_loader.h), plus a writer for such checkpoints.

    ck = Checkpoint("/path/to/model")                    # index + shards, or one file
    w = ck.moe_layer("model.layers.3.", synth.GLM, ep_size=8, ep_rank=r, placement=slots, device=dev)
    layer = moe.MoELayer(synth.GLM, w, max_tokens=T, ep_size=8, ep_rank=r, comm=comm)
    a = ck.attn_rank("model.layers.3.", synth.GLM_ATTN, tp=8, rank=r, device=dev)

The reference reads the same files in src/terra/engine.t:412-720 but never
fills its per-layer weights; tensor names follow the HF GLM-4.x layout
(mlp.experts.{e}.{gate,up,down}_proj.weight + weight_scale_inv, ...).
"""
from __future__ import annotations

import ctypes
import json
import os
import struct
from ctypes import c_char_p, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

import numpy as np

from . import moe as M

ST_DTYPES = {1: "F8_E4M3", 2: "F16", 3: "BF16", 4: "F32", 5: "I8", 6: "I16", 7: "I32", 8: "I64", 9: "U8",
             10: "BOOL", 11: "F64", 12: "F8_E5M2"}
# numpy storage of each dtype (F8 / BF16 kept as their raw bits)
NP_OF = {"F8_E4M3": np.uint8, "F8_E5M2": np.uint8, "F16": np.float16, "BF16": np.uint16, "F32": np.float32,
         "I8": np.int8, "I16": np.int16, "I32": np.int32, "I64": np.int64, "U8": np.uint8, "BOOL": np.bool_,
         "F64": np.float64}


class StTensor(ctypes.Structure):
    _fields_ = [("dtype", c_int), ("ndim", c_int), ("shape", c_int64 * 8), ("data", c_void_p), ("nbytes", c_uint64)]


class MoeSpec(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("num_experts", c_int), ("intermediate", c_int), ("num_shared", c_int),
                ("ep_size", c_int), ("ep_rank", c_int), ("slot_of_expert", c_void_p)]


class MoeSizes(ctypes.Structure):
    _fields_ = [(n, c_size_t) for n in ("gamma", "router_w", "router_bias", "w13", "s13", "w2", "s2")]


class AttnSpec(ctypes.Structure):
    _fields_ = [(n, c_int) for n in ("hidden", "num_q_heads", "num_kv_heads", "head_dim", "tp_size", "tp_rank")]


class AttnSizes(ctypes.Structure):
    _fields_ = [(n, c_size_t) for n in ("gamma", "w_qkv", "s_qkv", "w_o", "s_o")]


_bound = False


def lib():
    global _bound
    k = M.libs()["libkernels.so"]
    if not _bound:
        k.st_open.argtypes = [c_char_p, ctypes.POINTER(c_void_p)]
        k.st_close.argtypes = [c_void_p]
        k.st_close.restype = None
        k.st_num_tensors.argtypes = [c_void_p]
        k.st_tensor_name.argtypes = [c_void_p, c_int]
        k.st_tensor_name.restype = c_char_p
        k.st_get.argtypes = [c_void_p, c_char_p, ctypes.POINTER(StTensor)]
        k.st_moe_layer_sizes.argtypes = [ctypes.POINTER(MoeSpec), ctypes.POINTER(MoeSizes)]
        k.st_moe_layer_host.argtypes = [c_void_p, c_char_p, ctypes.POINTER(MoeSpec)] + [c_void_p] * 8
        k.st_attn_rank_sizes.argtypes = [ctypes.POINTER(AttnSpec), ctypes.POINTER(AttnSizes)]
        k.st_attn_rank_host.argtypes = [c_void_p, c_char_p, ctypes.POINTER(AttnSpec)] + [c_void_p] * 5
        _bound = True
    return k


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


class Checkpoint:
    def __init__(self, path):
        self._h = None
        self._k = lib()
        h = c_void_p()
        M.check("st_open", self._k.st_open(str(path).encode(), ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            self._k.st_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def names(self) -> list[str]:
        return [self._k.st_tensor_name(self._h, i).decode() for i in range(self._k.st_num_tensors(self._h))]

    def get(self, name: str) -> tuple[str, np.ndarray]:
        """(dtype name, a copy of the tensor as numpy; F8 / BF16 as raw bits)."""
        t = StTensor()
        M.check("st_get", self._k.st_get(self._h, name.encode(), ctypes.byref(t)))
        dt = ST_DTYPES[t.dtype]
        shape = tuple(t.shape[i] for i in range(t.ndim))
        raw = (ctypes.c_uint8 * t.nbytes).from_address(t.data) if t.nbytes else b""
        arr = np.frombuffer(bytes(raw), dtype=NP_OF[dt]).reshape(shape).copy()
        return dt, arr

    def moe_layer(self, prefix: str, shape, ep_size: int = 1, ep_rank: int = 0, placement=None, device=None) -> dict:
        """The MoE weights of `prefix` for one EP rank in MoELayer's layout (torch tensors)."""
        import torch
        slots = None if placement is None else np.ascontiguousarray(placement, dtype=np.int32)
        spec = MoeSpec(shape.hidden, shape.num_experts, shape.intermediate, shape.num_shared, ep_size, ep_rank,
                       None if slots is None else _p(slots))
        sz = MoeSizes()
        M.check("st_moe_layer_sizes", self._k.st_moe_layer_sizes(ctypes.byref(spec), ctypes.byref(sz)))
        H, I, E = shape.hidden, shape.intermediate, shape.num_experts
        G = E // ep_size + shape.num_shared
        gamma = np.empty(H, np.float32)
        router_w = np.empty((E, H), np.float32)
        bias = np.empty(E, np.float32)
        has_bias = c_int(0)
        w13 = np.empty((G, 2 * I, H), np.uint8)
        s13 = np.empty((G, 2 * I // 128, H // 128), np.float32)
        w2 = np.empty((G, H, I), np.uint8)
        s2 = np.empty((G, H // 128, I // 128), np.float32)
        M.check("st_moe_layer_host", self._k.st_moe_layer_host(
            self._h, prefix.encode(), ctypes.byref(spec), _p(gamma), _p(router_w), _p(bias), ctypes.addressof(has_bias),
            _p(w13), _p(s13), _p(w2), _p(s2)))
        out = {"gamma": gamma, "router_w": router_w, "router_bias": bias if has_bias.value else None,
               "w13": w13, "s13": s13, "w2": w2, "s2": s2}
        return {k: (None if v is None else torch.from_numpy(v).to(device) if device is not None else torch.from_numpy(v))
                for k, v in out.items()}

    def attn_rank(self, prefix: str, shape, tp: int = 1, rank: int = 0, device=None) -> dict:
        """One TP rank's attention weights of `prefix` in AttnBlock's layout (torch tensors)."""
        import torch
        spec = AttnSpec(shape.hidden, shape.num_q_heads, shape.num_kv_heads, shape.head_dim, tp, rank)
        sz = AttnSizes()
        M.check("st_attn_rank_sizes", self._k.st_attn_rank_sizes(ctypes.byref(spec), ctypes.byref(sz)))
        H, d = shape.hidden, shape.head_dim
        nq, nkv = shape.num_q_heads // tp, shape.num_kv_heads // tp
        gamma = np.empty(H, np.float32)
        w_qkv = np.empty(((nq + 2 * nkv) * d, H), np.uint8)
        s_qkv = np.empty(((nq + 2 * nkv) * d // 128, H // 128), np.float32)
        w_o = np.empty((H, nq * d), np.uint8)
        s_o = np.empty((H // 128, nq * d // 128), np.float32)
        M.check("st_attn_rank_host", self._k.st_attn_rank_host(self._h, prefix.encode(), ctypes.byref(spec), _p(gamma),
                                                               _p(w_qkv), _p(s_qkv), _p(w_o), _p(s_o)))
        out = {"gamma": gamma, "w_qkv": w_qkv, "s_qkv": s_qkv, "w_o": w_o, "s_o": s_o}
        return {k: (torch.from_numpy(v).to(device) if device is not None else torch.from_numpy(v)) for k, v in out.items()}


# ---------------------------------------------------------------- writing

def write_safetensors(path, tensors: dict, metadata: dict | None = None) -> None:
    """tensors: name -> (dtype name, numpy array holding that dtype's bytes)."""
    header = {}
    off = 0
    blobs = []
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = metadata
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def write_checkpoint(directory, tensors: dict, shards: int = 1) -> None:
    """A model directory: one model.safetensors, or `shards` files plus
    model.safetensors.index.json (tensors split round-robin by name order)."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    if shards == 1:
        write_safetensors(d / "model.safetensors", tensors)
        return
    names = list(tensors)
    weight_map = {}
    for s in range(shards):
        fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        part = {n: tensors[n] for i, n in enumerate(names) if i % shards == s}
        write_safetensors(d / fname, part)
        weight_map.update({n: fname for n in part})
    (d / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))


def glm_tensors_from_synth(moe_w: dict, shape, layer: int, attn_w: dict | None = None, router_dtype: str = "BF16",
                           norm_dtype: str = "BF16") -> dict:
    """HF GLM-4.x-named tensors of one layer from this package's synthetic
    weights (synth.make_moe_weights / make_attn_weights, all experts): the
    inverse of the loader's assembly."""
    def f32_as(dt: str, a: np.ndarray):
        a = np.asarray(a, dtype=np.float32)
        if dt == "F32":
            return "F32", a
        if dt == "F16":
            return "F16", a.astype(np.float16)
        u = a.view(np.uint32)
        return "BF16", ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

    P = f"model.layers.{layer}."
    out = {}
    H, I, E = shape.hidden, shape.intermediate, shape.num_experts
    w13, s13, w2, s2 = (moe_w[k].cpu().numpy() for k in ("w13", "s13", "w2", "s2"))
    out[P + "post_attention_layernorm.weight"] = f32_as(norm_dtype, moe_w["gamma"].cpu().numpy())
    out[P + "mlp.gate.weight"] = f32_as(router_dtype, moe_w["router_w"].cpu().numpy())
    if moe_w.get("router_bias") is not None:
        out[P + "mlp.gate.e_score_correction_bias"] = ("F32", moe_w["router_bias"].cpu().numpy())
    for g in range(E + shape.num_shared):
        base = P + (f"mlp.experts.{g}." if g < E else "mlp.shared_experts.")
        out[base + "gate_proj.weight"] = ("F8_E4M3", w13[g, :I])
        out[base + "gate_proj.weight_scale_inv"] = ("F32", s13[g, :I // 128])
        out[base + "up_proj.weight"] = ("F8_E4M3", w13[g, I:])
        out[base + "up_proj.weight_scale_inv"] = ("F32", s13[g, I // 128:])
        out[base + "down_proj.weight"] = ("F8_E4M3", w2[g])
        out[base + "down_proj.weight_scale_inv"] = ("F32", s2[g])
    if attn_w is not None:
        out[P + "input_layernorm.weight"] = f32_as(norm_dtype, attn_w["gamma"].cpu().numpy())
        for n in ("q", "k", "v", "o"):
            out[P + f"self_attn.{n}_proj.weight"] = ("F8_E4M3", attn_w["w_" + n].cpu().numpy())
            out[P + f"self_attn.{n}_proj.weight_scale_inv"] = ("F32", attn_w["s_" + n].cpu().numpy())
    return out


def glm_model_tensors(shape, weights: dict, norm_dtype: str = "F32") -> dict:
    """Every HF GLM-4.x-named tensor of a whole model from
    synth.make_model_weights: model.embed_tokens.weight / lm_head.weight
    (BF16), model.norm.weight, and per layer the attention, the layer norms and
    the FFN (dense layers as mlp.{gate,up,down}_proj, MoE layers as
    glm_tensors_from_synth writes them)."""
    def bf16_bits(t):
        return t.detach().cpu().contiguous().view(torch_u16()).numpy()

    out = {
        "model.embed_tokens.weight": ("BF16", bf16_bits(weights["embed"])),
        "lm_head.weight": ("BF16", bf16_bits(weights["lm_head"])),
        "model.norm.weight": ("F32", weights["final_norm"].detach().cpu().numpy().astype(np.float32)),
    }
    for l, layer in enumerate(weights["layers"]):
        if not layer["dense"]:
            out.update(glm_tensors_from_synth(layer["ffn"], shape.moe(), l, attn_w=layer["attn"],
                                              router_dtype="F32", norm_dtype=norm_dtype))
            continue
        # the dense FFN: glm_tensors_from_synth's single expert, renamed
        one = glm_tensors_from_synth(layer["ffn"], shape.dense(), l, attn_w=layer["attn"], router_dtype="F32",
                                     norm_dtype=norm_dtype)
        P = f"model.layers.{l}."
        for name, v in one.items():
            if name.startswith(P + "mlp.experts.0."):
                out[name.replace("mlp.experts.0.", "mlp.")] = v
            elif not name.startswith(P + "mlp.gate."):
                out[name] = v
    return out


def torch_u16():
    import torch
    return torch.uint16 if hasattr(torch, "uint16") else torch.int16


def write_model(directory, shape, weights: dict, shards: int = 1, tie_embeddings: bool = False) -> None:
    """A model directory the engine's init_engine reads: config.json (HF
    GLM-4.x keys) and the checkpoint (glm_model_tensors)."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    cfg = {
        "architectures": ["Glm4MoeForCausalLM"],
        "hidden_size": shape.hidden,
        "num_hidden_layers": shape.num_layers,
        "num_attention_heads": shape.num_q_heads,
        "num_key_value_heads": shape.num_kv_heads,
        "head_dim": shape.head_dim,
        "partial_rotary_factor": shape.rotary_dim / shape.head_dim,
        "vocab_size": shape.vocab_size,
        "n_routed_experts": shape.num_experts,
        "num_experts_per_tok": shape.top_k,
        "moe_intermediate_size": shape.moe_intermediate,
        "intermediate_size": shape.dense_intermediate,
        "n_shared_experts": shape.num_shared,
        "first_k_dense_replace": shape.first_dense,
        "rope_theta": shape.rope_theta,
        "rms_norm_eps": shape.eps,
        "tie_word_embeddings": tie_embeddings,
    }
    (d / "config.json").write_text(json.dumps(cfg, indent=1))
    tensors = glm_model_tensors(shape, weights)
    if tie_embeddings:
        del tensors["lm_head.weight"]
    write_checkpoint(d, tensors, shards=shards)
