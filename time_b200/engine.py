"""ctypes front-end of the serving engine (time_b200/lib/engine.so,
include/engine.h).

:class:`NativeEngine` has the interface of the reference's
src/server/engine_wrapper.py NativeEngine (load / is_loaded / get_info /
prefill / decode_step / batch_decode / free_request / shutdown) over the same
seven engine.so symbols, so the reference's server code drives this engine
unchanged.  :meth:`NativeEngine.from_weights` builds an engine from weights
already in device memory (synth.make_model_weights), for tests and
benchmarks without a checkpoint on disk.
"""
from __future__ import annotations

import ctypes
import dataclasses
from ctypes import c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path
from typing import List, Optional, Tuple

import numpy as np

from . import attn as A
from . import lib_path
from . import moe as M


class EngineConfig(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("num_layers", c_int), ("first_dense", c_int), ("num_q_heads", c_int),
                ("num_kv_heads", c_int), ("head_dim", c_int), ("rotary_dim", c_int), ("vocab_size", c_int),
                ("num_experts", c_int), ("top_k", c_int), ("moe_intermediate", c_int), ("num_shared", c_int),
                ("dense_intermediate", c_int), ("rope_theta", c_float), ("rms_eps", c_float), ("max_batch", c_int),
                ("max_seq", c_int), ("prefill_chunk", c_int), ("num_cache_pages", c_int), ("num_gpus", c_int)]


@dataclasses.dataclass
class EngineInfo:
    hidden_dim: int
    num_layers: int
    num_heads: int
    vocab_size: int
    num_experts: int
    top_k_experts: int
    num_gpus: int
    max_batch: int
    max_seq: int
    kv_pages_used: int
    kv_pages_max: int
    active_requests: int
    num_tensors: int
    use_gpu: int


_bound = False


def lib() -> ctypes.CDLL:
    global _bound
    e = M.load()["engine.so"]
    if not _bound:
        e.init_engine.argtypes = [ctypes.c_char_p, c_int32, c_int32, c_int32]
        e.init_engine.restype = c_void_p
        e.prefill_opaque.argtypes = [c_void_p, c_int64, ctypes.POINTER(c_int64), c_int32, c_float, c_float, c_float,
                                     c_int32]
        e.prefill_opaque.restype = c_void_p
        e.decode_step_opaque.argtypes = [c_void_p, c_void_p, ctypes.POINTER(c_int64), ctypes.POINTER(c_int32)]
        e.decode_step_opaque.restype = c_int32
        e.free_request_opaque.argtypes = [c_void_p, c_void_p]
        e.free_request_opaque.restype = None
        e.free_engine.argtypes = [c_void_p]
        e.free_engine.restype = None
        e.get_engine_info.argtypes = [c_void_p, c_int32]
        e.get_engine_info.restype = c_int64
        e.run_batch_decode_ext.argtypes = [c_void_p, ctypes.POINTER(c_void_p), c_int32, ctypes.POINTER(c_int64),
                                           ctypes.POINTER(c_int32)]
        e.run_batch_decode_ext.restype = c_int32
        e.glm_engine_create.argtypes = [ctypes.POINTER(EngineConfig), ctypes.POINTER(c_void_p)]
        e.glm_engine_set_embedding.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p]
        e.glm_engine_set_layer.argtypes = [c_void_p, c_int, ctypes.POINTER(A.BlockWeights),
                                           ctypes.POINTER(M.LayerWeights)]
        e.glm_engine_set_layer_rank.argtypes = [c_void_p, c_int, c_int, ctypes.POINTER(A.BlockWeights),
                                                ctypes.POINTER(M.LayerWeights)]
        e.glm_engine_set_embedding_rank.argtypes = [c_void_p, c_int, c_void_p, c_void_p, c_void_p]
        e.glm_engine_copy_logits.argtypes = [c_void_p, c_void_p, c_int]
        e.glm_engine_check_error.argtypes = [c_void_p]
        e.glm_engine_set_capture.argtypes = [c_void_p, c_int]
        e.glm_engine_copy_routing.argtypes = [c_void_p, c_int, c_int, c_void_p, c_void_p]
        e.glm_engine_request_pages.argtypes = [c_void_p, c_void_p, c_void_p, c_int]
        e.glm_engine_copy_kv.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]
        e.glm_engine_set_timing.argtypes = [c_void_p, c_int]
        e.glm_engine_stage_ms.argtypes = [c_void_p, ctypes.POINTER(c_float)]
        e.glm_engine_device_bytes.argtypes = [ctypes.POINTER(EngineConfig)]
        e.glm_engine_device_bytes.restype = c_size_t
        _bound = True
    return e


def engine_config(shape, max_batch: int, max_seq: int, prefill_chunk: int = 0,
                  num_cache_pages: int = 0, num_gpus: int = 1) -> EngineConfig:
    """EngineConfig of a synth.ModelShape."""
    return EngineConfig(shape.hidden, shape.num_layers, shape.first_dense, shape.num_q_heads, shape.num_kv_heads,
                        shape.head_dim, shape.rotary_dim, shape.vocab_size, shape.num_experts, shape.top_k,
                        shape.moe_intermediate, shape.num_shared, shape.dense_intermediate, shape.rope_theta,
                        shape.eps, max_batch, max_seq, prefill_chunk, num_cache_pages, num_gpus)


def device_bytes(shape, max_batch: int, max_seq: int, prefill_chunk: int = 0, num_cache_pages: int = 0) -> int:
    """Device bytes the engine allocates beyond the weights (KV pool, activations, logits)."""
    cfg = engine_config(shape, max_batch, max_seq, prefill_chunk, num_cache_pages)
    return int(lib().glm_engine_device_bytes(ctypes.byref(cfg)))


class NativeEngine:
    """The reference's NativeEngine interface (src/server/engine_wrapper.py:33-196)
    over this package's engine.so."""

    def __init__(self, engine_path: Optional[str] = None, model_dir: str = "", max_batch: int = 64,
                 max_seq: int = 4096, num_gpus: int = 1):
        self.engine_path = engine_path or str(lib_path("engine.so"))
        self.model_dir = model_dir
        self.max_batch = max_batch
        self.max_seq = max_seq
        self.num_gpus = num_gpus
        self.lib = None
        self.handle = None
        self._loaded = False
        self._keep = []          # device tensors an in-memory engine reads

    # ---------------------------------------------------------------- reference interface

    def load(self) -> bool:
        if not Path(self.engine_path).exists():
            return False
        self.lib = lib()
        h = self.lib.init_engine(self.model_dir.encode("utf-8"), self.max_batch, self.max_seq, self.num_gpus)
        if h:
            self.handle = h
            self._loaded = True
            return True
        return False

    def is_loaded(self) -> bool:
        return self._loaded and self.handle is not None

    def get_info(self) -> Optional[EngineInfo]:
        if not self.is_loaded():
            return None
        v = [int(self.lib.get_engine_info(self.handle, i)) for i in range(14)]
        return EngineInfo(*v)

    def prefill(self, request_id: int, token_ids: List[int], temperature: float, top_p: float, rep_penalty: float,
                max_tokens: int) -> Optional[int]:
        if not self.is_loaded():
            return None
        arr = (c_int64 * len(token_ids))(*token_ids)
        st = self.lib.prefill_opaque(self.handle, request_id, arr, len(token_ids), temperature, top_p, rep_penalty,
                                     max_tokens)
        return st if st else None

    def decode_step(self, state_ptr) -> Tuple[Optional[int], bool]:
        if not self.is_loaded() or not state_ptr:
            return None, True
        tok, done = c_int64(0), c_int32(0)
        status = self.lib.decode_step_opaque(self.handle, state_ptr, ctypes.byref(tok), ctypes.byref(done))
        if status < 0:
            return None, True
        return int(tok.value), bool(done.value)

    def batch_decode(self, state_ptrs) -> List[Tuple[Optional[int], bool]]:
        """Like the reference: a finished request's last token is reported as None."""
        raw = self.batch_decode_raw(state_ptrs)
        if raw is None:
            return [(None, True) for _ in state_ptrs]
        return [(t if not d else None, d) for t, d in raw]

    def batch_decode_raw(self, state_ptrs) -> Optional[List[Tuple[int, bool]]]:
        """run_batch_decode_ext's tokens and done flags as returned (the token
        of a request's final step included)."""
        if not self.is_loaded() or not state_ptrs:
            return None
        n = len(state_ptrs)
        arr = (c_void_p * n)(*state_ptrs)
        toks = (c_int64 * n)()
        done = (c_int32 * n)()
        status = self.lib.run_batch_decode_ext(self.handle, arr, n, toks, done)
        if status < 0:
            return None
        return [(int(toks[i]), bool(done[i])) for i in range(n)]

    def free_request(self, state_ptr) -> None:
        if self.is_loaded() and state_ptr:
            self.lib.free_request_opaque(self.handle, state_ptr)

    def shutdown(self) -> None:
        if self.is_loaded():
            self.lib.free_engine(self.handle)
        self.handle = None
        self._loaded = False
        self._keep = []

    def __del__(self):
        try:
            self.shutdown()
        except Exception:
            pass

    # ---------------------------------------------------------------- in-memory weights

    @classmethod
    def from_weights(cls, shape, weights: dict, max_batch: int, max_seq: int, prefill_chunk: int = 0,
                     num_cache_pages: int = 0, num_gpus: int = 1) -> "NativeEngine":
        """An engine over device tensors (synth.make_model_weights on a CUDA
        device; layers may share tensors).  The tensors, and the rank-layout
        copies of whole-model attention weights made here, are kept alive by
        the returned object; `weights` is not modified.  num_gpus > 1: the
        engine spans the devices from the current one on; each rank's slices
        (its heads, its experts) are copied to its device here."""
        if num_gpus > 1:
            return cls._from_weights_ranks(shape, weights, max_batch, max_seq, prefill_chunk, num_cache_pages,
                                           num_gpus)
        self = cls(max_batch=max_batch, max_seq=max_seq)
        self.lib = lib()
        cfg = engine_config(shape, max_batch, max_seq, prefill_chunk, num_cache_pages)
        h = c_void_p()
        M.check("glm_engine_create", self.lib.glm_engine_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.handle = h.value
        self._loaded = True
        try:
            # the engine reads these tensors for its whole life: keep them here
            # (rank-layout copies made below included), never in the caller's dict
            own = {}
            self._keep = [weights, own]
            M.check("glm_engine_set_embedding",
                    self.lib.glm_engine_set_embedding(self.handle, M.ptr(weights["embed"]),
                                                      M.ptr(weights["final_norm"]), M.ptr(weights["lm_head"])))
            for l, layer in enumerate(weights["layers"]):
                a = layer["attn"]
                if a.get("w_qkv") is None:   # whole-model layout -> the tp 1 rank layout (one copy per weight set)
                    from . import synth
                    if id(a) not in own:
                        own[id(a)] = synth.attn_rank_slice(a, shape.attn(), 1, 0)
                    a = own[id(a)]
                aw = A.BlockWeights(M.ptr(a["gamma"]), M.ptr(a["w_qkv"]), M.ptr(a["s_qkv"]), M.ptr(a["w_o"]),
                                    M.ptr(a["s_o"]))
                f = layer["ffn"]
                fw = M.LayerWeights(M.ptr(f["gamma"]), M.ptr(f["router_w"]), M.ptr(f.get("router_bias")),
                                    M.ptr(f["w13"]), M.ptr(f["s13"]), M.ptr(f["w2"]), M.ptr(f["s2"]))
                M.check("glm_engine_set_layer",
                        self.lib.glm_engine_set_layer(self.handle, l, ctypes.byref(aw), ctypes.byref(fw)))
        except Exception:
            self.shutdown()
            raise
        return self

    @classmethod
    def _from_weights_ranks(cls, shape, weights: dict, max_batch: int, max_seq: int, prefill_chunk: int,
                            num_cache_pages: int, n: int) -> "NativeEngine":
        import torch
        from . import synth
        self = cls(max_batch=max_batch, max_seq=max_seq, num_gpus=n)
        self.lib = lib()
        dev0 = torch.cuda.current_device()
        cfg = engine_config(shape, max_batch, max_seq, prefill_chunk, num_cache_pages, n)
        h = c_void_p()
        M.check("glm_engine_create", self.lib.glm_engine_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.handle = h.value
        self._loaded = True
        try:
            own = {}                    # (id of a weight set, rank) -> that rank's copy
            self._keep = [weights, own]

            def on(t, r):
                return None if t is None else t.to(torch.device("cuda", dev0 + r)).contiguous()

            for r in range(n):
                key = ("embed", r)
                own[key] = {"embed": on(weights["embed"], r)}
                if r == 0:
                    own[key]["final_norm"] = on(weights["final_norm"], 0)
                    own[key]["lm_head"] = on(weights["lm_head"], 0)
                e = own[key]
                M.check("glm_engine_set_embedding_rank",
                        self.lib.glm_engine_set_embedding_rank(self.handle, r, M.ptr(e["embed"]),
                                                               M.ptr(e.get("final_norm")), M.ptr(e.get("lm_head"))))
            for l, layer in enumerate(weights["layers"]):
                a, f = layer["attn"], layer["ffn"]
                dense = l < shape.first_dense
                for r in range(n):
                    if (id(a), r) not in own:
                        src = a if a.get("w_qkv") is None else None
                        if src is None:
                            raise ValueError("several GPUs need whole-model attention weights (w_q/w_k/w_v/w_o)")
                        own[(id(a), r)] = {k: on(v, r) for k, v in synth.attn_rank_slice(a, shape.attn(), n, r).items()}
                    if (id(f), r) not in own:
                        sl = f if dense else synth.expert_slice(f, shape.moe(), n, r)
                        own[(id(f), r)] = {k: on(v, r) for k, v in sl.items()}
                    ar, fr = own[(id(a), r)], own[(id(f), r)]
                    aw = A.BlockWeights(M.ptr(ar["gamma"]), M.ptr(ar["w_qkv"]), M.ptr(ar["s_qkv"]), M.ptr(ar["w_o"]),
                                        M.ptr(ar["s_o"]))
                    fw = M.LayerWeights(M.ptr(fr["gamma"]), M.ptr(fr["router_w"]), M.ptr(fr.get("router_bias")),
                                        M.ptr(fr["w13"]), M.ptr(fr["s13"]), M.ptr(fr["w2"]), M.ptr(fr["s2"]))
                    M.check("glm_engine_set_layer_rank",
                            self.lib.glm_engine_set_layer_rank(self.handle, r, l, ctypes.byref(aw),
                                                               ctypes.byref(fw)))
            torch.cuda.set_device(dev0)
        except Exception:
            self.shutdown()
            raise
        return self

    def copy_logits(self, rows: int) -> np.ndarray:
        """fp32 logits [rows][vocab] of the last decode step."""
        V = int(self.lib.get_engine_info(self.handle, 3))
        out = np.empty((rows, V), np.float32)
        M.check("glm_engine_copy_logits", self.lib.glm_engine_copy_logits(self.handle, out.ctypes.data, rows))
        return out

    def set_capture(self, on: bool) -> None:
        M.check("glm_engine_set_capture", self.lib.glm_engine_set_capture(self.handle, 1 if on else 0))

    def routing(self, layer: int, rows: int, top_k: int) -> tuple[np.ndarray, np.ndarray]:
        """Layer `layer`'s top-k ids and weights of the last forward's rows (capture on)."""
        idx = np.empty((rows, top_k), np.int32)
        w = np.empty((rows, top_k), np.float32)
        M.check("glm_engine_copy_routing",
                self.lib.glm_engine_copy_routing(self.handle, layer, rows, idx.ctypes.data, w.ctypes.data))
        return idx, w

    def request_pages(self, state) -> np.ndarray:
        n = int(self.lib.glm_engine_request_pages(self.handle, state, None, 0))
        assert n >= 0
        out = np.empty(max(n, 1), np.int32)
        self.lib.glm_engine_request_pages(self.handle, state, out.ctypes.data, n)
        return out[:n]

    def kv_pages(self, layer: int, pages, kv_heads: int) -> tuple[np.ndarray, np.ndarray]:
        """K and V (fp32 copies of the bf16 pages) of the given page ids, [n][16][kv_heads][128]."""
        import torch
        ks, vs = [], []
        for p in pages:
            k = np.empty((16, kv_heads, 128), np.uint16)
            v = np.empty((16, kv_heads, 128), np.uint16)
            M.check("glm_engine_copy_kv", self.lib.glm_engine_copy_kv(self.handle, layer, int(p), 1, k.ctypes.data,
                                                                      v.ctypes.data))
            ks.append(torch.from_numpy(k.view(np.int16)).view(torch.bfloat16).float().numpy())
            vs.append(torch.from_numpy(v.view(np.int16)).view(torch.bfloat16).float().numpy())
        return np.stack(ks), np.stack(vs)

    def check_error(self) -> None:
        M.check("glm_engine_check_error", self.lib.glm_engine_check_error(self.handle))

    def set_timing(self, on: bool) -> None:
        M.check("glm_engine_set_timing", self.lib.glm_engine_set_timing(self.handle, 1 if on else 0))

    def stage_ms(self) -> dict:
        v = (c_float * 4)()
        M.check("glm_engine_stage_ms", self.lib.glm_engine_stage_ms(self.handle, v))
        return {"embed": v[0], "attention": v[1], "ffn": v[2], "head": v[3]}
