"""ctypes bindings of include/moe_layer.h and the new entry points of
include/cublas_wrappers.h / nccl_wrappers.h, plus a small host-side driver in
the style of the reference's ctypes engine wrapper
(src/server/engine_wrapper.py:64-98): explicit argtypes, device pointers as
integers, status codes turned into exceptions.

Device memory and streams come from torch (plumbing only); every computation
runs in the package's CUDA libraries.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import load

c_int, c_float, c_size_t, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p
c_i32p = ctypes.POINTER(ctypes.c_int32)

STATUS = {0: "ok", 1: "invalid argument", 2: "CUDA error", 3: "unsupported configuration",
          4: "device-side wait timed out", 5: "NCCL error", 6: "workspace too small or row capacity exceeded"}


class MoEError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {STATUS.get(code, code)} ({code})")
        self.code = code


class LayerConfig(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("num_experts", c_int), ("top_k", c_int), ("intermediate", c_int),
                ("num_shared", c_int), ("rms_eps", c_float), ("max_tokens", c_int), ("ep_size", c_int),
                ("ep_rank", c_int)]


class LayerWeights(ctypes.Structure):
    _fields_ = [("norm_gamma", c_void_p), ("router_w", c_void_p), ("router_bias", c_void_p), ("w13", c_void_p),
                ("s13", c_void_p), ("w2", c_void_p), ("s2", c_void_p)]


class GroupedGemmArgs(ctypes.Structure):
    _fields_ = [("mode", c_int), ("num_groups", c_int), ("K", c_int), ("N", c_int), ("rows", c_int),
                ("a", c_void_p), ("a_scale", c_void_p), ("a_ld", c_int), ("w", c_void_p), ("w_scale", c_void_p),
                ("count", c_void_p), ("start", c_void_p), ("out", c_void_p), ("out_scale", c_void_p),
                ("out_ld", c_int)]


NUM_STAGES = 7
STAGE_NAMES = ("rmsnorm_quant", "router_topk", "permute", "gather", "gemm_gate_up", "gemm_down", "combine")

GEMM_GATED_SWIGLU = 0
GEMM_DOWN_BF16 = 1
GEMM_SMALL_TILES = 0x10   # or-ed into a mode: the decode form (tiles of <= 32 rows)
GEMM_FULL_TILES = 0x20
GEMM_ONE_SM_TILES = 0x40  # the full form on one SM per tile
GEMM_PAIR_TILES = 0x80    # the full form on pairs of SMs (tcgen05 cta_group::2)
GEMM_TOKEN_TILES = 0x30   # the full form with 128 token rows x 256 weight rows per instruction
GEMM_ACT_X2 = 0x100       # two-term e4m3 activations (hi plane, lo plane rows*K bytes on)

_bound = False


def libs():
    global _bound
    L = load()
    if not _bound:
        k = L["libkernels.so"]
        k.moe_layer_create.argtypes = [ctypes.POINTER(LayerConfig), ctypes.POINTER(LayerWeights), c_void_p,
                                       ctypes.POINTER(c_void_p)]
        k.moe_layer_destroy.argtypes = [c_void_p]
        k.moe_layer_workspace_bytes.argtypes = [c_void_p]
        k.moe_layer_workspace_bytes.restype = c_size_t
        k.moe_layer_forward.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p]
        k.moe_layer_forward_routed.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p,
                                               c_size_t, c_void_p]
        k.moe_layer_last_routing.argtypes = [c_void_p, c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p),
                                             ctypes.POINTER(c_void_p)]
        k.moe_layer_check_error.argtypes = [c_void_p, c_void_p]
        k.moe_layer_set_stage_events.argtypes = [c_void_p, c_void_p]
        k.moe_rmsnorm_quant.argtypes = [c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p, c_void_p,
                                        c_int, c_void_p]
        k.moe_router_topk.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                      c_void_p, c_void_p, c_void_p, c_void_p]
        k.moe_permute.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_int, c_void_p, c_void_p]
        k.moe_gather_rows.argtypes = [c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int,
                                      c_void_p]
        k.moe_combine.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                  c_void_p, c_void_p]
        k.moe_rmsnorm_quant_n.argtypes = [c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_int, c_void_p]
        k.moe_router_logits.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]
        k.moe_router_logits_rc.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]
        k.moe_router_columns.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p]
        k.moe_rmsnorm_quant_rc.argtypes = [c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_int, c_void_p]
        k.moe_topk_softmax.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]
        k.moe_router_topk_noalloc.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                              c_void_p, c_void_p]
        k.moe_combine_split.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                        c_int, c_int, c_void_p, c_void_p]
        k.moe_permute_padded.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p]
        k.moe_layer_set_expert_placement.argtypes = [c_void_p, c_void_p]
        k.moe_layer_set_gemm_form.argtypes = [c_void_p, c_int]
        k.moe_layer_set_act_planes.argtypes = [c_void_p, c_int]
        k.moe_ep_pack_rows_x2.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int,
                                          c_void_p, c_void_p]
        k.moe_ep_gather_x2.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                                       c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p]
        k.moe_layer_get_act_planes.argtypes = [c_void_p, ctypes.POINTER(c_int)]
        k.moe_rmsnorm_quant_x2.argtypes = [c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p, c_int,
                                           c_void_p, c_void_p, c_void_p, c_int, c_void_p]
        k.moe_gather_rows_x2.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int,
                                         c_void_p, c_void_p, c_void_p, c_int, c_void_p]
        k.moe_ep_remap_experts.argtypes = [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p]
        k.moe_scatter_rows_x2.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_int,
                                          c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int,
                                          c_void_p]
        k.moe_ep_token_rows.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p]
        k.moe_layer_peer_bytes.argtypes = [c_void_p]
        k.moe_layer_peer_bytes.restype = c_size_t
        k.moe_layer_set_peer_buffers.argtypes = [c_void_p, c_void_p, c_int]
        k.moe_permute_mb_scratch_bytes.argtypes = [c_int, c_int, c_int, c_int]
        k.moe_permute_mb_scratch_bytes.restype = c_size_t
        k.moe_permute_mb.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_size_t, c_void_p]
        k.moe_ep_row_bytes.argtypes = [c_int]
        k.moe_ep_row_bytes.restype = c_size_t
        sz_p = ctypes.POINTER(c_size_t)
        k.moe_ep_plan_host.argtypes = [c_int, c_int, c_i32p, c_i32p, sz_p, sz_p, sz_p, sz_p, sz_p, sz_p]
        k.moe_ep_pack_rows.argtypes = [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p,
                                       c_void_p]
        k.moe_ep_recv_plan.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_void_p, c_int, c_int, c_void_p, c_void_p]
        k.moe_ep_gather.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p,
                                    c_void_p, c_int, c_void_p]
        k.moe_ep_pack_y.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]
        k.moe_status_string.restype = ctypes.c_char_p
        k.kernels_last_error.restype = c_int
        b = L["libcublaswrap.so"]
        b.cbwFp8BlockScaledGroupedGemm.argtypes = [ctypes.POINTER(GroupedGemmArgs), c_void_p, c_void_p]
        b.cbwFp8BlockScaledGroupedGemmRowOut.argtypes = [ctypes.POINTER(GroupedGemmArgs), c_void_p, c_void_p,
                                                         c_void_p]
        n = L["libncclwrap.so"]
        n.ncwGetUniqueId.argtypes = [ctypes.POINTER(UniqueId)]
        n.ncwCommInitRank.argtypes = [ctypes.POINTER(c_void_p), c_int, UniqueId, c_int]
        n.ncwCommInitRankTimeout.argtypes = [ctypes.POINTER(c_void_p), c_int, UniqueId, c_int, c_int]
        n.ncwCommDestroy.argtypes = [c_void_p]
        n.ncwCommAbort.argtypes = [c_void_p]
        n.ncwCommGetAsyncError.argtypes = [c_void_p]
        n.ncwGetErrorString.restype = ctypes.c_char_p
        _bound = True
    return L


class UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_char * 128)]


def ep_plan_host(ep_size: int, experts_per_rank: int, send_expert_counts, recv_counts):
    """moe_ep_plan_host on host int32 sequences; returns
    (send_rows, send_offsets, recv_rows, recv_offsets, send_total, recv_total)."""
    import numpy as np
    k = libs()["libkernels.so"]
    a = np.ascontiguousarray(send_expert_counts, dtype=np.int32)
    b = np.ascontiguousarray(recv_counts, dtype=np.int32)
    assert a.size == ep_size * experts_per_rank and b.size == ep_size * experts_per_rank
    outs = [(c_size_t * ep_size)() for _ in range(4)]
    st, rt = c_size_t(), c_size_t()
    check("moe_ep_plan_host", k.moe_ep_plan_host(ep_size, experts_per_rank, a.ctypes.data_as(c_i32p),
                                                 b.ctypes.data_as(c_i32p), *outs, ctypes.byref(st),
                                                 ctypes.byref(rt)))
    return tuple(list(o) for o in outs) + (st.value, rt.value)


def nccl_comm(rank: int, world: int, timeout_ms: int | None = None) -> int:
    """An ncwComm_t over the torch.distributed world: rank 0 draws the NCCL
    unique id (ncwGetUniqueId) and torch.distributed broadcasts it."""
    import torch.distributed as dist
    n = libs()["libncclwrap.so"]
    uid = UniqueId()
    if rank == 0:
        rc = n.ncwGetUniqueId(ctypes.byref(uid))
        if rc != 0:
            raise RuntimeError(f"ncwGetUniqueId failed: {n.ncwGetErrorString(rc).decode()}")
    raw = bytes(ctypes.string_at(ctypes.addressof(uid), 128)) if rank == 0 else None
    box = [raw]
    dist.broadcast_object_list(box, src=0)
    ctypes.memmove(ctypes.addressof(uid), box[0], 128)
    comm = c_void_p()
    if timeout_ms is None:
        rc = n.ncwCommInitRank(ctypes.byref(comm), world, uid, rank)
    else:
        rc = n.ncwCommInitRankTimeout(ctypes.byref(comm), world, uid, rank, timeout_ms)
    if rc != 0:
        raise RuntimeError(f"ncwCommInitRank failed: {n.ncwGetErrorString(rc).decode()}")
    return comm.value


def nccl_comm_destroy(comm: int | None) -> None:
    if comm:
        libs()["libncclwrap.so"].ncwCommDestroy(comm)


def check(fn: str, code: int) -> None:
    if code != 0:
        raise MoEError(fn, code)


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None passes NULL)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


@dataclass
class MoELayer:
    """A MoE FFN block bound to device weights (dict from time_b200.synth or
    real checkpoint tensors) -- the object the engine would hold per layer."""
    shape: object
    weights: dict
    max_tokens: int
    ep_size: int = 1
    ep_rank: int = 0
    comm: int | None = None

    def __post_init__(self):
        self._k = libs()["libkernels.so"]
        sh = self.shape
        self._cfg = LayerConfig(sh.hidden, sh.num_experts, sh.top_k, sh.intermediate, sh.num_shared, sh.eps,
                                self.max_tokens, self.ep_size, self.ep_rank)
        w = self.weights
        self._w = LayerWeights(ptr(w["gamma"]), ptr(w["router_w"]), ptr(w.get("router_bias")), ptr(w["w13"]),
                               ptr(w["s13"]), ptr(w["w2"]), ptr(w["s2"]))
        h = c_void_p()
        check("moe_layer_create", self._k.moe_layer_create(ctypes.byref(self._cfg), ctypes.byref(self._w),
                                                           self.comm, ctypes.byref(h)))
        self._h = h
        self.workspace_bytes = self._k.moe_layer_workspace_bytes(h)
        self.workspace = None

    def ensure_workspace(self):
        import torch
        if self.workspace is None:
            dev = self.weights["w13"].device
            self.workspace = torch.empty(self.workspace_bytes, dtype=torch.uint8, device=dev)
        return self.workspace

    def forward(self, x, out=None, stream=None, routing=None):
        import torch
        ws = self.ensure_workspace()
        if out is None:
            out = torch.empty_like(x)
        T = x.shape[0]
        if routing is None:
            rc = self._k.moe_layer_forward(self._h, ptr(x), ptr(out), T, ptr(ws), self.workspace_bytes,
                                           stream_ptr(stream))
            check("moe_layer_forward", rc)
        else:
            idx, wts = routing
            rc = self._k.moe_layer_forward_routed(self._h, ptr(x), ptr(idx), ptr(wts), ptr(out), T, ptr(ws),
                                                  self.workspace_bytes, stream_ptr(stream))
            check("moe_layer_forward_routed", rc)
        return out

    def set_stage_events(self, events):
        """events: list of MOE_NUM_STAGES + 1 torch.cuda.Event (created with
        enable_timing) or None to stop recording."""
        if events is None:
            self._ev_arr = None
            check("moe_layer_set_stage_events", self._k.moe_layer_set_stage_events(self._h, None))
            return
        assert len(events) == NUM_STAGES + 1
        for e in events:
            if not e.cuda_event:        # torch creates the CUDA event on first record
                e.record()
        self._ev_arr = (c_void_p * len(events))(*[e.cuda_event for e in events])
        check("moe_layer_set_stage_events", self._k.moe_layer_set_stage_events(self._h, self._ev_arr))

    def set_expert_placement(self, slot_of_expert):
        """Expert -> slot permutation (list of E ints) for expert parallelism;
        the weights this layer was built with must hold the rank's experts in
        slot order (synth.expert_slice(..., slot_of_expert=...))."""
        import numpy as np
        if slot_of_expert is None:
            check("moe_layer_set_expert_placement", self._k.moe_layer_set_expert_placement(self._h, None))
            return
        arr = np.ascontiguousarray(slot_of_expert, dtype=np.int32)
        check("moe_layer_set_expert_placement",
              self._k.moe_layer_set_expert_placement(self._h, arr.ctypes.data_as(c_void_p)))

    def set_gemm_form(self, form: int):
        """GEMM_SMALL_TILES, GEMM_FULL_TILES or 0 (the layer's rule)."""
        check("moe_layer_set_gemm_form", self._k.moe_layer_set_gemm_form(self._h, form))

    def set_act_planes(self, planes: int):
        """1: e4m3 activations; 2: two-term e4m3 (hi + lo residual, one scale).
        Re-sizes the workspace (allocated again on the next forward)."""
        check("moe_layer_set_act_planes", self._k.moe_layer_set_act_planes(self._h, planes))
        nbytes = self._k.moe_layer_workspace_bytes(self._h)
        if nbytes != self.workspace_bytes:
            self.workspace_bytes = nbytes
            self.workspace = None

    @property
    def act_planes(self) -> int:
        v = c_int()
        check("moe_layer_get_act_planes", self._k.moe_layer_get_act_planes(self._h, ctypes.byref(v)))
        return v.value

    def use_peer_memory(self, group=None):
        """Switch the expert-parallel exchange to NVLink peer memory: allocate
        this rank's buffer with torch's symmetric-memory allocator (every rank
        maps every other rank's), zero it, rendezvous, and hand the mapped
        pointers to the layer.  Collective over the torch.distributed group."""
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        nbytes = self._k.moe_layer_peer_bytes(self._h)
        if nbytes == 0:
            raise ValueError("peer memory needs ep_size > 1")
        group = group or dist.group.WORLD
        dev = self.weights["w13"].device
        buf = symm.empty(nbytes, dtype=torch.uint8, device=dev)
        buf.zero_()
        handle = symm.rendezvous(buf, group.group_name)
        torch.cuda.synchronize()
        dist.barrier(group=group)                 # every rank zeroed its buffer before any peer writes
        ptrs = (c_void_p * len(handle.buffer_ptrs))(*handle.buffer_ptrs)
        check("moe_layer_set_peer_buffers", self._k.moe_layer_set_peer_buffers(self._h, ptrs, len(handle.buffer_ptrs)))
        self._peer = (buf, handle, ptrs)          # keep the mapping alive with the layer

    def check_error(self, stream=None):
        check("moe_layer_check_error", self._k.moe_layer_check_error(self._h, stream_ptr(stream)))

    def last_routing(self, T: int):
        """(topk_idx [T][k] int32, topk_w [T][k] f32, group counts [G]) copied to host tensors."""
        import torch
        a, b, c = c_void_p(), c_void_p(), c_void_p()
        check("moe_layer_last_routing", self._k.moe_layer_last_routing(self._h, ptr(self.workspace), ctypes.byref(a),
                                                                       ctypes.byref(b), ctypes.byref(c)))
        k = self.shape.top_k
        G = self.shape.num_experts // self.ep_size + self.shape.num_shared
        dev = self.workspace.device
        base = self.workspace.data_ptr()

        def view(p, n, dt):
            off = p.value - base
            return self.workspace[off: off + n * torch.tensor([], dtype=dt).element_size()].view(dt).clone()

        return view(a, T * k, torch.int32).view(T, k), view(b, T * k, torch.float32).view(T, k), view(c, G, torch.int32)

    def close(self):
        if getattr(self, "_h", None):
            self._k.moe_layer_destroy(self._h)
            self._h = None
        self._peer = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def grouped_gemm(mode: int, a, a_scale, a_ld: int, w, w_scale, count, start, out, out_scale, out_ld: int,
                 K: int, N: int, rows: int, error_word=None, stream=None, row_out=None):
    """cbwFp8BlockScaledGroupedGemm; with row_out (an int64 device tensor of
    [rows] output row addresses, 0 for rows that go to out) the down
    projection's cbwFp8BlockScaledGroupedGemmRowOut."""
    L = libs()
    args = GroupedGemmArgs(mode, count.numel(), K, N, rows, ptr(a), ptr(a_scale), a_ld, ptr(w), ptr(w_scale),
                           ptr(count), ptr(start), ptr(out), ptr(out_scale), out_ld)
    b = L["libcublaswrap.so"]
    if row_out is None:
        check("cbwFp8BlockScaledGroupedGemm", b.cbwFp8BlockScaledGroupedGemm(ctypes.byref(args), ptr(error_word),
                                                                            stream_ptr(stream)))
    else:
        check("cbwFp8BlockScaledGroupedGemmRowOut",
              b.cbwFp8BlockScaledGroupedGemmRowOut(ctypes.byref(args), ptr(row_out), ptr(error_word),
                                                   stream_ptr(stream)))


def router_load(shape, weights, x) -> "torch.Tensor":
    """Per-expert routed pairs of the tokens x under this router (RMSNorm +
    router logits + top-k on the device, all tokens on this GPU): the load
    statistics a balanced expert placement is computed from."""
    import torch
    k = libs()["libkernels.so"]
    dev = x.device
    T, H, E, K = x.shape[0], shape.hidden, shape.num_experts, shape.top_k
    s = torch.cuda.current_stream().cuda_stream
    rms = torch.empty(T, device=dev)
    n = torch.empty(T, H, device=dev)
    xq = torch.empty(T, H, dtype=torch.uint8, device=dev)
    ld = (T + 3) // 4 * 4
    xs = torch.empty(H // 128, ld, device=dev)
    logits = torch.empty(T, E, device=dev)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, device=dev)
    check("moe_rmsnorm_quant_n", k.moe_rmsnorm_quant_n(ptr(x), ptr(weights["gamma"]), T, H, shape.eps, ptr(rms),
                                                      ptr(n), ptr(xq), ptr(xs), ld, s))
    check("moe_router_logits", k.moe_router_logits(ptr(n), ptr(weights["router_w"]), ptr(weights.get("router_bias")),
                                                   T, H, E, ptr(logits), s))
    check("moe_topk_softmax", k.moe_topk_softmax(ptr(logits), T, E, K, ptr(idx), ptr(w), s))
    v = idx.flatten()
    return torch.bincount(v[v >= 0].long(), minlength=E).cpu()
