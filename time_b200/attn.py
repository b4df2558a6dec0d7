"""ctypes front-end of the decode-attention entry points of libkernels.so
(include/attn_block.h): partial RoPE + bf16 page write, split-context paged
flash decode (with the e4m3 1x128 output the o_proj GEMM reads), and the
fixed-order tensor-parallel sum of o_proj partials.

The reference runs this path through launch_rope / launch_update_kv_cache /
launch_paged_attention_decode (csrc/kernels.h, fp32, src/terra/engine.t:1269-1310);
those stay exported unchanged as drop-ins.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_size_t, c_void_p

import numpy as np

from . import moe as M

HEAD_DIM = 128
PAGE = 16

_bound = False


class BlockConfig(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("num_q_heads", c_int), ("num_kv_heads", c_int), ("head_dim", c_int),
                ("rotary_dim", c_int), ("rope_theta", c_float), ("eps", c_float), ("max_batch", c_int),
                ("max_pages_per_seq", c_int), ("max_context", c_int), ("tp_size", c_int), ("tp_rank", c_int)]


class BlockWeights(ctypes.Structure):
    _fields_ = [("gamma", c_void_p), ("w_qkv", c_void_p), ("s_qkv", c_void_p), ("w_o", c_void_p), ("s_o", c_void_p)]


def lib():
    global _bound
    k = M.libs()["libkernels.so"]
    if not _bound:
        k.attn_rope_kv_write.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                         c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p]
        k.attn_decode_workspace_bytes.argtypes = [c_int, c_int, c_int]
        k.attn_decode_workspace_bytes.restype = c_size_t
        k.attn_decode_paged.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int,
                                        c_int, c_int, c_int, c_float, c_int, c_int, c_void_p, c_size_t, c_void_p,
                                        c_void_p, c_void_p, c_int, c_void_p, c_void_p]
        rows_args = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int,
                     c_int, c_int, c_int, c_float, c_int, c_int, c_void_p, c_size_t, c_void_p, c_void_p, c_void_p,
                     c_int, c_void_p, c_void_p]
        k.attn_decode_paged_rows.argtypes = rows_args
        k.attn_paged_rows.argtypes = rows_args[:10] + [c_int] + rows_args[10:]
        k.attn_tp_reduce_residual.argtypes = [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]
        k.attn_block_create.argtypes = [ctypes.POINTER(BlockConfig), ctypes.POINTER(BlockWeights),
                                        ctypes.POINTER(c_void_p)]
        k.attn_block_destroy.argtypes = [c_void_p]
        k.attn_block_workspace_bytes.argtypes = [c_void_p]
        k.attn_block_workspace_bytes.restype = c_size_t
        k.attn_block_split_tokens.argtypes = [c_void_p]
        k.attn_block_peer_bytes.argtypes = [c_void_p]
        k.attn_block_peer_bytes.restype = c_size_t
        k.attn_block_set_peer_buffers.argtypes = [c_void_p, c_void_p, c_int]
        blk = [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
               c_void_p]
        k.attn_block_decode.argtypes = blk
        k.attn_block_decode_partial.argtypes = blk
        rows = [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                c_void_p, c_size_t, c_void_p]
        k.attn_block_forward.argtypes = rows
        k.attn_block_forward_partial.argtypes = rows
        k.attn_block_check_error.argtypes = [c_void_p, c_void_p]
        k.fp8_gemm_small_workspace_bytes.argtypes = [c_int, c_int, c_int]
        k.fp8_gemm_small_workspace_bytes.restype = c_size_t
        k.fp8_gemm_small.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_void_p,
                                     c_void_p, c_size_t, c_void_p]
        _bound = True
    return k


def rope_inv_freq(rot: int, theta: float) -> np.ndarray:
    """theta^(-2i/rot) for i < rot/2, computed in double and rounded once."""
    i = np.arange(rot // 2, dtype=np.float64)
    return (theta ** (-2.0 * i / rot)).astype(np.float32)


def rope_kv_write(qkv, positions, page_table, k_cache, v_cache, nq: int, nkv: int, rot: int, inv_freq,
                  error_word=None, stream=None):
    """qkv bf16 [B][(nq+2nkv)*128] -> rotated q bf16 [B][nq][128]; k, v into their page slots."""
    import torch
    B = qkv.shape[0]
    q_out = torch.empty(B, nq, HEAD_DIM, dtype=torch.bfloat16, device=qkv.device)
    M.check("attn_rope_kv_write", lib().attn_rope_kv_write(
        M.ptr(qkv), B, nq, nkv, HEAD_DIM, rot, M.ptr(inv_freq), M.ptr(positions), M.ptr(page_table),
        page_table.shape[1], PAGE, k_cache.shape[0], M.ptr(q_out), M.ptr(k_cache), M.ptr(v_cache), None,
        M.ptr(error_word), M.stream_ptr(stream)))
    return q_out


def decode_paged(q, k_cache, v_cache, page_table, seq_lens, nq: int, nkv: int, scale: float,
                 split_tokens: int = 2048, max_splits: int | None = None, quant: bool = False, workspace=None,
                 error_word=None, stream=None):
    """Paged decode attention.  Returns (out bf16 [B][nq][128], out_q e4m3 [B][nq*128] or None,
    out_s [nq][ld] or None)."""
    import torch
    B = q.shape[0]
    max_pages = page_table.shape[1]
    if max_splits is None:
        max_splits = -(-max_pages * PAGE // split_tokens)
    k = lib()
    need = k.attn_decode_workspace_bytes(B, nq, max_splits)
    if workspace is None:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    out = torch.empty(B, nq, HEAD_DIM, dtype=torch.bfloat16, device=q.device)
    out_q = out_s = None
    ld = (B + 3) // 4 * 4
    if quant:
        out_q = torch.empty(B, nq * HEAD_DIM, dtype=torch.uint8, device=q.device)
        out_s = torch.empty(nq, ld, dtype=torch.float32, device=q.device)
    M.check("attn_decode_paged", k.attn_decode_paged(
        M.ptr(q), M.ptr(k_cache), M.ptr(v_cache), k_cache.shape[0], M.ptr(page_table), max_pages, M.ptr(seq_lens), B,
        nq, nkv, HEAD_DIM, PAGE, scale, split_tokens, max_splits, M.ptr(workspace), workspace.numel(), M.ptr(out),
        M.ptr(out_q), M.ptr(out_s), ld, M.ptr(error_word), M.stream_ptr(stream)))
    return out, out_q, out_s


def paged_rows(q, k_cache, v_cache, page_table, row_seq, seq_lens, nq: int, nkv: int, scale: float,
               split_tokens: int = 2048, max_splits: int | None = None, prefill_rows: int | None = None,
               quant: bool = False, error_word=None, stream=None):
    """Attention over rows of several sequences (row r: page-table row row_seq[r], seq_lens[r] =
    position + 1).  prefill_rows=P: attn_paged_rows (rows [0, P) through the prefill kernel, the rest
    through split decode); None: attn_decode_paged_rows (split decode for all).
    Returns (out bf16 [B][nq][128], out_q or None, out_s or None)."""
    import torch
    B = q.shape[0]
    num_seqs, max_pages = page_table.shape
    if max_splits is None:
        max_splits = -(-max_pages * PAGE // split_tokens)
    k = lib()
    need = k.attn_decode_workspace_bytes(B, nq, max_splits)
    workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    out = torch.empty(B, nq, HEAD_DIM, dtype=torch.bfloat16, device=q.device)
    out_q = out_s = None
    ld = (B + 3) // 4 * 4
    if quant:
        out_q = torch.empty(B, nq * HEAD_DIM, dtype=torch.uint8, device=q.device)
        out_s = torch.empty(nq, ld, dtype=torch.float32, device=q.device)
    head = (M.ptr(q), M.ptr(k_cache), M.ptr(v_cache), k_cache.shape[0], M.ptr(page_table), max_pages,
            M.ptr(row_seq), num_seqs, M.ptr(seq_lens), B)
    tail = (nq, nkv, HEAD_DIM, PAGE, scale, split_tokens, max_splits, M.ptr(workspace), workspace.numel(),
            M.ptr(out), M.ptr(out_q), M.ptr(out_s), ld, M.ptr(error_word), M.stream_ptr(stream))
    if prefill_rows is None:
        M.check("attn_decode_paged_rows", k.attn_decode_paged_rows(*head, *tail))
    else:
        M.check("attn_paged_rows", k.attn_paged_rows(*head, prefill_rows, *tail))
    return out, out_q, out_s


def tp_reduce_residual(partials, residual, stream=None):
    """bf16(residual + sum_r partials[r]) with the ranks summed in fp32 in list order."""
    import torch
    T, H = residual.shape
    ptrs = torch.tensor([p.data_ptr() for p in partials], dtype=torch.int64, device=residual.device)
    out = torch.empty_like(residual)
    M.check("attn_tp_reduce_residual", lib().attn_tp_reduce_residual(
        M.ptr(ptrs), len(partials), M.ptr(residual), T, H, M.ptr(out), M.stream_ptr(stream)))
    torch.cuda.current_stream().synchronize() if stream is None else stream.synchronize()
    return out


class AttnBlock:
    """One TP rank of the decode attention block (include/attn_block.h).
    `weights`: the rank's slice (synth.attn_rank_slice) as device tensors."""

    def __init__(self, shape, weights: dict, max_batch: int, max_pages_per_seq: int, max_context: int,
                 tp_size: int = 1, tp_rank: int = 0):
        import torch
        self._h = None
        self.shape, self.tp_size, self.tp_rank = shape, tp_size, tp_rank
        self.nq, self.nkv = shape.num_q_heads // tp_size, shape.num_kv_heads // tp_size
        self._w = weights
        self._k = lib()
        cfg = BlockConfig(shape.hidden, self.nq, self.nkv, shape.head_dim, shape.rotary_dim, shape.rope_theta,
                          shape.eps, max_batch, max_pages_per_seq, max_context, tp_size, tp_rank)
        wts = BlockWeights(*(M.ptr(weights[n]) for n in ("gamma", "w_qkv", "s_qkv", "w_o", "s_o")))
        h = c_void_p()
        M.check("attn_block_create", self._k.attn_block_create(ctypes.byref(cfg), ctypes.byref(wts), ctypes.byref(h)))
        self._h = h
        dev = weights["w_qkv"].device
        self.workspace = torch.empty(self._k.attn_block_workspace_bytes(h), dtype=torch.uint8, device=dev)
        self.split_tokens = self._k.attn_block_split_tokens(h)
        self._peer = None

    def use_peer_memory(self, group=None):
        """tp > 1: allocate the peer-visible partial buffers with torch symmetric memory."""
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        nbytes = self._k.attn_block_peer_bytes(self._h)
        buf = symm.empty(nbytes, dtype=torch.uint8, device=self.workspace.device)
        buf.zero_()
        torch.cuda.synchronize()
        handle = symm.rendezvous(buf, group if group is not None else dist.group.WORLD)
        dist.barrier(group=group)
        ptrs = (c_void_p * self.tp_size)(*[handle.buffer_ptrs[r] for r in range(self.tp_size)])
        M.check("attn_block_set_peer_buffers", self._k.attn_block_set_peer_buffers(self._h, ptrs, self.tp_size))
        self._peer = (buf, handle, ptrs)

    def _call(self, fn, x, positions, page_table, k_cache, v_cache, out, stream):
        M.check(fn.__name__, fn(self._h, M.ptr(x), x.shape[0], M.ptr(positions), M.ptr(page_table), k_cache.shape[0],
                                M.ptr(k_cache), M.ptr(v_cache), M.ptr(out), M.ptr(self.workspace),
                                self.workspace.numel(), M.stream_ptr(stream)))
        return out

    def decode(self, x, positions, page_table, k_cache, v_cache, out=None, stream=None):
        import torch
        out = torch.empty_like(x) if out is None else out
        return self._call(self._k.attn_block_decode, x, positions, page_table, k_cache, v_cache, out, stream)

    def decode_partial(self, x, positions, page_table, k_cache, v_cache, out=None, stream=None):
        import torch
        out = torch.empty_like(x) if out is None else out
        return self._call(self._k.attn_block_decode_partial, x, positions, page_table, k_cache, v_cache, out, stream)

    def forward(self, x, positions, row_seq, page_table, k_cache, v_cache, out=None, partial=False, stream=None):
        """Rows of several sequences (prefill chunks, slot-indexed batches):
        row r is the token at positions[r] of page-table row row_seq[r]."""
        import torch
        out = torch.empty_like(x) if out is None else out
        fn = self._k.attn_block_forward_partial if partial else self._k.attn_block_forward
        M.check(fn.__name__, fn(self._h, M.ptr(x), x.shape[0], M.ptr(positions), M.ptr(row_seq), page_table.shape[0],
                                M.ptr(page_table), k_cache.shape[0], M.ptr(k_cache), M.ptr(v_cache), M.ptr(out),
                                M.ptr(self.workspace), self.workspace.numel(), M.stream_ptr(stream)))
        return out

    def check_error(self, stream=None):
        M.check("attn_block_check_error", self._k.attn_block_check_error(self._h, M.stream_ptr(stream)))

    def close(self):
        if self._h:
            self._k.attn_block_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

