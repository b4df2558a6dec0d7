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


def lib():
    global _bound
    k = M.libs()["libkernels.so"]
    if not _bound:
        k.attn_rope_kv_write.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                         c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
        k.attn_decode_workspace_bytes.argtypes = [c_int, c_int, c_int]
        k.attn_decode_workspace_bytes.restype = c_size_t
        k.attn_decode_paged.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int,
                                        c_int, c_int, c_int, c_float, c_int, c_int, c_void_p, c_size_t, c_void_p,
                                        c_void_p, c_void_p, c_int, c_void_p, c_void_p]
        k.attn_tp_reduce_residual.argtypes = [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]
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
        page_table.shape[1], PAGE, k_cache.shape[0], M.ptr(q_out), M.ptr(k_cache), M.ptr(v_cache), M.ptr(error_word),
        M.stream_ptr(stream)))
    return q_out


def decode_paged(q, k_cache, v_cache, page_table, seq_lens, nq: int, nkv: int, scale: float,
                 split_tokens: int = 512, max_splits: int | None = None, quant: bool = False, workspace=None,
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
