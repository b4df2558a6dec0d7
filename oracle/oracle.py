"""ctypes front-end of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's CPU-baseline leg.  The product never imports
it.  See moe_oracle.h for the semantics and the reference lines each function
restates.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_KERNELS = HERE / "_ref" / "libref_kernels.so"

_lib = None

f32p = ctypes.POINTER(ctypes.c_float)
i32p = ctypes.POINTER(ctypes.c_int32)
u8p = ctypes.POINTER(ctypes.c_uint8)
u16p = ctypes.POINTER(ctypes.c_uint16)


class MoeCfg(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("num_experts", ctypes.c_int), ("top_k", ctypes.c_int),
                ("intermediate", ctypes.c_int), ("num_shared", ctypes.c_int), ("eps", ctypes.c_float)]


class MoeWeights(ctypes.Structure):
    _fields_ = [("gamma", f32p), ("router_w", f32p), ("router_bias", f32p), ("w13", u8p), ("s13", f32p),
                ("w2", u8p), ("s2", f32p)]


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)
        L = ctypes.CDLL(str(LIB))
        L.orc_e4m3_decode_ref.restype = ctypes.c_float
        L.orc_e4m3_decode_ref.argtypes = [ctypes.c_uint8]
        L.orc_e4m3_decode.restype = ctypes.c_float
        L.orc_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.orc_e4m3_encode_ref.restype = ctypes.c_uint8
        L.orc_e4m3_encode_ref.argtypes = [ctypes.c_float]
        L.orc_e4m3_encode_rne.restype = ctypes.c_uint8
        L.orc_e4m3_encode_rne.argtypes = [ctypes.c_float]
        L.orc_bf16_to_f32.restype = ctypes.c_float
        L.orc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_rmsnorm_ref.argtypes = [f32p, f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_rms_ref.argtypes = [f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_moe_gate_ref.argtypes = [f32p, f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_moe_router_logits.argtypes = [f32p, f32p, f32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_moe_topk_ref.argtypes = [f32p, i32p, f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_moe_permute.restype = ctypes.c_int
        L.orc_moe_permute.argtypes = [i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      i32p, i32p, i32p, i32p, ctypes.c_int]
        L.orc_quant_row_1x128.argtypes = [f32p, ctypes.c_int, u8p, f32p]
        L.orc_quant_row_1x128_x2.argtypes = [f32p, ctypes.c_int, u8p, u8p, f32p]
        L.orc_moe_ffn_forward.argtypes = [ctypes.POINTER(MoeCfg), ctypes.POINTER(MoeWeights), u16p, u16p,
                                          ctypes.c_int, ctypes.c_int, i32p, f32p, f32p, ctypes.c_int]
        L.orc_moe_ffn_experts.argtypes = [ctypes.POINTER(MoeCfg), ctypes.POINTER(MoeWeights), u16p, i32p, f32p,
                                          u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_gemm_fp8_block.argtypes = [u8p, f32p, ctypes.c_int, u8p, f32p, ctypes.c_int, ctypes.c_int, f32p]
        L.orc_rope_inv_freq.argtypes = [ctypes.c_int, ctypes.c_float, f32p]
        L.orc_rope_partial.argtypes = [f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, f32p]
        L.orc_attn_decode_paged.argtypes = [f32p, f32p, f32p, i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_float, f32p]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- scalars

def e4m3_decode_ref(b: int) -> float:
    return lib().orc_e4m3_decode_ref(b)


def e4m3_decode(b: int) -> float:
    return lib().orc_e4m3_decode(b)


def e4m3_encode_ref(x: float) -> int:
    return lib().orc_e4m3_encode_ref(x)


def e4m3_encode_rne(x: float) -> int:
    return lib().orc_e4m3_encode_rne(x)


def e4m3_encode_rne_array(x: np.ndarray) -> np.ndarray:
    f = np.vectorize(lambda v: lib().orc_e4m3_encode_rne(float(v)), otypes=[np.uint8])
    return f(np.asarray(x, dtype=np.float32))


def decode_table(ref: bool = False) -> np.ndarray:
    fn = lib().orc_e4m3_decode_ref if ref else lib().orc_e4m3_decode
    return np.array([fn(b) for b in range(256)], dtype=np.float32)


def bf16_bits_to_f32(u: np.ndarray) -> np.ndarray:
    return (np.asarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# ---------------------------------------------------------------- kernels

def rmsnorm_ref(x: np.ndarray, gamma: np.ndarray, eps: float) -> np.ndarray:
    x = _f32(x)
    T, H = x.shape
    out = np.empty_like(x)
    lib().orc_rmsnorm_ref(_p(x, f32p), _p(_f32(gamma), f32p), _p(out, f32p), H, T, eps)
    return out


def rms_ref(x: np.ndarray, eps: float) -> np.ndarray:
    x = _f32(x)
    T, H = x.shape
    out = np.empty(T, np.float32)
    lib().orc_rms_ref(_p(x, f32p), _p(out, f32p), H, T, eps)
    return out


def moe_gate_ref(h: np.ndarray, w: np.ndarray, bias=None) -> np.ndarray:
    """Router logits in the reference's order (csrc/kernels.cu:412-435); with
    `bias`, the MoE layer's routing bias added to each logit after the tree."""
    h, w = _f32(h), _f32(w)
    T, H = h.shape
    E = w.shape[0]
    out = np.empty((T, E), np.float32)
    if bias is None:
        lib().orc_moe_gate_ref(_p(h, f32p), _p(w, f32p), _p(out, f32p), H, E, T)
    else:
        b = _f32(bias)
        lib().orc_moe_router_logits(_p(h, f32p), _p(w, f32p), _p(b, f32p), _p(out, f32p), H, E, T)
    return out


def moe_topk_ref(logits: np.ndarray, k: int):
    logits = _f32(logits)
    T, E = logits.shape
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lib().orc_moe_topk_ref(_p(logits, f32p), _p(idx, i32p), _p(w, f32p), E, k, T)
    return idx, w


def moe_permute(idx: np.ndarray, num_experts: int, num_shared: int, pad: int = 16):
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    T, k = idx.shape
    G = num_experts + num_shared
    cap = T * k + num_shared * T + pad * G
    counts = np.empty(G, np.int32)
    start = np.empty(G, np.int32)
    pos = np.empty(T * k, np.int32)
    row_token = np.empty(cap, np.int32)
    R = lib().orc_moe_permute(_p(idx, i32p), T, k, num_experts, num_shared, pad, _p(counts, i32p), _p(start, i32p),
                              _p(pos, i32p), _p(row_token, i32p), cap)
    return counts, start, pos.reshape(T, k), row_token[:R], R


def quant_rows_1x128(v: np.ndarray):
    v = _f32(v)
    rows, cols = v.shape
    q = np.empty((rows, cols), np.uint8)
    s = np.empty((rows, cols // 128), np.float32)
    for r in range(rows):
        lib().orc_quant_row_1x128(_p(v[r], f32p), cols, _p(q[r], u8p), _p(s[r], f32p))
    return q, s


def quant_rows_1x128_x2(v: np.ndarray):
    """Two-term 1x128 quantisation: (hi bytes, lo bytes, scales)."""
    v = _f32(v)
    rows, cols = v.shape
    q = np.empty((rows, cols), np.uint8)
    ql = np.empty((rows, cols), np.uint8)
    s = np.empty((rows, cols // 128), np.float32)
    for r in range(rows):
        lib().orc_quant_row_1x128_x2(_p(v[r], f32p), cols, _p(q[r], u8p), _p(ql[r], u8p), _p(s[r], f32p))
    return q, ql, s


class OracleWeights:
    """numpy copies of the weights + the ctypes structs pointing at them."""

    def __init__(self, shape, w: dict):
        self.cfg = MoeCfg(shape.hidden, shape.num_experts, shape.top_k, shape.intermediate, shape.num_shared,
                          shape.eps)

        def arr(t, dt):
            if t is None:
                return None
            a = t.detach().cpu().numpy() if hasattr(t, "detach") else np.asarray(t)
            return np.ascontiguousarray(a, dtype=dt)

        self.gamma = arr(w["gamma"], np.float32)
        self.router_w = arr(w["router_w"], np.float32)
        self.router_bias = arr(w.get("router_bias"), np.float32)
        self.w13 = arr(w["w13"], np.uint8)
        self.s13 = arr(w["s13"], np.float32)
        self.w2 = arr(w["w2"], np.uint8)
        self.s2 = arr(w["s2"], np.float32)
        self.st = MoeWeights(_p(self.gamma, f32p), _p(self.router_w, f32p),
                             _p(self.router_bias, f32p) if self.router_bias is not None else None,
                             _p(self.w13, u8p), _p(self.s13, f32p), _p(self.w2, u8p), _p(self.s2, f32p))


def moe_ffn_forward(ow: OracleWeights, x_bf16_bits: np.ndarray, mode: int = 0, threads: int = 0):
    """Full MoE FFN block.  x as bf16 bit patterns (uint16) [T][H].
    Returns (out bf16 bits [T][H], idx [T][k], weights [T][k], logits [T][E])."""
    x = np.ascontiguousarray(x_bf16_bits, dtype=np.uint16)
    T, H = x.shape
    k, E = ow.cfg.top_k, ow.cfg.num_experts
    out = np.empty_like(x)
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lg = np.empty((T, E), np.float32)
    lib().orc_moe_ffn_forward(ctypes.byref(ow.cfg), ctypes.byref(ow.st), _p(x, u16p), _p(out, u16p), T, mode,
                              _p(idx, i32p), _p(w, f32p), _p(lg, f32p), threads)
    return out, idx, w, lg


def moe_ffn_experts(ow: OracleWeights, x_bf16_bits: np.ndarray, idx: np.ndarray, w: np.ndarray, mode: int = 0,
                    threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16_bits, dtype=np.uint16)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T = x.shape[0]
    out = np.empty_like(x)
    lib().orc_moe_ffn_experts(ctypes.byref(ow.cfg), ctypes.byref(ow.st), _p(x, u16p), _p(idx, i32p), _p(w, f32p),
                              _p(out, u16p), T, mode, threads)
    return out


def max_rel_and_mae(y: np.ndarray, ref: np.ndarray):
    """The north-star tolerance metrics: max|y-ref| / max|ref| and mean|y-ref|."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(y - ref)
    return float(d.max() / max(np.abs(ref).max(), 1e-30)), float(d.mean())


# ---------------------------------------------------------------- decode attention (attn_oracle.c)

def gemm_fp8_block(xq: np.ndarray, xs: np.ndarray, w: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """out [rows][N] = block-scaled FP8 projection (xs [rows][K/128], ws [N/128][K/128])."""
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    rows, K = xq.shape
    N = w.shape[0]
    xs, ws = _f32(xs), _f32(ws)
    out = np.empty((rows, N), dtype=np.float32)
    lib().orc_gemm_fp8_block(_p(xq, u8p), _p(xs, f32p), rows, _p(w, u8p), _p(ws, f32p), N, K, _p(out, f32p))
    return out


def rope_inv_freq(rot: int, theta: float) -> np.ndarray:
    out = np.empty(rot // 2, dtype=np.float32)
    lib().orc_rope_inv_freq(rot, theta, _p(out, f32p))
    return out


def rope_partial(x: np.ndarray, rot: int, pos: int, inv_freq: np.ndarray) -> np.ndarray:
    """x [heads][d] fp32 -> rotated copy (first `rot` dims, rotate-half)."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    heads, d = y.shape
    f = _f32(inv_freq)
    lib().orc_rope_partial(_p(y, f32p), heads, d, rot, pos, _p(f, f32p))
    return y


def attn_decode_paged(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, page_table: np.ndarray, seq_len: int,
                      scale: float) -> np.ndarray:
    """One sequence: q [nq][d], caches [pages][page_size][nkv][d] (fp32), page_table [pages_of_seq]."""
    q, kc, vc = _f32(q), _f32(k_cache), _f32(v_cache)
    pt = np.ascontiguousarray(page_table, dtype=np.int32)
    nq, d = q.shape
    _, ps, nkv, _ = kc.shape
    out = np.empty((nq, d), dtype=np.float32)
    lib().orc_attn_decode_paged(_p(q, f32p), _p(kc, f32p), _p(vc, f32p), _p(pt, i32p), seq_len, nq, nkv, d, ps,
                                scale, _p(out, f32p))
    return out



def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(_f32(x)))


def attn_block_partial_ref(w: dict, x: np.ndarray, positions, page_table: np.ndarray, k_cache: np.ndarray,
                           v_cache: np.ndarray, nq: int, nkv: int, rot: int, theta: float, eps: float) -> np.ndarray:
    """One TP rank's decode-attention partial with the kernels' rounding points:
    rmsnorm -> e4m3 1x128 -> QKV (bf16) -> partial RoPE (bf16) -> K/V written
    into the fp32 copies of the rank's caches (in place) -> decode attention
    over pos + 1 tokens -> e4m3 1x128 -> o_proj (bf16).  w: numpy gamma, w_qkv,
    s_qkv, w_o, s_o; x: [B][H] fp32 holding bf16 values."""
    d = 128
    n = rmsnorm_ref(x, w["gamma"], eps)
    q8, s8 = quant_rows_1x128(n)
    qkv = bf16_round(gemm_fp8_block(q8, s8, w["w_qkv"], w["s_qkv"]))
    inv = rope_inv_freq(rot, theta)
    B = x.shape[0]
    qs = []
    for b in range(B):
        pos = int(positions[b])
        r = bf16_round(rope_partial(qkv[b, :(nq + nkv) * d].reshape(nq + nkv, d), rot, pos, inv))
        page, slot = page_table[b, pos // 16], pos % 16
        k_cache[page, slot] = r[nq:]
        v_cache[page, slot] = qkv[b, (nq + nkv) * d:].reshape(nkv, d)
        qs.append(r[:nq])
    attn = np.stack([attn_decode_paged(qs[b], k_cache, v_cache, page_table[b], int(positions[b]) + 1,
                                       1.0 / np.sqrt(d)).reshape(nq * d) for b in range(B)])
    aq, as_ = quant_rows_1x128(attn)
    return bf16_round(gemm_fp8_block(aq, as_, w["w_o"], w["s_o"]))


# ---------------------------------------------------------------- serving engine (composition)

class EngineRef:
    """CPU restatement of the serving engine's forward (include/engine.h),
    composed from the functions above with the engine's rounding points:
    embedding rows (bf16 values) -> per layer the attention block
    (attn_block_partial_ref, tp 1) and bf16(x + partial) -> the FFN block
    (moe_ffn_experts, mode 0: RMSNorm, experts, shared expert, residual; a
    dense layer is one expert with weight 1.0) -> final RMSNorm in double,
    rounded to bf16 -> lm_head (bf16 weights, double dot products) -> fp32
    logits.  The reference's layer sequence is src/terra/engine.t:1235-1371
    (run_layer_forward_gpu) and its head engine.t:1432-1445.

    layers: per layer {"attn": numpy gamma / w_qkv / s_qkv / w_o / s_o (the
    tp 1 rank layout), "ffn": OracleWeights, "dense": bool}.  K/V caches are
    fp32 copies [num_pages][16][nkv][128] per layer, written by forward()."""

    def __init__(self, layers, embed, final_norm, lm_head, nq: int, nkv: int, rot: int, theta: float, eps: float,
                 num_pages: int):
        self.layers = layers
        self.embed = np.asarray(embed, dtype=np.float32)
        self.final_norm = np.asarray(final_norm, dtype=np.float64)
        self.lm_head = np.asarray(lm_head, dtype=np.float64)
        self.nq, self.nkv, self.rot, self.theta, self.eps = nq, nkv, rot, theta, eps
        self.k = [np.zeros((num_pages, 16, nkv, 128), np.float32) for _ in layers]
        self.v = [np.zeros((num_pages, 16, nkv, 128), np.float32) for _ in layers]

    def forward(self, tokens, positions, page_rows: np.ndarray, routing=None, logits: bool = False,
                own_routing: list | None = None):
        """Rows = tokens at positions (page_rows [R][max_pages]: each row's page
        table).  routing: per layer (idx [R][k], w [R][k]) to evaluate the
        experts with (None for dense layers), or None to route here.
        own_routing, when a list: receives per MoE layer this oracle's own
        (idx, w, logits) for the same inputs.  Returns fp32 logits [R][V] or None."""
        x = self.embed[np.asarray(tokens, dtype=np.int64)].astype(np.float32)
        positions = np.asarray(positions, dtype=np.int64)
        R = x.shape[0]
        for l, L in enumerate(self.layers):
            part = attn_block_partial_ref(L["attn"], x, positions, page_rows, self.k[l], self.v[l], self.nq,
                                          self.nkv, self.rot, self.theta, self.eps)
            x = bf16_round(x + part)
            xb = f32_to_bf16_bits(x)
            if L["dense"]:
                out = moe_ffn_experts(L["ffn"], xb, np.zeros((R, 1), np.int32), np.ones((R, 1), np.float32))
            else:
                if own_routing is not None or routing is None:
                    _, idx, w, lg = moe_ffn_forward(L["ffn"], xb, mode=0)
                    if own_routing is not None:
                        own_routing.append((idx, w, lg))
                if routing is not None:
                    idx, w = routing[l]
                out = moe_ffn_experts(L["ffn"], xb, idx, w, mode=0)
            x = bf16_bits_to_f32(out)
        if not logits:
            return None
        x64 = x.astype(np.float64)
        inv = 1.0 / np.sqrt((x64 * x64).mean(axis=1, keepdims=True) + self.eps)
        xn = bf16_round((x64 * inv * self.final_norm).astype(np.float32)).astype(np.float64)
        return (xn @ self.lm_head.T).astype(np.float32)
