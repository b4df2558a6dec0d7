"""Generate tests/golden/ref_kernels.npz: outputs of the REFERENCE's own CUDA
kernels (csrc/kernels.cu of kollarsandor/time, compiled unmodified by
`make -C oracle ref` into oracle/_ref/libref_kernels.so) on seeded inputs.

Run on a machine with a GPU and the built oracle/_ref library:

    python tests/golden/make_ref_golden.py [--out tests/golden/ref_kernels.npz]

The fixture pins the CPU oracle (tests/test_golden_ref.py, no GPU) and this
package's drop-in launch_* kernels (tests/test_gpu_legacy.py) to the
reference itself.  Inputs are stored beside the outputs, so the tests never
need the reference or this script.  Kernels covered (reference
csrc/kernels.h:12-31): fp8_dequantize, f32_to_fp8, rms_norm, moe_gate,
moe_topk, swiglu, moe_combine, add_residual, argmax, rope; into
tests/golden/ref_attn.npz paged_attention_decode and update_kv_cache
(`--only attn` writes just that file); and into tests/golden/ref_legacy.npz
softmax, gelu, embedding_lookup (e4m3 / fp16 / fp32 tables), top_p_sampling
(sampling and argmax paths), apply_rep_penalty, paged_attention_prefill,
moe_dispatch and copy_hidden (`--only legacy`).
"""
from __future__ import annotations

import argparse
import ctypes
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
c_int, c_float, c_size_t, c_void_p = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p


def load_ref():
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_kernels.so"))
    lib.launch_fp8_dequantize.argtypes = [c_void_p, c_void_p, c_size_t, c_void_p]
    lib.launch_f32_to_fp8.argtypes = [c_void_p, c_void_p, c_size_t, c_void_p]
    lib.launch_rms_norm.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]
    lib.launch_moe_gate.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]
    lib.launch_moe_topk.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]
    lib.launch_swiglu.argtypes = [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]
    lib.launch_moe_combine.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]
    lib.launch_add_residual.argtypes = [c_void_p, c_void_p, c_size_t, c_void_p]
    lib.launch_argmax.argtypes = [c_void_p, c_void_p, c_int, c_int, c_void_p]
    lib.launch_rope.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_float, c_void_p]
    lib.launch_paged_attention_decode.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                                  c_int, c_int, c_int, c_int, c_float, c_void_p]
    lib.launch_update_kv_cache.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                           c_int, c_int, c_void_p]
    lib.launch_softmax.argtypes = [c_void_p, c_int, c_int, c_void_p]
    lib.launch_gelu.argtypes = [c_void_p, c_size_t, c_void_p]
    lib.launch_embedding_lookup.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]
    lib.launch_top_p_sampling.argtypes = [c_void_p, c_void_p, c_float, c_float, c_int, c_int, c_void_p, c_void_p]
    lib.launch_apply_rep_penalty.argtypes = [c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]
    lib.launch_paged_attention_prefill.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                                   c_int, c_int, c_int, c_float, c_void_p]
    lib.launch_moe_dispatch.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]
    lib.launch_copy_hidden.argtypes = [c_void_p, c_void_p, c_size_t, c_void_p]
    return lib


_KEEP = []


def dev(a: np.ndarray) -> torch.Tensor:
    """Device copy that stays alive until the end of the run: a temporary
    freed right after .data_ptr() could be handed to the next copy by the
    caching allocator before the asynchronous kernel has read it."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def attn_goldens(lib, out_path: str) -> None:
    """tests/golden/ref_attn.npz: the reference's paged decode attention
    (kernels.cu:328-392, one sequence per call, caches [page][16][nkv][d] fp32)
    on GQA cases with shuffled page tables, and its KV-cache scatter
    (kernels.cu:394-410)."""
    rng = np.random.default_rng(20261202)
    st = None
    g = {}
    cases = [(8, 2, 64, 77, 12), (12, 1, 128, 300, 24), (4, 4, 128, 16, 3), (16, 2, 128, 1000, 70)]
    for ci, (nq, nkv, d, past, pages) in enumerate(cases):
        ps = 16
        q = rng.standard_normal((nq, d)).astype(np.float32)
        kc = rng.standard_normal((pages, ps, nkv, d)).astype(np.float32)
        vc = rng.standard_normal((pages, ps, nkv, d)).astype(np.float32)
        pt = rng.permutation(pages)[: (past + ps - 1) // ps].astype(np.int32)
        out = torch.zeros(nq, d, device="cuda")
        scale = float(1.0 / np.sqrt(d))
        lib.launch_paged_attention_decode(dev(q).data_ptr(), dev(kc).data_ptr(), dev(vc).data_ptr(), out.data_ptr(),
                                          dev(pt).data_ptr(), len(pt), ps, nq, nkv, d, past, scale, st)
        for name, v in (("q", q), ("k", kc), ("v", vc), ("pt", pt), ("out", host(out))):
            g[f"attn{ci}_{name}"] = v
        g[f"attn{ci}_shape"] = np.array([nq, nkv, d, past, ps], dtype=np.int32)
        g[f"attn{ci}_scale"] = np.array([scale], dtype=np.float32)
    # KV scatter: 5 tokens at start_pos 13 (crossing a page), 2 kv heads
    S_, nkv, d, ps, pages = 5, 2, 64, 16, 4
    k = rng.standard_normal((S_, nkv, d)).astype(np.float32)
    v = rng.standard_normal((S_, nkv, d)).astype(np.float32)
    pt = np.array([2, 0, 3, 1], dtype=np.int32)
    kc = torch.zeros(pages, ps, nkv, d, device="cuda")
    vc = torch.zeros(pages, ps, nkv, d, device="cuda")
    lib.launch_update_kv_cache(dev(k).data_ptr(), dev(v).data_ptr(), kc.data_ptr(), vc.data_ptr(), dev(pt).data_ptr(),
                               ps, nkv, d, S_, 13, st)
    g["kvw_k"], g["kvw_v"], g["kvw_pt"] = k, v, pt
    g["kvw_kc"], g["kvw_vc"] = host(kc), host(vc)
    np.savez_compressed(out_path, **g)
    print(f"wrote {out_path}: {len(g)} arrays")


def legacy_goldens(lib, out_path: str) -> None:
    """tests/golden/ref_legacy.npz: the remaining drop-in kernels.  Inputs stay
    inside what the reference's kernels handle: token ids and past tokens
    within the vocabulary (out-of-range past tokens are skipped by the
    reference's own bounds check), no duplicate past tokens (the reference's
    in-place penalty races on duplicates), prefill chunks of at most 1024
    positions (its score buffer) whose every query has a positive score
    (k correlated with q: the reference's float max through an integer
    atomicMax is exact only then)."""
    rng = np.random.default_rng(20261203)
    st = None
    g = {}
    # softmax (in place), rows of varied scale and length
    for B, L in ((4, 1000), (3, 77), (2, 5000)):
        x = (rng.standard_normal((B, L)) * np.array([[1.0], [10.0], [0.1], [3.0]][:B])).astype(np.float32)
        t = dev(x)
        lib.launch_softmax(t.data_ptr(), B, L, st)
        g[f"softmax_in_{L}"], g[f"softmax_out_{L}"] = x, host(t)
    # gelu (in place)
    x = (4 * rng.standard_normal(5000)).astype(np.float32)
    t = dev(x)
    lib.launch_gelu(t.data_ptr(), x.size, st)
    g["gelu_in"], g["gelu_out"] = x, host(t)
    # embedding lookup: e4m3, fp16 and fp32 tables
    V, H, T = 50, 384, 9
    ids = rng.integers(0, V, T).astype(np.int64)
    ids[0], ids[1] = 0, V - 1
    tabs = {1: rng.integers(0, 256, (V, H)).astype(np.uint8),
            2: rng.standard_normal((V, H)).astype(np.float16),
            0: rng.standard_normal((V, H)).astype(np.float32)}
    g["embed_ids"] = ids
    for dt, tab in tabs.items():
        o = torch.empty(T, H, device="cuda")
        lib.launch_embedding_lookup(dev(tab).data_ptr(), dev(ids).data_ptr(), o.data_ptr(), H, T, dt, st)
        g[f"embed_tab_{dt}"], g[f"embed_out_{dt}"] = tab, host(o)
    # top-p sampling: the sampling path (temperature 0.7, top_p 0.9 and 1.0) and
    # the argmax path (temperature < 0.01)
    B, Vv = 6, 3000
    lg = (2 * rng.standard_normal((B, Vv))).astype(np.float32)
    lg[3, 123] = 15.0
    seeds = rng.integers(0, 2 ** 63, B, dtype=np.int64).astype(np.uint64)
    g["topp_logits"], g["topp_seeds"] = lg, seeds
    for name, temp, tp in (("a", 0.7, 0.9), ("b", 1.3, 1.0), ("c", 0.001, 0.9)):
        o = torch.empty(B, dtype=torch.int64, device="cuda")
        lib.launch_top_p_sampling(dev(lg).data_ptr(), o.data_ptr(), temp, tp, Vv, B, dev(seeds).data_ptr(), st)
        g[f"topp_out_{name}"] = host(o)
        g[f"topp_args_{name}"] = np.array([temp, tp], np.float32)
    # repetition penalty (in place): positive and negative logits, ids out of range skipped
    Vv = 1000
    lg = rng.standard_normal(Vv).astype(np.float32)
    past = np.concatenate([rng.choice(Vv, 300, replace=False), [-1, Vv, Vv + 7]]).astype(np.int64)
    t = dev(lg)
    lib.launch_apply_rep_penalty(t.data_ptr(), dev(past).data_ptr(), past.size, Vv, 1.3, st)
    g["rep_logits"], g["rep_past"], g["rep_out"] = lg, past, host(t)
    # paged attention prefill: causal attention over the chunk, [seq][heads][d]
    for ci, (S_, NH, D) in enumerate(((37, 4, 64), (300, 2, 128))):
        q = rng.standard_normal((S_, NH, D)).astype(np.float32)
        k = (q + 0.3 * rng.standard_normal((S_, NH, D))).astype(np.float32)
        v = rng.standard_normal((S_, NH, D)).astype(np.float32)
        pt = np.arange(4, dtype=np.int32)
        o = torch.zeros(S_, NH, D, device="cuda")
        scale = float(1.0 / np.sqrt(D))
        lib.launch_paged_attention_prefill(dev(q).data_ptr(), dev(k).data_ptr(), dev(v).data_ptr(), o.data_ptr(),
                                           dev(pt).data_ptr(), 4, 16, NH, D, S_, scale, st)
        for name, val in (("q", q), ("k", k), ("v", v), ("out", host(o))):
            g[f"prefill{ci}_{name}"] = val
        g[f"prefill{ci}_scale"] = np.array([scale], np.float32)
    # moe_dispatch: every token replicated top_k times
    T, K, H = 7, 3, 200
    x = rng.standard_normal((T, H)).astype(np.float32)
    idx = rng.integers(0, 8, (T, K)).astype(np.int32)
    o = torch.full((T, K, H), float("nan"), device="cuda")
    lib.launch_moe_dispatch(dev(x).data_ptr(), o.data_ptr(), dev(idx).data_ptr(), H, K, T, st)
    g["dispatch_in"], g["dispatch_idx"], g["dispatch_out"] = x, idx, host(o)
    # copy_hidden
    x = rng.standard_normal(3001).astype(np.float32)
    o = torch.full((3001,), float("nan"), device="cuda")
    lib.launch_copy_hidden(dev(x).data_ptr(), o.data_ptr(), 3001, st)
    g["copy_in"], g["copy_out"] = x, host(o)
    np.savez_compressed(out_path, **g)
    print(f"wrote {out_path}: {len(g)} arrays")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(ROOT / "tests" / "golden" / "ref_kernels.npz"))
    ap.add_argument("--attn-out", default=str(ROOT / "tests" / "golden" / "ref_attn.npz"))
    ap.add_argument("--legacy-out", default=str(ROOT / "tests" / "golden" / "ref_legacy.npz"))
    ap.add_argument("--only", choices=["all", "kernels", "attn", "legacy"], default="all")
    a = ap.parse_args()
    lib = load_ref()
    if a.only in ("all", "legacy"):
        legacy_goldens(lib, a.legacy_out)
    if a.only == "legacy":
        return 0
    if a.only in ("all", "attn"):
        attn_goldens(lib, a.attn_out)
    if a.only == "attn":
        return 0
    rng = np.random.default_rng(20261201)
    st = None   # legacy default stream, as the reference engine passes its context stream
    g = {}

    # fp8 decode: every code
    codes = np.arange(256, dtype=np.uint8)
    out = torch.empty(256, dtype=torch.float32, device="cuda")
    lib.launch_fp8_dequantize(dev(codes).data_ptr(), out.data_ptr(), 256, st)
    g["dequant_in"], g["dequant_out"] = codes, host(out)

    # fp8 encode: the reference test's values, specials, a log-uniform sweep and
    # all rounding midpoints between adjacent e4m3 values
    pos = np.array([0.0, 1.0, 0.5, 2.0, 0.125, 100.0, 448.0, 464.0, 500.0, 1e6, 2.0 ** -6, 2.0 ** -9, 2.0 ** -10,
                    1e-30, 3.0, 7.5, 0.3, 240.0, 0.001953125], dtype=np.float32)
    sweep = (np.exp(rng.uniform(np.log(1e-4), np.log(600.0), 4000)) * rng.choice([-1, 1], 4000)).astype(np.float32)
    dec = host(out)
    finite = np.sort(np.unique(dec[np.isfinite(dec) & (dec >= 0)]))
    mids = ((finite[1:] + finite[:-1]) / 2).astype(np.float32)
    enc_in = np.concatenate([pos, -pos, np.array([np.inf, -np.inf, np.nan], np.float32), sweep, mids, -mids])
    enc_out = torch.empty(enc_in.size, dtype=torch.uint8, device="cuda")
    lib.launch_f32_to_fp8(dev(enc_in).data_ptr(), enc_out.data_ptr(), enc_in.size, st)
    g["encode_in"], g["encode_out"] = enc_in, host(enc_out)

    # rms_norm: rows of varied scale, hidden 512 and 5120
    for H, T in ((512, 8), (5120, 4)):
        x = (rng.standard_normal((T, H)) * np.exp(rng.standard_normal((T, 1)))).astype(np.float32)
        gam = (1.0 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        o = torch.empty(T, H, dtype=torch.float32, device="cuda")
        lib.launch_rms_norm(dev(x).data_ptr(), dev(gam).data_ptr(), o.data_ptr(), H, T, 1e-5, st)
        g[f"rms_x_{H}"], g[f"rms_gamma_{H}"], g[f"rms_out_{H}"] = x, gam, host(o)

    # moe_gate: router logits (gate dtype argument ignored by the reference)
    for H, E, T in ((512, 64, 16), (5120, 160, 4)):
        x = rng.standard_normal((T, H)).astype(np.float32)
        W = (0.02 * rng.standard_normal((E, H))).astype(np.float32)
        o = torch.empty(T, E, dtype=torch.float32, device="cuda")
        lib.launch_moe_gate(dev(x).data_ptr(), dev(W).data_ptr(), o.data_ptr(), H, E, T, 4, st)
        g[f"gate_x_{H}_{E}"], g[f"gate_w_{H}_{E}"], g[f"gate_out_{H}_{E}"] = x, W, host(o)

    # moe_topk: ties, NaN and large logits included
    T, E, K = 64, 160, 8
    lg = rng.standard_normal((T, E)).astype(np.float32)
    lg[1, :] = 0.5                                   # all tied
    lg[2, 10:20] = 3.0                               # a block of ties at the top
    lg[3, ::7] = np.nan                              # NaN never selected
    lg[4, :] = np.nan
    lg[4, [5, 77]] = [1.0, 2.0]                      # fewer finite than K
    lg[5, 3] = 50.0                                  # large (no overflow below 88)
    lg[6] = np.round(lg[6] * 4) / 4                  # many ties
    ti = torch.empty(T, K, dtype=torch.int32, device="cuda")
    tw = torch.empty(T, K, dtype=torch.float32, device="cuda")
    lib.launch_moe_topk(dev(lg).data_ptr(), ti.data_ptr(), tw.data_ptr(), E, K, T, st)
    g["topk_logits"], g["topk_idx"], g["topk_w"] = lg, host(ti), host(tw)
    lg2 = rng.standard_normal((37, 8)).astype(np.float32)
    ti2 = torch.empty(37, 2, dtype=torch.int32, device="cuda")
    tw2 = torch.empty(37, 2, dtype=torch.float32, device="cuda")
    lib.launch_moe_topk(dev(lg2).data_ptr(), ti2.data_ptr(), tw2.data_ptr(), 8, 2, 37, st)
    g["topk2_logits"], g["topk2_idx"], g["topk2_w"] = lg2, host(ti2), host(tw2)

    # swiglu
    n = 4096
    gt = (3 * rng.standard_normal(n)).astype(np.float32)
    up = rng.standard_normal(n).astype(np.float32)
    o = torch.empty(n, dtype=torch.float32, device="cuda")
    lib.launch_swiglu(dev(gt).data_ptr(), dev(up).data_ptr(), o.data_ptr(), n, st)
    g["swiglu_gate"], g["swiglu_up"], g["swiglu_out"] = gt, up, host(o)

    # moe_combine: [T][k][H] expert outputs with [T][k] weights
    T, K, H = 5, 3, 256
    eo = rng.standard_normal((T, K, H)).astype(np.float32)
    ew = rng.random((T, K)).astype(np.float32)
    o = torch.empty(T, H, dtype=torch.float32, device="cuda")
    lib.launch_moe_combine(dev(eo).data_ptr(), dev(ew).data_ptr(), o.data_ptr(), H, K, T, st)
    g["combine_eo"], g["combine_w"], g["combine_out"] = eo, ew, host(o)

    # add_residual (in place on a)
    aa = rng.standard_normal(1000).astype(np.float32)
    bb = rng.standard_normal(1000).astype(np.float32)
    ta = dev(aa)
    lib.launch_add_residual(ta.data_ptr(), dev(bb).data_ptr(), 1000, st)
    g["resid_a"], g["resid_b"], g["resid_out"] = aa, bb, host(ta)

    # argmax with ties (first index wins)
    lg = rng.standard_normal((6, 1000)).astype(np.float32)
    lg[2, [10, 500]] = 9.0
    am = torch.empty(6, dtype=torch.int64, device="cuda")
    lib.launch_argmax(dev(lg).data_ptr(), am.data_ptr(), 1000, 6, st)
    g["argmax_in"], g["argmax_out"] = lg, host(am)

    # rope: q, k both [seq][heads][d] (the reference strides k by num_heads)
    S_, NH, D = 5, 4, 64
    q = rng.standard_normal((S_, NH, D)).astype(np.float32)
    k = rng.standard_normal((S_, NH, D)).astype(np.float32)
    tq, tk = dev(q), dev(k)
    lib.launch_rope(tq.data_ptr(), tk.data_ptr(), D, NH, S_, 7, 10000.0, st)
    g["rope_q"], g["rope_k"], g["rope_q_out"], g["rope_k_out"] = q, k, host(tq), host(tk)

    np.savez_compressed(a.out, **g)
    print(f"wrote {a.out}: {len(g)} arrays")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
