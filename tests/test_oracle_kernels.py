"""The oracle's reductions, routing, permutation and MoE forward against
independent numpy restatements (float64) and the reference's tie rules."""
import numpy as np
import pytest

from time_b200 import synth


def test_rmsnorm_close_to_float64(oracle):
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (17, 640)).astype(np.float32)
    g = rng.normal(1, 0.1, 640).astype(np.float32)
    got = oracle.rmsnorm_ref(x, g, 1e-5)
    x64 = x.astype(np.float64)
    exp = x64 / np.sqrt((x64 ** 2).mean(1, keepdims=True) + 1e-5) * g
    assert np.allclose(got, exp, rtol=2e-6, atol=1e-7)


def test_rmsnorm_tree_order_is_not_sequential(oracle):
    """The reference order (256 partials + tree) is observable: it differs
    from a sequential fp32 sum for some rows; equal to float32 tree emulation."""
    rng = np.random.default_rng(1)
    x = (rng.normal(0, 1, (64, 1024)) * np.exp(rng.normal(0, 3, (64, 1024)))).astype(np.float32)
    rms = oracle.rms_ref(x, 0.0)
    # numpy emulation of the same order (no fma in numpy: compare to 1 ulp)
    p = np.zeros((64, 256), np.float32)
    for j in range(0, 1024, 256):
        p = (p + x[:, j:j + 256] * x[:, j:j + 256]).astype(np.float32)
    s = 128
    while s:
        p[:, :s] = p[:, :s] + p[:, s:2 * s]
        s //= 2
    emu = np.sqrt(p[:, 0] / np.float32(1024))
    assert np.allclose(rms, emu, rtol=3e-7)


def _fma_f32(a: float, b: float, c: float) -> float:
    """fp32 fma with one rounding: the exact a*b + c (as a fraction), rounded
    to the nearest fp32 (ties to even)."""
    from fractions import Fraction
    exact = Fraction(a) * Fraction(b) + Fraction(c)
    lo = np.float32(float(exact))              # within one fp32 ulp of exact
    cands = [np.nextafter(lo, np.float32(-np.inf)), lo, np.nextafter(lo, np.float32(np.inf))]
    best = min(cands, key=lambda v: (abs(Fraction(float(v)) - exact), int(np.array(v).view(np.uint32)) & 1))
    return float(best)


def test_router_logits_tree_restated_in_python(oracle):
    """moe_gate_ref against a pure-Python restatement of kernel_moe_gate
    (csrc/kernels.cu:412-435, blockDim 256): 256 fma chains, then the pairwise
    tree with fp32 adds; and the bias is one fp32 add after the tree."""
    rng = np.random.default_rng(2)
    H = 640                                  # not a multiple of 256: chains of 3 and 2 steps
    h = (rng.normal(0, 1, (3, H)) * np.exp(rng.normal(0, 2, (3, 1)))).astype(np.float32)
    w = rng.normal(0, 0.02, (4, H)).astype(np.float32)
    got = oracle.moe_gate_ref(h, w)
    for t in range(3):
        for e in range(4):
            p = []
            for lane in range(256):
                acc = 0.0
                for i in range(lane, H, 256):
                    acc = _fma_f32(float(h[t, i]), float(w[e, i]), acc)
                p.append(np.float32(acc))
            stride = 128
            while stride:
                for lane in range(stride):
                    p[lane] = np.float32(p[lane] + p[lane + stride])
                stride //= 2
            assert np.float32(p[0]).view(np.uint32) == got[t, e].view(np.uint32), (t, e)
    b = rng.normal(0, 1, 4).astype(np.float32)
    assert np.array_equal(oracle.moe_gate_ref(h, w, b).view(np.uint32), (got + b).astype(np.float32).view(np.uint32))


def _topk_insertion_py(row, k):
    """csrc/kernels.cu:437-462 restated in Python."""
    fmax = np.finfo(np.float32).max
    mv = [-fmax] * k
    mi = [-1] * k
    for e, val in enumerate(row):
        for j in range(k):
            if val > mv[j]:
                mv[j + 1:] = mv[j:k - 1]
                mi[j + 1:] = mi[j:k - 1]
                mv[j] = val
                mi[j] = e
                break
    return mi, mv


@pytest.mark.parametrize("k", [1, 2, 8, 16])
def test_topk_ties_and_nan(oracle, k):
    rng = np.random.default_rng(k)
    E = 40
    lg = rng.integers(-3, 3, (50, E)).astype(np.float32)   # many exact ties
    lg[0, :] = np.nan
    lg[1, 5] = np.nan
    lg[2, :] = -np.finfo(np.float32).max                   # never strictly greater than the init
    lg[3, :] = -np.inf
    lg[4, 7] = np.inf
    idx, w = oracle.moe_topk_ref(lg, k)
    for t in range(50):
        mi, mv = _topk_insertion_py(list(lg[t]), k)
        assert list(idx[t]) == mi, t
        valid = [v for v, i in zip(mv, mi) if i >= 0]
        if valid and all(np.isfinite(valid)):
            e = np.exp(np.array(mv, np.float64))
            assert np.allclose(w[t], e / e.sum(), rtol=1e-5, atol=1e-7)
    assert (idx[0] == -1).all() and (idx[2] == -1).all() and (idx[3] == -1).all()


def test_topk_weights_no_overflow(oracle):
    lg = np.array([[100.0, 99.0, 90.0, 1.0]], np.float32)
    idx, w = oracle.moe_topk_ref(lg, 2)
    assert list(idx[0]) == [0, 1]
    assert np.allclose(w[0], [1 / (1 + np.exp(-1)), np.exp(-1) / (1 + np.exp(-1))], rtol=1e-6)


def test_permute_stable_and_padded(oracle):
    rng = np.random.default_rng(3)
    T, k, E = 37, 4, 9
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    idx[5, 2] = -1                                          # an unassigned slot
    counts, start, pos, row_token, R = oracle.moe_permute(idx, E, 1, pad=16)
    assert counts[E] == T and counts[:E].sum() == T * k - 1
    assert all(s % 16 == 0 for s in start)
    assert R == start[-1] + ((T + 15) // 16) * 16
    for e in range(E):
        pairs = [p for p in range(T * k) if idx.flat[p] == e]   # ascending pair order
        rows = [pos.flat[p] for p in pairs]
        assert rows == list(range(start[e], start[e] + len(pairs)))
        assert all(row_token[r] == p // k for r, p in zip(rows, pairs))
        assert all(row_token[r] == -1 for r in range(start[e] + counts[e], start[e] + (counts[e] + 15) // 16 * 16))
    assert pos[5, 2] == -1
    assert list(row_token[start[E]:start[E] + T]) == list(range(T))


def test_quant_row_1x128(oracle):
    import ml_dtypes
    rng = np.random.default_rng(4)
    v = rng.normal(0, 1, (3, 384)).astype(np.float32)
    v[1, 128:256] = 0.0
    q, s = oracle.quant_rows_1x128(v)
    for r in range(3):
        for b in range(3):
            blk = v[r, b * 128:(b + 1) * 128]
            amax = np.float32(np.abs(blk).max())
            if amax == 0:
                assert s[r, b] == 0 and (q[r, b * 128:(b + 1) * 128] == 0).all()
                continue
            inv = np.float32(448.0) / amax
            exp = (blk * inv).astype(ml_dtypes.float8_e4m3fn).view(np.uint8)
            assert np.array_equal(q[r, b * 128:(b + 1) * 128], exp)
            assert s[r, b] == np.float32(amax / np.float32(448.0))


def _numpy_moe(case, shape, mode):
    """Independent float64 numpy restatement of the MoE FFN block."""
    import ml_dtypes
    H, E, k, I, S = shape.hidden, shape.num_experts, shape.top_k, shape.intermediate, shape.num_shared
    x = case["x"].float().numpy().astype(np.float64)
    n32 = None
    from oracle import oracle as orc
    n32 = orc.rmsnorm_ref(case["x"].float().numpy(), case["gamma"].numpy(), shape.eps)
    logits = orc.moe_gate_ref(n32, case["router_w"].numpy(),
                              case["router_bias"].numpy() if case["router_bias"] is not None else None)
    idx, wts = orc.moe_topk_ref(logits, k)
    lut = np.arange(256, dtype=np.uint8).view(ml_dtypes.float8_e4m3fn).astype(np.float64)

    def deq(q, s):
        rows, cols = q.shape
        return lut[q] * np.repeat(np.repeat(s.astype(np.float64), 128, 0), 128, 1)

    def quant(v):
        qq, ss = orc.quant_rows_1x128(v.astype(np.float32))
        return lut[qq] * np.repeat(ss.astype(np.float64), 128, 1)

    a = quant(n32) if mode == 0 else n32.astype(np.float64)
    out = x.copy()
    w13, s13, w2, s2 = (case[n].numpy() for n in ("w13", "s13", "w2", "s2"))

    def expert(e, rows):
        W13 = deq(w13[e], s13[e])
        W2 = deq(w2[e], s2[e])
        gu = rows @ W13.T
        g, u = gu[:, :I], gu[:, I:]
        g32 = g.astype(np.float32)
        h = (g32 / (np.float32(1) + np.exp(-g32))).astype(np.float64) * u
        hh = quant(h) if mode == 0 else h
        y = hh @ W2.T
        if mode == 0:
            y = y.astype(np.float32).astype(ml_dtypes.bfloat16).astype(np.float64)
        return y

    for s_ in range(S):
        out += expert(E + s_, a)
    for t in range(x.shape[0]):
        for j in range(k):
            e = idx[t, j]
            if e >= 0:
                out[t] += wts[t, j] * expert(e, a[t:t + 1])[0]
    return out, idx


@pytest.mark.parametrize("mode", [0, 1])
def test_oracle_forward_vs_numpy(oracle, mode):
    shape = synth.TINY
    case = synth.make_case(shape, 24, seed=5)
    ow = oracle.OracleWeights(shape, case)
    xb = case["x"].view(__import__("torch").int16).numpy().view(np.uint16)
    out, idx, w, lg = oracle.moe_ffn_forward(ow, xb, mode=mode)
    exp, eidx = _numpy_moe(case, shape, mode)
    assert np.array_equal(idx, eidx)
    got = oracle.bf16_bits_to_f32(out).astype(np.float64)
    exp_bf16 = oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(exp.astype(np.float32))).astype(np.float64)
    mr, mae = oracle.max_rel_and_mae(got, exp_bf16)
    assert mr < 4e-3 and mae < 2e-4, (mr, mae)


def test_oracle_q_vs_ref_modes_differ_by_fp8_activation_error(oracle):
    shape = synth.TINY
    case = synth.make_case(shape, 32, seed=6)
    ow = oracle.OracleWeights(shape, case)
    xb = case["x"].view(__import__("torch").int16).numpy().view(np.uint16)
    q, *_ = oracle.moe_ffn_forward(ow, xb, mode=0)
    r, *_ = oracle.moe_ffn_forward(ow, xb, mode=1)
    x = case["x"].float().numpy()
    dq = oracle.bf16_bits_to_f32(q) - x
    dr = oracle.bf16_bits_to_f32(r) - x
    rel = np.linalg.norm(dq - dr) / np.linalg.norm(dr)
    assert 1e-3 < rel < 0.1, rel     # e4m3 activations: a few percent on the MoE delta
