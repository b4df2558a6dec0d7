"""Two-term e4m3 activations (CBW_GEMM_ACT_X2, moe_layer_set_act_planes(2))
through the C-ABI.

Each 1x128 block keeps one scale s and two e4m3 planes, hi = e4m3(v/s) and
lo = e4m3(v/s - decode(hi)).  Bars:
  * the quantisers (RMSNorm, gather) bit-exact against the oracle's
    restatement, the hi plane identical to the one-plane quantiser's bytes;
  * the grouped GEMMs within the one-plane tests' relative bars of a float64
    product of the dequantised two-plane operands, in every tile form that
    has a two-plane variant;
  * the layer within the north-star bar (max-rel 1e-2, MAE 2e-3) of the
    oracle's two-plane mirror ("q2") AND of the reference's semantics (fp32
    activations, oracle "ref" mode) -- the bar one e4m3 plane cannot meet at
    the GLM shape.
"""
import numpy as np
import pytest
import torch

from time_b200 import synth
from time_b200 import moe as M

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MAE = 2e-3


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def stream():
    return torch.cuda.current_stream().cuda_stream


def _lut():
    return torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).to(torch.float64)


def _split(v):
    """float64 [r][c] -> (hi, lo, scales [c/128][r]) with the fp32 arithmetic
    of the kernels (the oracle's restatement)."""
    from oracle import oracle as orc
    q, ql, s = orc.quant_rows_1x128_x2(v.float().numpy())
    return torch.from_numpy(q), torch.from_numpy(ql), torch.from_numpy(np.ascontiguousarray(s.T))


@pytest.mark.parametrize("T,H,rc", [(1, 256, 0), (37, 512, 1), (300, 5120, 1), (2500, 1280, 0), (2049, 640, 0),
                                    (4096, 5120, 1)])
def test_rmsnorm_quant_x2_bit_exact(gpu, oracle, T, H, rc):
    """hi plane identical to the one-plane quantiser, lo plane and scales
    bit-exact to the oracle; n written as moe_rmsnorm_quant_n / _rc write it."""
    k = M.libs()["libkernels.so"]
    g = torch.Generator().manual_seed(T + H)
    x = (torch.randn(T, H, generator=g) * torch.exp(torch.randn(T, 1, generator=g))).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(H, generator=g)).float()
    xd, gd = x.to(gpu), gamma.to(gpu)
    ld = (T + 3) // 4 * 4
    rms = torch.empty(T, device=gpu)
    n = torch.empty(T, H, device=gpu)
    xq = torch.empty(T, H, dtype=torch.uint8, device=gpu)
    xl = torch.empty(T, H, dtype=torch.uint8, device=gpu)
    xs = torch.empty(H // 128, ld, device=gpu)
    M.check("x2", k.moe_rmsnorm_quant_x2(M.ptr(xd), M.ptr(gd), T, H, 1e-5, M.ptr(rms), M.ptr(n), rc, M.ptr(xq),
                                         M.ptr(xl), M.ptr(xs), ld, stream()))
    n1 = torch.empty(T, H, device=gpu)
    xq1 = torch.empty(T, H, dtype=torch.uint8, device=gpu)
    xs1 = torch.empty(H // 128, ld, device=gpu)
    fn = k.moe_rmsnorm_quant_rc if rc else k.moe_rmsnorm_quant_n
    M.check("one", fn(M.ptr(xd), M.ptr(gd), T, H, 1e-5, M.ptr(rms), M.ptr(n1), M.ptr(xq1), M.ptr(xs1), ld, stream()))
    torch.cuda.synchronize()
    assert torch.equal(xq, xq1) and torch.equal(xs[:, :T], xs1[:, :T]) and torch.equal(n, n1)
    nref = oracle.rmsnorm_ref(x.float().numpy(), gamma.numpy(), 1e-5)
    q, ql, s = oracle.quant_rows_1x128_x2(nref)
    assert np.array_equal(xq.cpu().numpy(), q)
    assert np.array_equal(xl.cpu().numpy(), ql)
    assert np.array_equal(xs.cpu().numpy()[:, :T], s.T)


def test_gather_rows_x2(gpu):
    k = M.libs()["libkernels.so"]
    T, H, R = 50, 512, 96
    g = torch.Generator().manual_seed(5)
    xq = torch.randint(0, 255, (T, H), generator=g, dtype=torch.uint8).to(gpu)
    xl = torch.randint(0, 255, (T, H), generator=g, dtype=torch.uint8).to(gpu)
    xs = torch.rand(H // 128, 52, generator=g).to(gpu)
    rowtok = torch.tensor([(i * 7) % T if i % 5 else -1 for i in range(R)], dtype=torch.int32, device=gpu)
    xp = torch.full((2, R, H), 0x33, dtype=torch.uint8, device=gpu)
    xps = torch.full((H // 128, R), -1.0, device=gpu)
    M.check("gather", k.moe_gather_rows_x2(M.ptr(xq), M.ptr(xl), M.ptr(xs), 52, M.ptr(rowtok), None, R, H,
                                           M.ptr(xp[0]), M.ptr(xp[1]), M.ptr(xps), R, stream()))
    torch.cuda.synchronize()
    rt = rowtok.cpu()
    for r in range(R):
        t = int(rt[r])
        if t < 0:
            assert (xp[0, r] == 0).all() and (xp[1, r] == 0).all() and (xps[:, r] == 0).all()
        else:
            assert torch.equal(xp[0, r], xq[t]) and torch.equal(xp[1, r], xl[t])
            assert torch.equal(xps[:, r], xs[:, t])



@pytest.mark.parametrize("T,K,E,shared,planes,H", [(4096, 8, 160, 1, 2, 5120), (300, 8, 160, 1, 1, 512),
                                                   (37, 4, 9, 0, 2, 640), (1, 16, 32, 1, 2, 512)])
def test_scatter_rows_matches_gather(gpu, T, K, E, shared, planes, H):
    """moe_scatter_rows_x2 (token-major: each token read once, stored to its
    routed and shared rows) writes exactly the bytes of moe_gather_rows_x2 for
    the layer's permutation, padding rows zeroed, over every row of the
    layout (H = 5120: two 8-piece batches per lane, the second partial)."""
    k = M.libs()["libkernels.so"]
    g = torch.Generator().manual_seed(T * 3 + K)
    idx = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
    if T > 2:
        idx[1, 0] = -1                                   # an empty slot
    d_idx = idx.to(gpu)
    G = E + shared
    cap = (T * K + shared * T + 16 * G + 15) // 16 * 16
    counts = torch.zeros(G, dtype=torch.int32, device=gpu)
    start = torch.zeros(G, dtype=torch.int32, device=gpu)
    pos = torch.full((T * K,), -9, dtype=torch.int32, device=gpu)
    rowtok = torch.full((cap,), -9, dtype=torch.int32, device=gpu)
    total = torch.zeros(1, dtype=torch.int32, device=gpu)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    nbytes = k.moe_permute_mb_scratch_bytes(T, K, 0, E)
    scratch = torch.empty(max(nbytes, 4), dtype=torch.uint8, device=gpu)
    M.check("permute_mb", k.moe_permute_mb(M.ptr(d_idx), T, K, 0, E, shared, M.ptr(counts), M.ptr(start), M.ptr(pos),
                                           M.ptr(rowtok), M.ptr(total), cap, M.ptr(err), 16, M.ptr(scratch), nbytes,
                                           stream()))
    ld = (T + 3) // 4 * 4
    xq = torch.randint(0, 255, (T, H), generator=g, dtype=torch.uint8).to(gpu)
    xl = torch.randint(0, 255, (T, H), generator=g, dtype=torch.uint8).to(gpu) if planes == 2 else None
    xs = torch.rand(H // 128, ld, generator=g).to(gpu)
    outs = []
    for fn in ("gather", "scatter"):
        xp = torch.full((2, cap, H), 0x33, dtype=torch.uint8, device=gpu)
        xps = torch.full((H // 128, cap), -1.0, device=gpu)
        lo_in = M.ptr(xl) if xl is not None else None
        lo_out = M.ptr(xp[1]) if xl is not None else None
        if fn == "gather":
            M.check("gather", k.moe_gather_rows_x2(M.ptr(xq), lo_in, M.ptr(xs), ld, M.ptr(rowtok), M.ptr(total), cap,
                                                   H, M.ptr(xp[0]), lo_out, M.ptr(xps), cap, stream()))
        else:
            M.check("scatter", k.moe_scatter_rows_x2(M.ptr(xq), lo_in, M.ptr(xs), ld, M.ptr(pos), T, K,
                                                     M.ptr(start[E:]) if shared else None, shared, M.ptr(rowtok),
                                                     M.ptr(total), cap, H, M.ptr(xp[0]), lo_out, M.ptr(xps), cap,
                                                     stream()))
        torch.cuda.synchronize()
        outs.append((xp.cpu(), xps.cpu()))
    R = int(total.item())
    assert err.item() == 0 and R > 0
    assert torch.equal(outs[0][0][:, :R], outs[1][0][:, :R])
    assert torch.equal(outs[0][1][:, :R], outs[1][1][:, :R])


def _groups_x2(counts, K, Nw, g):
    G = len(counts)
    starts, row = [], 0
    for c in counts:
        starts.append(row)
        row += (c + 15) // 16 * 16
    rows = row + 32
    v = torch.randn(rows, K, generator=g, dtype=torch.float64) * torch.exp(
        torch.randn(rows, 1, generator=g, dtype=torch.float64))
    hi, lo, s = _split(v)
    a_ld = (rows + 3) // 4 * 4
    A_s = torch.zeros(K // 128, a_ld)
    A_s[:, :rows] = s
    W = (torch.randn(G, Nw, K, generator=g) * 0.5).clamp(-440, 440).to(torch.float8_e4m3fn).view(torch.uint8)
    W_s = (torch.rand(G, Nw // 128, K // 128, generator=g) * 0.01 + 0.0005).float()
    return starts, rows, torch.stack([hi, lo]), A_s, a_ld, W, W_s


def _ref_x2(A2, A_s, W, W_s, starts, counts):
    lut = _lut()
    out = {}
    for gi, (st, c) in enumerate(zip(starts, counts)):
        if c == 0:
            continue
        sc = A_s[:, st:st + c].T.double().repeat_interleave(128, 1)
        a = (lut[A2[0, st:st + c].long()] + lut[A2[1, st:st + c].long()]) * sc
        w = lut[W[gi].long()] * W_s[gi].double().repeat_interleave(128, 0).repeat_interleave(128, 1)
        out[gi] = a @ w.T
    return out


FORMS = [("small", M.GEMM_SMALL_TILES), ("one_sm", M.GEMM_ONE_SM_TILES), ("pair", M.GEMM_PAIR_TILES),
         ("token", M.GEMM_TOKEN_TILES)]


@pytest.mark.parametrize("form", [f for f in FORMS if f[0] != "one_sm"], ids=["small", "pair", "token"])
@pytest.mark.parametrize("counts,K,N", [([16], 256, 256), ([1, 0, 130, 255, 300], 512, 256), ([40, 257], 1536, 512)])
def test_grouped_gemm_down_x2(gpu, form, counts, K, N):
    g = torch.Generator().manual_seed(11 + sum(counts))
    starts, rows, A2, A_s, a_ld, W, W_s = _groups_x2(counts, K, N, g)
    out = torch.full((rows, N), float("nan"), dtype=torch.bfloat16, device=gpu)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    cnt = torch.tensor(counts, dtype=torch.int32, device=gpu)
    st = torch.tensor(starts, dtype=torch.int32, device=gpu)
    M.grouped_gemm(M.GEMM_DOWN_BF16 | form[1] | M.GEMM_ACT_X2, A2.contiguous().to(gpu), A_s.to(gpu), a_ld,
                   W.to(gpu), W_s.to(gpu), cnt, st, out, None, 0, K, N, rows, error_word=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    o = out.cpu().double()
    for gi, r in _ref_x2(A2, A_s, W, W_s, starts, counts).items():
        y = o[starts[gi]:starts[gi] + counts[gi]]
        assert torch.isfinite(y).all()
        rel = (y - r).abs().max() / r.abs().max()
        assert rel < 8e-3, (gi, float(rel))


def test_grouped_gemm_down_x2_one_sm_refused(gpu):
    """The one-SM full down form has no two-plane variant: the host refuses it."""
    counts, K, N = [16], 256, 256
    g = torch.Generator().manual_seed(1)
    starts, rows, A2, A_s, a_ld, W, W_s = _groups_x2(counts, K, N, g)
    out = torch.zeros((rows, N), dtype=torch.bfloat16, device=gpu)
    with pytest.raises(Exception):
        M.grouped_gemm(M.GEMM_DOWN_BF16 | M.GEMM_ONE_SM_TILES | M.GEMM_ACT_X2, A2.contiguous().to(gpu), A_s.to(gpu),
                       a_ld, W.to(gpu), W_s.to(gpu), torch.tensor(counts, dtype=torch.int32, device=gpu),
                       torch.tensor(starts, dtype=torch.int32, device=gpu), out, None, 0, K, N, rows)


@pytest.mark.parametrize("form", FORMS, ids=[f[0] for f in FORMS])
@pytest.mark.parametrize("counts,K,N", [([16], 256, 256), ([3, 0, 128, 129, 260], 256, 256), ([70, 300], 512, 384)])
def test_grouped_gemm_gated_x2(gpu, form, counts, K, N):
    """Gate/up in two-plane mode: h = silu(gate) * up written as hi/lo planes
    with one scale; its dequantisation within 5e-3 of the float64 h (one
    plane: 4e-2); the lo plane at most half an e4m3 step of the hi plane."""
    g = torch.Generator().manual_seed(3 + sum(counts))
    starts, rows, A2, A_s, a_ld, W, W_s = _groups_x2(counts, K, 2 * N, g)
    hq = torch.full((2, rows, N), 0x55, dtype=torch.uint8, device=gpu)
    hs = torch.full((N // 128, a_ld), -1.0, device=gpu)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    cnt = torch.tensor(counts, dtype=torch.int32, device=gpu)
    st = torch.tensor(starts, dtype=torch.int32, device=gpu)
    M.grouped_gemm(M.GEMM_GATED_SWIGLU | form[1] | M.GEMM_ACT_X2, A2.contiguous().to(gpu), A_s.to(gpu), a_ld,
                   W.to(gpu), W_s.to(gpu), cnt, st, hq, hs, a_ld, K, N, rows, error_word=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    lut = _lut()
    hq_c, hs_c = hq.cpu(), hs.cpu()
    for gi, r in _ref_x2(A2, A_s, W, W_s, starts, counts).items():
        gte, up = r[:, :N].float(), r[:, N:]
        h = (gte / (1 + torch.exp(-gte))).double() * up
        sl = slice(starts[gi], starts[gi] + counts[gi])
        s = hs_c[:, sl].T.double().repeat_interleave(128, 1)
        hi_v = lut[hq_c[0, sl].long()]
        lo_v = lut[hq_c[1, sl].long()]
        deq = (hi_v + lo_v) * s
        rel = (deq - h).abs().max() / h.abs().max()
        assert rel < 5e-3, (gi, float(rel))
        assert (lo_v.abs() <= hi_v.abs() * 2.0 ** -4 + 2.0 ** -9).all()
        pad_end = starts[gi] + (counts[gi] + 15) // 16 * 16
        assert (hq_c[:, starts[gi] + counts[gi]:pad_end] == 0).all()


@pytest.mark.parametrize("counts,K", [([16], 256), ([3, 0, 128, 129, 260, 1], 512), ([1000, 45], 1536)])
def test_grouped_gemm_x2_token_major_bit_identical(gpu, counts, K):
    """Two-plane token-major tiles give the bits of the other full forms: the
    gated output (both planes and the scales) equal to the one-SM form's, the
    down output equal to the CTA-pair form's."""
    N = 256
    g = torch.Generator().manual_seed(29 + sum(counts))
    cnt = torch.tensor(counts, dtype=torch.int32, device=gpu)
    starts, rows, A2, A_s, a_ld, W, W_s = _groups_x2(counts, K, 2 * N, g)
    st = torch.tensor(starts, dtype=torch.int32, device=gpu)
    gated = {}
    for form in (M.GEMM_ONE_SM_TILES, M.GEMM_TOKEN_TILES):
        hq = torch.full((2, rows, N), 0x55, dtype=torch.uint8, device=gpu)
        hs = torch.full((N // 128, a_ld), -1.0, device=gpu)
        err = torch.zeros(1, dtype=torch.int32, device=gpu)
        M.grouped_gemm(M.GEMM_GATED_SWIGLU | form | M.GEMM_ACT_X2, A2.contiguous().to(gpu), A_s.to(gpu), a_ld,
                       W.to(gpu), W_s.to(gpu), cnt, st, hq, hs, a_ld, K, N, rows, error_word=err)
        torch.cuda.synchronize()
        assert err.item() == 0
        gated[form] = (hq.cpu(), hs.cpu())
    _, _, _, _, _, Wd, Wd_s = _groups_x2(counts, K, N, g)
    down = {}
    for form in (M.GEMM_PAIR_TILES, M.GEMM_TOKEN_TILES):
        out = torch.full((rows, N), float("nan"), dtype=torch.bfloat16, device=gpu)
        err = torch.zeros(1, dtype=torch.int32, device=gpu)
        M.grouped_gemm(M.GEMM_DOWN_BF16 | form | M.GEMM_ACT_X2, A2.contiguous().to(gpu), A_s.to(gpu), a_ld,
                       Wd.to(gpu), Wd_s.to(gpu), cnt, st, out, None, 0, K, N, rows, error_word=err)
        torch.cuda.synchronize()
        assert err.item() == 0
        down[form] = out.cpu()
    for s0, c in zip(starts, counts):
        pad = (c + 15) // 16 * 16
        a_, b_ = gated[M.GEMM_TOKEN_TILES], gated[M.GEMM_ONE_SM_TILES]
        assert torch.equal(a_[0][:, s0:s0 + pad], b_[0][:, s0:s0 + pad])
        assert torch.equal(a_[1][:, s0:s0 + pad], b_[1][:, s0:s0 + pad])
        assert torch.equal(down[M.GEMM_TOKEN_TILES][s0:s0 + c].view(torch.int16),
                           down[M.GEMM_PAIR_TILES][s0:s0 + c].view(torch.int16))


def _layer_x2(shape, w, x, T, routing=None):
    layer = M.MoELayer(shape, w, max_tokens=max(T, 1))
    layer.set_act_planes(2)
    assert layer.act_planes == 2
    out = layer.forward(x, routing=routing)
    torch.cuda.synchronize()
    layer.check_error()
    return layer, out


@pytest.mark.parametrize("T", [64, 1, 200])
def test_layer_x2_tiny(gpu, oracle, T):
    shape = synth.TINY
    case = synth.make_case(shape, T, seed=0)
    layer, out = _layer_x2(shape, {k_: (v.to(gpu) if isinstance(v, torch.Tensor) else v) for k_, v in case.items()},
                           case["x"].to(gpu), T)
    idx, _, _ = layer.last_routing(T)
    ow = oracle.OracleWeights(shape, case)
    y = out.float().cpu().numpy()
    q2, oidx, *_ = oracle.moe_ffn_forward(ow, bits(case["x"]), mode=2)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    mr, mae = oracle.max_rel_and_mae(y, oracle.bf16_bits_to_f32(q2))
    assert mr <= MAX_REL and mae <= MAE, (mr, mae)
    ref, *_ = oracle.moe_ffn_forward(ow, bits(case["x"]), mode=1)
    mr1, mae1 = oracle.max_rel_and_mae(y, oracle.bf16_bits_to_f32(ref))
    print(f"x2 tiny T={T}: vs q2 {mr:.2e}/{mae:.2e}, vs ref (fp32 activations) {mr1:.2e}/{mae1:.2e}")
    assert mr1 <= MAX_REL and mae1 <= MAE, (mr1, mae1)


def test_layer_x2_glm_shape_within_the_reference_bar(gpu, oracle):
    """BASELINE configs[1] at full size with two-plane activations: 256 sampled
    tokens within the north-star bar of the reference's fp32-activation
    semantics (oracle "ref" mode) and of the two-plane mirror."""
    shape = synth.GLM
    T = 4096
    w = synth.make_moe_weights(shape, seed=0, device=gpu, zipf_bias=True)
    x = synth.make_x(shape, T, seed=1, device=gpu)
    layer, out = _layer_x2(shape, w, x, T)
    sample = np.random.default_rng(0).choice(T, 256, replace=False)
    ow = oracle.OracleWeights(shape, {k_: v for k_, v in w.items()})
    xs = bits(x.cpu()[sample])
    y = out.cpu()[sample].float().numpy()
    ref, *_ = oracle.moe_ffn_forward(ow, xs, mode=1)
    mr1, mae1 = oracle.max_rel_and_mae(y, oracle.bf16_bits_to_f32(ref))
    q2, *_ = oracle.moe_ffn_forward(ow, xs, mode=2)
    mr, mae = oracle.max_rel_and_mae(y, oracle.bf16_bits_to_f32(q2))
    print(f"x2 GLM 256 sampled tokens: vs q2 {mr:.2e}/{mae:.2e}, vs ref (fp32 activations) {mr1:.2e}/{mae1:.2e}")
    assert mr <= MAX_REL and mae <= MAE, (mr, mae)
    assert mr1 <= MAX_REL and mae1 <= MAE, (mr1, mae1)


def test_layer_x2_decode_routed_and_deterministic(gpu, oracle):
    """The routed entry (decode form, supplied routing) in two-plane mode, and
    bit-identical repeat calls."""
    shape = synth.TINY
    T = 48
    case = synth.make_case(shape, T, seed=6)
    wd = {k_: (v.to(gpu) if isinstance(v, torch.Tensor) else v) for k_, v in case.items()}
    ow = oracle.OracleWeights(shape, case)
    _, oidx, ow_, _ = oracle.moe_ffn_forward(ow, bits(case["x"]), mode=2)
    routing = (torch.from_numpy(oidx).to(gpu), torch.from_numpy(ow_).to(gpu))
    layer, out = _layer_x2(shape, wd, case["x"].to(gpu), T, routing=routing)
    out2 = layer.forward(case["x"].to(gpu), routing=routing).clone()
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    ref, *_ = oracle.moe_ffn_forward(ow, bits(case["x"]), mode=1)
    mr1, mae1 = oracle.max_rel_and_mae(out.float().cpu().numpy(), oracle.bf16_bits_to_f32(ref))
    assert mr1 <= MAX_REL and mae1 <= MAE, (mr1, mae1)
