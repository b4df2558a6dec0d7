"""The layer's column-ordered router path (include/moe_layer.h:
moe_router_columns, moe_rmsnorm_quant_rc, moe_router_logits_rc) through the
C-ABI.  The column order is this library's own layout, so the bar is
identity with the plain-layout entry points and with the oracle's logits in
the reference's summation order (csrc/kernels.cu:412-435): bit-exact.
"""
import numpy as np
import pytest
import torch

from time_b200 import synth
from time_b200 import moe as M


def router_col_index(H: int) -> np.ndarray:
    """dst column of each source column i = 256j + 32m + 4q + r
    (r = 2 r_hi + r_lo): r_lo*128J + m*16J + 16j + 8 r_hi + q."""
    J = H // 256
    i = np.arange(H)
    r, q, m, j = i & 3, (i >> 2) & 7, (i >> 5) & 7, i >> 8
    return (r & 1) * 128 * J + m * 16 * J + 16 * j + 8 * (r >> 1) + q


def to_router_cols(a: np.ndarray) -> np.ndarray:
    out = np.empty_like(a)
    out[..., router_col_index(a.shape[-1])] = a
    return out


@pytest.mark.parametrize("H", [256, 512, 1280, 5120, 12288])
def test_router_col_index_is_a_grouping_permutation(H):
    """CPU: a bijection, and for each (r_lo, m) the lanes (r_hi, q) of all
    steps j form one contiguous run of 16J columns in ascending j."""
    J = H // 256
    c = router_col_index(H)
    assert np.array_equal(np.sort(c), np.arange(H))
    i = np.arange(H)
    for r_lo in range(2):
        for m in range(8):
            sel = i[((i & 1) == r_lo) & (((i >> 5) & 7) == m)]
            cols = c[sel]
            base = r_lo * 128 * J + m * 16 * J
            assert cols.min() == base and cols.max() == base + 16 * J - 1
            # step j of the run holds lanes 8 r_hi + q of that step
            jj = sel >> 8
            assert np.array_equal((cols - base) // 16, jj)


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.gpu
@pytest.mark.parametrize("rows,H", [(1, 256), (7, 512), (160, 5120), (33, 12288)])
def test_router_columns_matches_the_layout(gpu, rows, H):
    k = M.libs()["libkernels.so"]
    g = torch.Generator().manual_seed(rows + H)
    src = torch.randn(rows, H, generator=g)
    dst = torch.full((rows, H), float("nan"), device=gpu)
    sd = src.to(gpu)
    M.check("router_columns", k.moe_router_columns(M.ptr(sd), M.ptr(dst), rows, H, _stream()))
    torch.cuda.synchronize()
    assert np.array_equal(dst.cpu().numpy().view(np.uint32), to_router_cols(src.numpy()).view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("T,H", [(1, 256), (37, 512), (300, 5120), (2500, 1280), (2304, 768), (4096, 5120)])
def test_rmsnorm_rc_is_the_reordered_plain_output(gpu, T, H):
    """moe_rmsnorm_quant_rc: n bit-identical to moe_rmsnorm_quant_n's n put
    in the router column order; rms, e4m3 bytes and scales identical (both
    the block-per-token form, T <= 2048, and the warp-per-token form)."""
    k = M.libs()["libkernels.so"]
    g = torch.Generator().manual_seed(T * 3 + H)
    x = (torch.randn(T, H, generator=g) * torch.exp(torch.randn(T, 1, generator=g))).to(torch.bfloat16).to(gpu)
    gamma = (1 + 0.1 * torch.randn(H, generator=g)).float().to(gpu)
    ld = (T + 3) // 4 * 4
    outs = []
    for fn in (k.moe_rmsnorm_quant_n, k.moe_rmsnorm_quant_rc):
        rms = torch.empty(T, device=gpu)
        n = torch.empty(T, H, device=gpu)
        xq = torch.empty(T, H, dtype=torch.uint8, device=gpu)
        xs = torch.empty(H // 128, ld, device=gpu)
        M.check("rmsnorm", fn(M.ptr(x), M.ptr(gamma), T, H, 1e-5, M.ptr(rms), M.ptr(n), M.ptr(xq), M.ptr(xs), ld,
                              _stream()))
        outs.append((rms, n, xq, xs))
    torch.cuda.synchronize()
    (r0, n0, q0, s0), (r1, n1, q1, s1) = outs
    assert torch.equal(r0, r1) and torch.equal(q0, q1) and torch.equal(s0[:, :T], s1[:, :T])
    assert np.array_equal(n1.cpu().numpy().view(np.uint32), to_router_cols(n0.cpu().numpy()).view(np.uint32))


def _logits_both(k, n, W, b, gpu):
    T, H = n.shape
    E = W.shape[0]
    nd = torch.from_numpy(np.ascontiguousarray(n)).to(gpu)
    Wd = torch.from_numpy(np.ascontiguousarray(W)).to(gpu)
    bd = torch.from_numpy(b).to(gpu) if b is not None else None
    nrc = torch.from_numpy(to_router_cols(n)).to(gpu)
    wrc = torch.empty_like(Wd)
    M.check("router_columns", k.moe_router_columns(M.ptr(Wd), M.ptr(wrc), E, H, _stream()))
    plain = torch.empty(T, E, device=gpu)
    rc = torch.full((T, E), float("nan"), device=gpu)
    M.check("router_logits", k.moe_router_logits(M.ptr(nd), M.ptr(Wd), M.ptr(bd), T, H, E, M.ptr(plain), _stream()))
    M.check("router_logits_rc", k.moe_router_logits_rc(M.ptr(nrc), M.ptr(wrc), M.ptr(bd), T, H, E, M.ptr(rc),
                                                         _stream()))
    torch.cuda.synchronize()
    return plain.cpu().numpy(), rc.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,E,bias", [(1, 256, 8, False), (5, 256, 8, True), (31, 512, 64, True),
                                        (33, 1280, 100, False), (70, 2560, 160, True), (300, 5120, 160, True),
                                        (64, 12288, 160, True), (1000, 512, 256, True), (129, 768, 33, False),
                                        (4096, 1024, 160, True)])
def test_router_logits_rc_bit_exact(gpu, oracle, T, H, E, bias):
    """Ragged token and expert counts (partial tiles), step counts that are
    not multiples of the 7-step chunk (J = 3, 1, 5, 10, 48), E up to 256: the
    column-ordered router equals moe_router_logits and the reference-order
    oracle bit for bit."""
    k = M.libs()["libkernels.so"]
    g = torch.Generator().manual_seed(T * 7 + H + E)
    n = (torch.randn(T, H, generator=g) * torch.exp(torch.randn(T, 1, generator=g))).numpy()
    W = (torch.randn(E, H, generator=g) * 0.02).numpy()
    b = synth.zipf_bias(E, seed=3).numpy() if bias else None
    plain, rc = _logits_both(k, n, W, b, gpu)
    assert np.array_equal(rc.view(np.uint32), plain.view(np.uint32))
    if T * E * H <= 2e9:
        lg = oracle.moe_gate_ref(n, W, b)
        assert np.array_equal(rc.view(np.uint32), lg.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_router_rc_glm_shape_every_token(gpu, oracle, seed):
    """BASELINE configs[1] router (4096 x 5120 x 160, zipf bias): every logit
    of the column-ordered path bit-identical to the reference-order oracle."""
    shape = synth.GLM
    k = M.libs()["libkernels.so"]
    T = 4096
    w = synth.make_moe_weights(shape, seed=seed, device="cpu", zipf_bias=True, experts=False)
    x = synth.make_x(shape, T, seed=seed + 1, device="cpu")
    n = oracle.rmsnorm_ref(x.float().numpy(), w["gamma"].numpy(), shape.eps)
    Wr, b = w["router_w"].numpy(), w["router_bias"].numpy()
    plain, rc = _logits_both(k, n, Wr, b, gpu)
    lg = oracle.moe_gate_ref(n, Wr, b)
    assert np.array_equal(rc.view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(plain.view(np.uint32), lg.view(np.uint32))


@pytest.mark.gpu
def test_router_rc_rejects_bad_arguments(gpu):
    k = M.libs()["libkernels.so"]
    a = torch.zeros(4, 384, device=gpu)
    b = torch.zeros(4, 384, device=gpu)
    lg = torch.zeros(4, 4, device=gpu)
    # H not a multiple of 256, aliasing, too many experts
    assert k.moe_router_columns(M.ptr(a), M.ptr(b), 4, 384, _stream()) != 0
    assert k.moe_router_columns(M.ptr(a), M.ptr(a), 4, 256, _stream()) != 0
    assert k.moe_router_logits_rc(M.ptr(a), M.ptr(b), None, 4, 384, 4, M.ptr(lg), _stream()) != 0
    assert k.moe_router_logits_rc(M.ptr(a), M.ptr(b), None, 4, 256, 257, M.ptr(lg), _stream()) != 0
