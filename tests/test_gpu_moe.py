"""GPU parity of the MoE FFN block, stage by stage and end to end, through
the C-ABI (include/moe_layer.h, cublas_wrappers.h) against the CPU oracle.

Bars (from the north star):
  * integer/byte/index work bit-exact: RMSNorm rms, e4m3 activation bytes and
    scales, router logits in the reference's order (csrc/kernels.cu:412-435:
    256 lane partials and a pairwise tree, pinned to the reference's own kernel
    by tests/golden/ref_kernels.npz), top-k indices, the expert permutation;
  * bf16 layer outputs: max|y - y_oracle| / max|y_oracle| <= 1e-2 and
    mean|y - y_oracle| <= 2e-3 against the oracle in "q" mode (the oracle
    mirrors the kernels' e4m3 activation rounding points, accumulates in
    float64).
"""
import ctypes

import numpy as np
import pytest
import torch

from time_b200 import synth
from time_b200 import moe as M

pytestmark = pytest.mark.gpu

MAX_REL = 1e-2
MAE = 2e-3


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_dev(case, dev):
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}


def stream():
    return torch.cuda.current_stream().cuda_stream


# ---------------------------------------------------------------- stages

@pytest.mark.parametrize("T,H", [(1, 256), (37, 512), (64, 5120), (2100, 640), (4096, 5120)])
def test_rmsnorm_quant_bit_exact(gpu, oracle, T, H):
    k = M.libs()["libkernels.so"]
    g = torch.Generator().manual_seed(T + H)
    x = (torch.randn(T, H, generator=g) * torch.exp(torch.randn(T, H, generator=g))).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(H, generator=g)).float()
    xd, gd = x.to(gpu), gamma.to(gpu)
    rms = torch.empty(T, device=gpu)
    xq = torch.empty(T, H, dtype=torch.uint8, device=gpu)
    ld = (T + 3) // 4 * 4
    xs = torch.empty(H // 128, ld, device=gpu)
    M.check("moe_rmsnorm_quant", k.moe_rmsnorm_quant(M.ptr(xd), M.ptr(gd), T, H, 1e-5, M.ptr(rms), M.ptr(xq),
                                                     M.ptr(xs), ld, stream()))
    torch.cuda.synchronize()
    xf = x.float().numpy()
    assert np.array_equal(rms.cpu().numpy(), oracle.rms_ref(xf, 1e-5))
    n = oracle.rmsnorm_ref(xf, gamma.numpy(), 1e-5)
    q, s = oracle.quant_rows_1x128(n)
    assert np.array_equal(xq.cpu().numpy(), q)
    assert np.array_equal(xs.cpu().numpy()[:, :T], s.T)


@pytest.mark.parametrize("T,H,E,K,bias", [(5, 256, 8, 2, False), (70, 512, 160, 8, True), (33, 256, 64, 16, False),
                                          (128, 5120, 160, 8, True)])
def test_router_topk_bit_exact(gpu, oracle, T, H, E, K, bias):
    k = M.libs()["libkernels.so"]
    g = torch.Generator().manual_seed(E * 7 + T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    gamma = torch.ones(H)
    W = torch.randn(E, H, generator=g) * 0.02
    b = synth.zipf_bias(E, seed=1) if bias else None
    xd, gd, Wd = x.to(gpu), gamma.to(gpu), W.to(gpu)
    bd = b.to(gpu) if b is not None else None
    rms = torch.empty(T, device=gpu)
    xq = torch.empty(T, H, dtype=torch.uint8, device=gpu)
    ld = (T + 3) // 4 * 4
    xs = torch.empty(H // 128, ld, device=gpu)
    M.check("rmsnorm", k.moe_rmsnorm_quant(M.ptr(xd), M.ptr(gd), T, H, 1e-5, M.ptr(rms), M.ptr(xq), M.ptr(xs), ld,
                                           stream()))
    logits = torch.empty(T, E, device=gpu)
    idx = torch.empty(T, K, dtype=torch.int32, device=gpu)
    w = torch.empty(T, K, device=gpu)
    M.check("router", k.moe_router_topk(M.ptr(xd), M.ptr(rms), M.ptr(gd), M.ptr(Wd), M.ptr(bd), T, H, E, K,
                                        M.ptr(logits), M.ptr(idx), M.ptr(w), stream()))
    torch.cuda.synchronize()
    n = oracle.rmsnorm_ref(x.float().numpy(), gamma.numpy(), 1e-5)
    lg = oracle.moe_gate_ref(n, W.numpy(), b.numpy() if b is not None else None)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), lg.view(np.uint32))
    oi, ow = oracle.moe_topk_ref(lg, K)
    assert np.array_equal(idx.cpu().numpy(), oi)
    assert np.allclose(w.cpu().numpy(), ow, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("T,H,E,K,bias", [(5, 256, 8, 2, False), (70, 512, 160, 8, True), (33, 256, 64, 16, False),
                                          (300, 5120, 160, 8, True), (17, 384, 200, 4, True), (9, 128, 40, 3, True),
                                          (45, 640, 100, 5, False), (64, 12288, 160, 8, True),
                                          (1000, 512, 160, 8, True), (512, 5120, 160, 8, True),
                                          (4096, 1024, 160, 8, True),
                                          (4096, 5120, 200, 8, False)])
def test_tiled_router_bit_exact(gpu, oracle, T, H, E, K, bias):
    """The layer's router (stored n -> tiled logits -> top-k kernel) against
    the oracle and against moe_router_topk: identical bits."""
    k = M.libs()["libkernels.so"]
    g = torch.Generator().manual_seed(E * 11 + T)
    x = (torch.randn(T, H, generator=g) * torch.exp(torch.randn(T, 1, generator=g))).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(H, generator=g)).float()
    W = torch.randn(E, H, generator=g) * 0.02
    b = synth.zipf_bias(E, seed=2) if bias else None
    xd, gd, Wd = x.to(gpu), gamma.to(gpu), W.to(gpu)
    bd = b.to(gpu) if b is not None else None
    rms = torch.empty(T, device=gpu)
    n = torch.empty(T, H, device=gpu)
    xq = torch.empty(T, H, dtype=torch.uint8, device=gpu)
    ld = (T + 3) // 4 * 4
    xs = torch.empty(H // 128, ld, device=gpu)
    M.check("rmsnorm_n", k.moe_rmsnorm_quant_n(M.ptr(xd), M.ptr(gd), T, H, 1e-5, M.ptr(rms), M.ptr(n), M.ptr(xq),
                                               M.ptr(xs), ld, stream()))
    logits = torch.empty(T, E, device=gpu)
    M.check("router_logits", k.moe_router_logits(M.ptr(n), M.ptr(Wd), M.ptr(bd), T, H, E, M.ptr(logits), stream()))
    idx = torch.empty(T, K, dtype=torch.int32, device=gpu)
    w = torch.empty(T, K, device=gpu)
    M.check("topk_softmax", k.moe_topk_softmax(M.ptr(logits), T, E, K, M.ptr(idx), M.ptr(w), stream()))
    logits2 = torch.empty(T, E, device=gpu)
    idx2 = torch.empty(T, K, dtype=torch.int32, device=gpu)
    w2 = torch.empty(T, K, device=gpu)
    M.check("router", k.moe_router_topk(M.ptr(xd), M.ptr(rms), M.ptr(gd), M.ptr(Wd), M.ptr(bd), T, H, E, K,
                                        M.ptr(logits2), M.ptr(idx2), M.ptr(w2), stream()))
    torch.cuda.synchronize()
    nref = oracle.rmsnorm_ref(x.float().numpy(), gamma.numpy(), 1e-5)
    assert np.array_equal(n.cpu().numpy().view(np.uint32), nref.view(np.uint32))
    lg = oracle.moe_gate_ref(nref, W.numpy(), b.numpy() if b is not None else None)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), lg.view(np.uint32))
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), logits2.cpu().numpy().view(np.uint32))
    oi, ow = oracle.moe_topk_ref(lg, K)
    assert np.array_equal(idx.cpu().numpy(), oi)
    assert np.array_equal(idx.cpu().numpy(), idx2.cpu().numpy())
    assert np.array_equal(w.cpu().numpy().view(np.uint32), w2.cpu().numpy().view(np.uint32))
    assert np.allclose(w.cpu().numpy(), ow, rtol=2e-6, atol=1e-7)


def _router_logits_gpu(k, n, W, b, gpu):
    T, H = n.shape
    E = W.shape[0]
    nd, Wd = torch.from_numpy(np.ascontiguousarray(n)).to(gpu), torch.from_numpy(np.ascontiguousarray(W)).to(gpu)
    bd = torch.from_numpy(b).to(gpu) if b is not None else None
    logits = torch.empty(T, E, device=gpu)
    M.check("router_logits", k.moe_router_logits(M.ptr(nd), M.ptr(Wd), M.ptr(bd), T, H, E, M.ptr(logits), stream()))
    torch.cuda.synchronize()
    return logits.cpu().numpy()


@pytest.mark.parametrize("H,E", [(512, 64), (5120, 160)])
def test_router_logits_match_reference_kernel_golden(gpu, H, E):
    """The layer's router kernel on the inputs of the reference's own
    kernel_moe_gate run (tests/golden/ref_kernels.npz): identical bits."""
    from pathlib import Path
    fix = Path(__file__).resolve().parent / "golden" / "ref_kernels.npz"
    g = np.load(fix)
    k = M.libs()["libkernels.so"]
    got = _router_logits_gpu(k, g[f"gate_x_{H}_{E}"], g[f"gate_w_{H}_{E}"], None, gpu)
    assert np.array_equal(got.view(np.uint32), g[f"gate_out_{H}_{E}"].view(np.uint32))


@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4])
def test_router_glm_shape_reference_order_every_token(gpu, oracle, seed):
    """BASELINE configs[1] router: 4096 tokens x 5120 x 160 experts with the
    zipf routing bias.  Every logit bit-identical to the reference-order
    oracle, and every token's top-8 index list equal to the reference's top-k
    of those logits."""
    shape = synth.GLM
    k = M.libs()["libkernels.so"]
    T, H, E, K = 4096, shape.hidden, shape.num_experts, shape.top_k
    w = synth.make_moe_weights(shape, seed=seed, device="cpu", zipf_bias=True, experts=False)
    x = synth.make_x(shape, T, seed=seed + 1, device="cpu")
    n = oracle.rmsnorm_ref(x.float().numpy(), w["gamma"].numpy(), shape.eps)
    Wr, b = w["router_w"].numpy(), w["router_bias"].numpy()
    got = _router_logits_gpu(k, n, Wr, b, gpu)
    lg = oracle.moe_gate_ref(n, Wr, b)
    assert np.array_equal(got.view(np.uint32), lg.view(np.uint32))
    ld = torch.from_numpy(got).to(gpu)
    idx = torch.empty(T, K, dtype=torch.int32, device=gpu)
    wts = torch.empty(T, K, device=gpu)
    M.check("topk_softmax", k.moe_topk_softmax(M.ptr(ld), T, E, K, M.ptr(idx), M.ptr(wts), stream()))
    torch.cuda.synchronize()
    oi, ow = oracle.moe_topk_ref(lg, K)
    assert np.array_equal(idx.cpu().numpy(), oi)
    assert np.allclose(wts.cpu().numpy(), ow, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("T,K,E,shared", [(1, 1, 4, 1), (37, 4, 9, 1), (4096, 8, 160, 1), (300, 2, 8, 0),
                                          (2048, 8, 160, 1)])
def test_permute_bit_exact(gpu, oracle, T, K, E, shared):
    k = M.libs()["libkernels.so"]
    rng = np.random.default_rng(T + E)
    if T == 2048:   # everything to one expert (max group size, other groups empty)
        idx = np.tile(np.arange(K, dtype=np.int32), (T, 1))
    else:
        idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    if T > 5:
        idx[3, 0] = -1
    G = E + shared
    cap = T * K + shared * T + 16 * G
    d_idx = torch.from_numpy(idx).to(gpu)
    counts = torch.empty(G, dtype=torch.int32, device=gpu)
    start = torch.empty(G, dtype=torch.int32, device=gpu)
    pos = torch.empty(T * K, dtype=torch.int32, device=gpu)
    rowtok = torch.full((cap,), -7, dtype=torch.int32, device=gpu)
    total = torch.empty(1, dtype=torch.int32, device=gpu)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    M.check("permute", k.moe_permute(M.ptr(d_idx), T, K, 0, E, shared, M.ptr(counts), M.ptr(start), M.ptr(pos),
                                     M.ptr(rowtok), M.ptr(total), cap, M.ptr(err), stream()))
    torch.cuda.synchronize()
    c, s, p, rt, R = oracle.moe_permute(idx, E, shared)
    assert err.item() == 0
    assert total.item() == R
    assert np.array_equal(counts.cpu().numpy(), c)
    assert np.array_equal(start.cpu().numpy(), s)
    assert np.array_equal(pos.cpu().numpy(), p.reshape(-1))
    assert np.array_equal(rowtok.cpu().numpy()[:R], rt)


@pytest.mark.parametrize("T,K,E,eb,ee,shared,pad", [(1, 1, 4, 0, 4, 1, 16), (37, 4, 9, 0, 9, 1, 16),
                                                     (4096, 8, 160, 0, 160, 1, 16), (4096, 8, 160, 0, 160, 0, 1),
                                                     (2048, 8, 160, 40, 60, 1, 16), (300, 2, 8, 0, 8, 0, 1),
                                                     (513, 8, 160, 0, 160, 1, 16), (5000, 8, 160, 0, 160, 1, 16)])
def test_permute_multiblock_matches_single_block(gpu, oracle, T, K, E, eb, ee, shared, pad):
    """moe_permute_mb (the layer's permutation) against moe_permute_padded:
    identical counts, segment starts, pair rows and row tokens; and against
    the oracle for the 16-row padding."""
    k = M.libs()["libkernels.so"]
    rng = np.random.default_rng(T * 3 + E + eb)
    if T == 2048:   # one hot group, the rest empty
        idx = np.tile(np.arange(eb, eb + K, dtype=np.int32) % E, (T, 1))
    else:
        idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    if T > 5:
        idx[3, 0] = -1
        idx[T - 1, K - 1] = -1
    G = (ee - eb) + shared
    cap = T * K + shared * T + pad * G
    d_idx = torch.from_numpy(idx).to(gpu)
    outs = []
    for which in ("single", "multi"):
        counts = torch.full((G,), -5, dtype=torch.int32, device=gpu)
        start = torch.full((G,), -5, dtype=torch.int32, device=gpu)
        pos = torch.full((T * K,), -5, dtype=torch.int32, device=gpu)
        rowtok = torch.full((cap,), -7, dtype=torch.int32, device=gpu)
        total = torch.full((1,), -5, dtype=torch.int32, device=gpu)
        err = torch.zeros(1, dtype=torch.int32, device=gpu)
        if which == "single":
            M.check("permute_padded", k.moe_permute_padded(M.ptr(d_idx), T, K, eb, ee, shared, M.ptr(counts),
                                                           M.ptr(start), M.ptr(pos), M.ptr(rowtok), M.ptr(total),
                                                           cap, M.ptr(err), pad, stream()))
        else:
            nbytes = k.moe_permute_mb_scratch_bytes(T, K, eb, ee)
            scratch = torch.full((max(nbytes, 4),), 0x5A, dtype=torch.uint8, device=gpu)
            M.check("permute_mb", k.moe_permute_mb(M.ptr(d_idx), T, K, eb, ee, shared, M.ptr(counts), M.ptr(start),
                                                   M.ptr(pos), M.ptr(rowtok), M.ptr(total), cap, M.ptr(err), pad,
                                                   M.ptr(scratch), nbytes, stream()))
        torch.cuda.synchronize()
        assert err.item() == 0
        R = total.item()
        outs.append((counts.cpu(), start.cpu(), pos.cpu(), rowtok.cpu()[:R], R))
    a, b = outs
    assert a[4] == b[4]
    for x, y in zip(a[:4], b[:4]):
        assert torch.equal(x, y)
    if pad == 16 and eb == 0 and ee == E:
        c, st_, p_, rt, R = oracle.moe_permute(idx, E, shared)
        assert b[4] == R and np.array_equal(b[2].numpy(), p_.reshape(-1)) and np.array_equal(b[3].numpy(), rt)


def test_permute_multiblock_refuses_overflow(gpu):
    k = M.libs()["libkernels.so"]
    T, K, E = 1000, 8, 160
    idx = torch.zeros(T, K, dtype=torch.int32, device=gpu)       # all pairs to expert 0
    counts = torch.empty(E + 1, dtype=torch.int32, device=gpu)
    start = torch.empty(E + 1, dtype=torch.int32, device=gpu)
    pos = torch.empty(T * K, dtype=torch.int32, device=gpu)
    rowtok = torch.full((100,), -7, dtype=torch.int32, device=gpu)
    total = torch.empty(1, dtype=torch.int32, device=gpu)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    nbytes = k.moe_permute_mb_scratch_bytes(T, K, 0, E)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=gpu)
    M.check("permute_mb", k.moe_permute_mb(M.ptr(idx), T, K, 0, E, 1, M.ptr(counts), M.ptr(start), M.ptr(pos),
                                           M.ptr(rowtok), M.ptr(total), 100, M.ptr(err), 16, M.ptr(scratch), nbytes,
                                           stream()))
    torch.cuda.synchronize()
    assert err.item() == 2 and total.item() == -1
    assert (counts == 0).all() and (pos == -1).all() and (rowtok == -7).all()
    assert k.moe_permute_mb(M.ptr(idx), T, K, 0, E, 1, M.ptr(counts), M.ptr(start), M.ptr(pos), M.ptr(rowtok),
                            M.ptr(total), 100, M.ptr(err), 16, M.ptr(scratch), nbytes - 4, stream()) == 6


def test_permute_capacity_overflow_reports(gpu):
    k = M.libs()["libkernels.so"]
    T, K, E = 64, 4, 8
    idx = torch.randint(0, E, (T, K), dtype=torch.int32, device=gpu)
    counts = torch.empty(E, dtype=torch.int32, device=gpu)
    start = torch.empty(E, dtype=torch.int32, device=gpu)
    pos = torch.empty(T * K, dtype=torch.int32, device=gpu)
    rowtok = torch.empty(16, dtype=torch.int32, device=gpu)
    total = torch.empty(1, dtype=torch.int32, device=gpu)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    M.check("permute", k.moe_permute(M.ptr(idx), T, K, 0, E, 0, M.ptr(counts), M.ptr(start), M.ptr(pos),
                                     M.ptr(rowtok), M.ptr(total), 16, M.ptr(err), stream()))
    torch.cuda.synchronize()
    assert err.item() == 2 and total.item() == 0 and int(counts.sum()) == 0


# ---------------------------------------------------------------- grouped GEMM

def _rand_e4m3(shape, g, scale=1.0):
    return (torch.randn(*shape, generator=g) * scale).clamp(-440, 440).to(torch.float8_e4m3fn).view(torch.uint8)


def _lut():
    return torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).to(torch.float64)


def _deq(q, s):
    """e4m3 bytes [r][c] with block scales [r/128][c/128] -> float64."""
    lut = _lut()
    return lut[q.long()] * s.double().repeat_interleave(128, 0).repeat_interleave(128, 1)


def _make_groups(counts, K, Nw, g):
    G = len(counts)
    starts, row = [], 0
    for c in counts:
        starts.append(row)
        row += (c + 15) // 16 * 16
    rows = row + 32
    A = _rand_e4m3((rows, K), g)
    a_ld = (rows + 3) // 4 * 4
    A_s = (torch.rand(K // 128, a_ld, generator=g) * 0.02 + 0.001).float()
    W = _rand_e4m3((G, Nw, K), g, 0.5)
    W_s = (torch.rand(G, Nw // 128, K // 128, generator=g) * 0.01 + 0.0005).float()
    return starts, rows, A, A_s, a_ld, W, W_s


def _gemm_ref(A, A_s, W, W_s, starts, counts, K):
    lut = _lut()
    out = {}
    for gi, (st, c) in enumerate(zip(starts, counts)):
        if c == 0:
            continue
        a = lut[A[st:st + c].long()] * A_s[:, st:st + c].T.double().repeat_interleave(128, 1)
        w = _deq(W[gi], W_s[gi])
        out[gi] = a @ w.T
    return out


@pytest.mark.parametrize("counts,K,N", [([16], 384, 256), ([1, 0, 130, 255, 300], 384, 256),
                                        ([128, 129, 17, 0, 0, 1000], 384, 256), ([40, 257], 1536, 512)])
def test_grouped_gemm_down(gpu, counts, K, N):
    g = torch.Generator().manual_seed(sum(counts))
    starts, rows, A, A_s, a_ld, W, W_s = _make_groups(counts, K, N, g)
    out = torch.full((rows, N), float("nan"), dtype=torch.bfloat16, device=gpu)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    cnt = torch.tensor(counts, dtype=torch.int32, device=gpu)
    st = torch.tensor(starts, dtype=torch.int32, device=gpu)
    M.grouped_gemm(M.GEMM_DOWN_BF16, A.to(gpu), A_s.to(gpu), a_ld, W.to(gpu), W_s.to(gpu), cnt, st, out, None, 0,
                   K, N, rows, error_word=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = _gemm_ref(A, A_s, W, W_s, starts, counts, K)
    o = out.cpu().double()
    for gi, r in ref.items():
        y = o[starts[gi]:starts[gi] + counts[gi]]
        assert torch.isfinite(y).all()
        rel = (y - r).abs().max() / r.abs().max()
        assert rel < 8e-3, (gi, float(rel))


@pytest.mark.parametrize("counts,K,N", [([16], 256, 256), ([3, 0, 128, 129, 260], 256, 256), ([1000, 1], 256, 256),
                                        ([70, 300], 640, 384)])
def test_grouped_gemm_gated_swiglu(gpu, oracle, counts, K, N):
    # weights hold 2N rows: gate [0,N), up [N,2N)
    g = torch.Generator().manual_seed(7 + sum(counts))
    starts, rows, A, A_s, a_ld, W, W_s = _make_groups(counts, K, 2 * N, g)
    hq = torch.full((rows, N), 0x55, dtype=torch.uint8, device=gpu)
    hs = torch.full((N // 128, a_ld), -1.0, device=gpu)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    cnt = torch.tensor(counts, dtype=torch.int32, device=gpu)
    st = torch.tensor(starts, dtype=torch.int32, device=gpu)
    M.grouped_gemm(M.GEMM_GATED_SWIGLU, A.to(gpu), A_s.to(gpu), a_ld, W.to(gpu), W_s.to(gpu), cnt, st, hq, hs, a_ld,
                   K, N, rows, error_word=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = _gemm_ref(A, A_s, W, W_s, starts, counts, K)
    lut = _lut()
    hq_c, hs_c = hq.cpu(), hs.cpu()
    for gi, r in ref.items():
        gte, up = r[:, :N].float(), r[:, N:]
        h = (gte / (1 + torch.exp(-gte))).double() * up
        q = hq_c[starts[gi]:starts[gi] + counts[gi]]
        s = hs_c[:, starts[gi]:starts[gi] + counts[gi]].T
        deq = lut[q.long()] * s.double().repeat_interleave(128, 1)
        rel = (deq - h).abs().max() / h.abs().max()
        assert rel < 4e-2, (gi, float(rel))          # one e4m3 step is 6.25 % relative; block-max relative much less
        # the scale is exactly amax/448 of the kernel's own fp32 h: check it is consistent with its bytes
        assert (s > 0).all()
        # padding rows of the segment are zeroed
        pad_end = starts[gi] + (counts[gi] + 15) // 16 * 16
        assert (hq_c[starts[gi] + counts[gi]:pad_end] == 0).all()
        assert (hs_c[:, starts[gi] + counts[gi]:pad_end] == 0).all()


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("counts", [[1, 0, 3, 16, 31, 32, 33, 70], [0, 5, 1000, 2], [64] * 12])
def test_grouped_gemm_small_tiles(gpu, gated, counts):
    """The decode form (CBW_GEMM_SMALL_TILES: tiles of at most 32 rows, a
    deeper weight ring) and the full form on the same inputs: both within the
    float64 reference's tolerance, padding rows zeroed; reports whether they
    agree bit for bit."""
    K, N = 640, 256
    g = torch.Generator().manual_seed(31 + sum(counts) + gated)
    starts, rows, A, A_s, a_ld, W, W_s = _make_groups(counts, K, 2 * N if gated else N, g)
    cnt = torch.tensor(counts, dtype=torch.int32, device=gpu)
    st = torch.tensor(starts, dtype=torch.int32, device=gpu)
    ref = _gemm_ref(A, A_s, W, W_s, starts, counts, K)
    lut = _lut()
    outs = {}
    for form in (M.GEMM_SMALL_TILES, M.GEMM_FULL_TILES):
        err = torch.zeros(1, dtype=torch.int32, device=gpu)
        if gated:
            hq = torch.full((rows, N), 0x55, dtype=torch.uint8, device=gpu)
            hs = torch.full((N // 128, a_ld), -1.0, device=gpu)
            M.grouped_gemm(M.GEMM_GATED_SWIGLU | form, A.to(gpu), A_s.to(gpu), a_ld, W.to(gpu), W_s.to(gpu), cnt, st,
                           hq, hs, a_ld, K, N, rows, error_word=err)
            torch.cuda.synchronize()
            outs[form] = (hq.cpu(), hs.cpu())
        else:
            out = torch.full((rows, N), float("nan"), dtype=torch.bfloat16, device=gpu)
            M.grouped_gemm(M.GEMM_DOWN_BF16 | form, A.to(gpu), A_s.to(gpu), a_ld, W.to(gpu), W_s.to(gpu), cnt, st,
                           out, None, 0, K, N, rows, error_word=err)
            torch.cuda.synchronize()
            outs[form] = (out.cpu(),)
        assert err.item() == 0
        for gi, r in ref.items():
            s0, c = starts[gi], counts[gi]
            if gated:
                hq_c, hs_c = outs[form]
                gte, up = r[:, :N].float(), r[:, N:]
                h = (gte / (1 + torch.exp(-gte))).double() * up
                deq = lut[hq_c[s0:s0 + c].long()] * hs_c[:, s0:s0 + c].T.double().repeat_interleave(128, 1)
                assert (deq - h).abs().max() / h.abs().max() < 4e-2, (form, gi)
                pad_end = s0 + (c + 15) // 16 * 16
                assert (hq_c[s0 + c:pad_end] == 0).all() and (hs_c[:, s0 + c:pad_end] == 0).all()
            else:
                y = outs[form][0][s0:s0 + c].double()
                assert torch.isfinite(y).all()
                assert (y - r).abs().max() / r.abs().max() < 8e-3, (form, gi)
    same = all(torch.equal(a_, b_) for a_, b_ in zip(outs[M.GEMM_SMALL_TILES], outs[M.GEMM_FULL_TILES]))
    print(f"small vs full tiles ({'gated' if gated else 'down'}, counts {counts}): bit-identical {same}")


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("counts,K", [([16], 256), ([1, 0, 130, 255, 300, 17], 512), ([128] * 9 + [7], 768),
                                      ([1000, 3, 129], 1536)])
def test_grouped_gemm_pair_matches_one_sm(gpu, gated, counts, K):
    """The full form on CTA pairs (tcgen05 cta_group::2) and in token-major
    tiles (128 token rows x 256 weight rows per instruction) against the same
    form on one SM per tile: identical bits, and all within the float64
    reference's tolerance."""
    N = 256
    g = torch.Generator().manual_seed(101 + sum(counts) + gated)
    starts, rows, A, A_s, a_ld, W, W_s = _make_groups(counts, K, 2 * N if gated else N, g)
    cnt = torch.tensor(counts, dtype=torch.int32, device=gpu)
    st = torch.tensor(starts, dtype=torch.int32, device=gpu)
    outs = {}
    for form in (M.GEMM_PAIR_TILES, M.GEMM_ONE_SM_TILES, M.GEMM_TOKEN_TILES):
        err = torch.zeros(1, dtype=torch.int32, device=gpu)
        if gated:
            hq = torch.full((rows, N), 0x55, dtype=torch.uint8, device=gpu)
            hs = torch.full((N // 128, a_ld), -1.0, device=gpu)
            M.grouped_gemm(M.GEMM_GATED_SWIGLU | form, A.to(gpu), A_s.to(gpu), a_ld, W.to(gpu), W_s.to(gpu), cnt, st,
                           hq, hs, a_ld, K, N, rows, error_word=err)
            torch.cuda.synchronize()
            outs[form] = (hq.cpu(), hs.cpu())
        else:
            out = torch.full((rows, N), float("nan"), dtype=torch.bfloat16, device=gpu)
            M.grouped_gemm(M.GEMM_DOWN_BF16 | form, A.to(gpu), A_s.to(gpu), a_ld, W.to(gpu), W_s.to(gpu), cnt, st,
                           out, None, 0, K, N, rows, error_word=err)
            torch.cuda.synchronize()
            outs[form] = (out.cpu(),)
        assert err.item() == 0, form
    ref = _gemm_ref(A, A_s, W, W_s, starts, counts, K)
    lut = _lut()
    for gi, r in ref.items():
        s0, c = starts[gi], counts[gi]
        for form in outs:
            if gated:
                hq_c, hs_c = outs[form]
                gte, up = r[:, :N].float(), r[:, N:]
                h = (gte / (1 + torch.exp(-gte))).double() * up
                deq = lut[hq_c[s0:s0 + c].long()] * hs_c[:, s0:s0 + c].T.double().repeat_interleave(128, 1)
                assert (deq - h).abs().max() / h.abs().max() < 4e-2, (form, gi)
                pad_end = s0 + (c + 15) // 16 * 16
                assert (hq_c[s0 + c:pad_end] == 0).all() and (hs_c[:, s0 + c:pad_end] == 0).all()
            else:
                y = outs[form][0][s0:s0 + c].double()
                assert torch.isfinite(y).all()
                assert (y - r).abs().max() / r.abs().max() < 8e-3, (form, gi)
        for other in (M.GEMM_PAIR_TILES, M.GEMM_TOKEN_TILES):
            if gated:
                a_, b_ = outs[other], outs[M.GEMM_ONE_SM_TILES]
                assert torch.equal(a_[0][s0:s0 + c], b_[0][s0:s0 + c]), (other, gi)
                assert torch.equal(a_[1][:, s0:s0 + c], b_[1][:, s0:s0 + c]), (other, gi)
            else:
                a_ = outs[other][0][s0:s0 + c].view(torch.int16)
                b_ = outs[M.GEMM_ONE_SM_TILES][0][s0:s0 + c].view(torch.int16)
                assert torch.equal(a_, b_), (other, gi)


@pytest.mark.parametrize("x2", [False, True])
@pytest.mark.parametrize("counts,K", [([16], 256), ([1, 0, 130, 255, 300, 17], 512), ([1000, 3, 129], 1536)])
def test_grouped_gemm_row_out_scatters_rows(gpu, counts, K, x2):
    """cbwFp8BlockScaledGroupedGemmRowOut (the down projection storing rows at
    per-row addresses, the expert-parallel return): every row with an address
    lands there with the bits the token-major form writes to out, rows without
    one go to out, and no other byte of either buffer changes."""
    N = 512
    g = torch.Generator().manual_seed(303 + sum(counts) + x2)
    starts, rows, A, A_s, a_ld, W, W_s = _make_groups(counts, K, N, g)
    A2 = torch.cat([A, torch.randint(0, 256, A.shape, generator=g, dtype=torch.uint8) & 0x77]) if x2 else A
    mode = M.GEMM_DOWN_BF16 | M.GEMM_TOKEN_TILES | (M.GEMM_ACT_X2 if x2 else 0)
    cnt = torch.tensor(counts, dtype=torch.int32, device=gpu)
    st = torch.tensor(starts, dtype=torch.int32, device=gpu)
    args = (A2.to(gpu), A_s.to(gpu), a_ld, W.to(gpu), W_s.to(gpu), cnt, st)
    err = torch.zeros(1, dtype=torch.int32, device=gpu)
    ref = torch.full((rows, N), float("nan"), dtype=torch.bfloat16, device=gpu)
    M.grouped_gemm(mode, *args, ref, None, 0, K, N, rows, error_word=err)
    # every other live row goes to a second buffer at a shuffled position
    live = [s0 + i for s0, c in zip(starts, counts) for i in range(c)]
    far = torch.full((rows + 7, N), -3.0, dtype=torch.bfloat16, device=gpu)
    perm = torch.randperm(rows + 7, generator=g).tolist()
    addr = torch.zeros(rows, dtype=torch.int64)
    sent = {}
    for j, r in enumerate(live):
        if j % 2 == 0:
            sent[r] = perm[j]
            addr[r] = far.data_ptr() + perm[j] * N * 2
    out = torch.full((rows, N), -5.0, dtype=torch.bfloat16, device=gpu)
    M.grouped_gemm(mode, *args, out, None, 0, K, N, rows, error_word=err, row_out=addr.to(gpu))
    torch.cuda.synchronize()
    assert err.item() == 0
    ref_c, out_c, far_c = ref.cpu().view(torch.int16), out.cpu().view(torch.int16), far.cpu().view(torch.int16)
    untouched_out = torch.full((N,), -5.0, dtype=torch.bfloat16).view(torch.int16)
    untouched_far = torch.full((N,), -3.0, dtype=torch.bfloat16).view(torch.int16)
    for r in live:
        if r in sent:
            assert torch.equal(far_c[sent[r]], ref_c[r]), r
            assert torch.equal(out_c[r], untouched_out), r
        else:
            assert torch.equal(out_c[r], ref_c[r]), r
    targets = set(sent.values())
    for q in range(rows + 7):
        if q not in targets:
            assert torch.equal(far_c[q], untouched_far), q
    liveset = set(live)
    for r in range(rows):
        if r not in liveset:
            assert torch.equal(out_c[r], untouched_out), r
    # a form that takes no row addresses is refused, nothing launched
    with pytest.raises(M.MoEError):
        M.grouped_gemm(M.GEMM_DOWN_BF16 | M.GEMM_ONE_SM_TILES, A.to(gpu), A_s.to(gpu), a_ld, W.to(gpu), W_s.to(gpu),
                       cnt, st, out, None, 0, K, N, rows, error_word=err, row_out=addr.to(gpu))


@pytest.mark.parametrize("gated", [False, True])
def test_grouped_gemm_small_tiles_placement_independent(gpu, gated):
    """The decode form's result for a row does not depend on where its tile
    runs: the same expert groups, run (a) twice and (b) after two extra
    leading groups that shift every tile to other CTAs and other positions in
    each CTA's K-block sequence, give bit-identical outputs."""
    K, N = 640, 256
    Nw = 2 * N if gated else N
    counts = [1, 7, 33, 64, 64, 20, 0, 31]
    pre = [45, 200]
    g = torch.Generator().manual_seed(77 + gated)
    starts, rows, A, A_s, a_ld, W, W_s = _make_groups(counts, K, Nw, g)
    p_starts, p_rows, pA, pA_s, p_ld, pW, pW_s = _make_groups(pre, K, Nw, g)
    p_used = p_starts[-1] + (pre[-1] + 15) // 16 * 16          # rows the prefix groups occupy
    A2 = torch.cat([pA[:p_used], A])
    rows2 = A2.shape[0]
    a_ld2 = (rows2 + 3) // 4 * 4
    A_s2 = torch.zeros(K // 128, a_ld2)
    A_s2[:, :p_used] = pA_s[:, :p_used]
    A_s2[:, p_used:p_used + rows] = A_s[:, :rows]
    W2, W_s2 = torch.cat([pW, W]), torch.cat([pW_s, W_s])
    starts2 = p_starts + [p_used + s_ for s_ in starts]
    counts2 = pre + counts

    def run(A_, A_s_, ld_, W_, W_s_, starts_, counts_, rows_):
        err = torch.zeros(1, dtype=torch.int32, device=gpu)
        cnt = torch.tensor(counts_, dtype=torch.int32, device=gpu)
        st = torch.tensor(starts_, dtype=torch.int32, device=gpu)
        form = M.GEMM_SMALL_TILES
        if gated:
            hq = torch.zeros((rows_, N), dtype=torch.uint8, device=gpu)
            hs = torch.zeros((N // 128, ld_), device=gpu)
            M.grouped_gemm(M.GEMM_GATED_SWIGLU | form, A_.to(gpu), A_s_.to(gpu), ld_, W_.to(gpu), W_s_.to(gpu), cnt,
                           st, hq, hs, ld_, K, N, rows_, error_word=err)
            torch.cuda.synchronize()
            assert err.item() == 0
            return hq.cpu(), hs.cpu()
        out = torch.zeros((rows_, N), dtype=torch.bfloat16, device=gpu)
        M.grouped_gemm(M.GEMM_DOWN_BF16 | form, A_.to(gpu), A_s_.to(gpu), ld_, W_.to(gpu), W_s_.to(gpu), cnt, st,
                       out, None, 0, K, N, rows_, error_word=err)
        torch.cuda.synchronize()
        assert err.item() == 0
        return (out.cpu(),)

    first = run(A, A_s, a_ld, W, W_s, starts, counts, rows)
    again = run(A, A_s, a_ld, W, W_s, starts, counts, rows)
    shifted = run(A2, A_s2, a_ld2, W2, W_s2, starts2, counts2, rows2)
    for gi, c in enumerate(counts):
        s0, s1 = starts[gi], starts2[len(pre) + gi]
        if gated:
            for a_, b_ in ((first, again), (first, shifted)):
                off = 0 if b_ is again else s1 - s0
                assert torch.equal(a_[0][s0:s0 + c], b_[0][s0 + off:s0 + off + c]), gi
                assert torch.equal(a_[1][:, s0:s0 + c], b_[1][:, s0 + off:s0 + off + c]), gi
        else:
            assert torch.equal(first[0][s0:s0 + c].view(torch.int16), again[0][s0:s0 + c].view(torch.int16)), gi
            assert torch.equal(first[0][s0:s0 + c].view(torch.int16), shifted[0][s1:s1 + c].view(torch.int16)), gi


# ---------------------------------------------------------------- full layer

def _run_layer(shape, case, T, dev, routing=None):
    layer = M.MoELayer(shape, to_dev(case, dev), max_tokens=max(T, 1))
    x = case["x"].to(dev)
    out = layer.forward(x, routing=routing)
    torch.cuda.synchronize()
    layer.check_error()
    idx, w, counts = layer.last_routing(T)
    return layer, out, idx, w, counts


@pytest.mark.parametrize("T", [64, 1, 50, 200])
def test_layer_tiny_config(gpu, oracle, T):
    """BASELINE configs[0] shapes (hidden 256, 8 experts top-2 + shared,
    intermediate 512); T = 2 x 32 is the configured batch."""
    shape = synth.TINY
    case = synth.make_case(shape, T, seed=0)
    _, out, idx, w, _ = _run_layer(shape, case, T, gpu)
    ow = oracle.OracleWeights(shape, case)
    ref, oidx, ow_, _ = oracle.moe_ffn_forward(ow, bits(case["x"]), mode=0)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert np.allclose(w.cpu().numpy(), ow_, rtol=2e-6, atol=1e-7)
    y = out.float().cpu().numpy().astype(np.float64)
    mr, mae = oracle.max_rel_and_mae(y, oracle.bf16_bits_to_f32(ref))
    assert mr <= MAX_REL and mae <= MAE, (mr, mae)
    # against the reference's semantics (fp32 activations, oracle "ref" mode): at this
    # configuration the e4m3 activations stay within the north-star bar as well
    refm, ridx, *_ = oracle.moe_ffn_forward(ow, bits(case["x"]), mode=1)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    mr1, mae1 = oracle.max_rel_and_mae(y, oracle.bf16_bits_to_f32(refm))
    print(f"tiny T={T}: vs q mode {mr:.2e}/{mae:.2e}, vs ref mode (fp32 activations) {mr1:.2e}/{mae1:.2e}")
    assert mr1 <= MAX_REL and mae1 <= MAE, (mr1, mae1)


def test_layer_zipf_bias_and_routed_entry(gpu, oracle):
    shape = synth.TINY
    T = 96
    case = synth.make_case(shape, T, seed=3, zipf_bias=True)
    _, out, idx, w, counts = _run_layer(shape, case, T, gpu)
    ow = oracle.OracleWeights(shape, case)
    ref, oidx, _, _ = oracle.moe_ffn_forward(ow, bits(case["x"]), mode=0)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    assert counts[: shape.num_experts].sum().item() == T * shape.top_k
    mr, mae = oracle.max_rel_and_mae(out.float().cpu().numpy(), oracle.bf16_bits_to_f32(ref))
    assert mr <= MAX_REL and mae <= MAE
    # same routing supplied by the caller -> identical output
    _, out2, _, _, _ = _run_layer(shape, case, T, gpu, routing=(idx.to(gpu), w.to(gpu)))
    assert torch.equal(out2.cpu(), out.cpu())


def test_layer_all_tokens_one_expert(gpu, oracle):
    """A router bias that sends every token to experts 0..k-1: maximal group,
    all other experts empty."""
    shape = synth.TINY
    T = 300
    case = synth.make_case(shape, T, seed=4)
    case["router_bias"] = torch.tensor([100.0, 90.0] + [0.0] * (shape.num_experts - 2))
    _, out, idx, _, counts = _run_layer(shape, case, T, gpu)
    assert (idx.cpu()[:, 0] == 0).all() and (idx.cpu()[:, 1] == 1).all()
    ow = oracle.OracleWeights(shape, case)
    ref, *_ = oracle.moe_ffn_forward(ow, bits(case["x"]), mode=0)
    mr, mae = oracle.max_rel_and_mae(out.float().cpu().numpy(), oracle.bf16_bits_to_f32(ref))
    assert mr <= MAX_REL and mae <= MAE


def test_layer_deterministic(gpu):
    shape = synth.TINY
    case = synth.make_case(shape, 64, seed=9)
    layer = M.MoELayer(shape, to_dev(case, gpu), max_tokens=64)
    x = case["x"].to(gpu)
    a = layer.forward(x).clone()
    b = layer.forward(x).clone()
    assert torch.equal(a, b)


def test_layer_glm_shape_sampled_tokens(gpu, oracle):
    """BASELINE configs[1] at full size (hidden 5120, 160 experts top-8 + shared,
    intermediate 1536, 4096 tokens, zipf-skewed router): the whole layer runs
    on the GPU; the oracle recomputes 256 sampled tokens (tokens are independent
    given the weights), and routing is checked bit-exact for all tokens.

    Against the oracle's e4m3-activation mirror ("q" mode) the outputs meet the
    north-star bar.  Against the reference's semantics (fp32 activations, "ref"
    mode) they do not: the e4m3 activations the north star specifies (1x128
    scales, 3 mantissa bits) round each activation by up to 6.25 % (about
    3.6 % RMS), and at this shape the MoE output differs from the
    fp32-activation one by max-rel ~3e-2 and MAE ~4e-2 (measured on the CPU
    oracle: q vs ref on 64 tokens, 3.2e-2 / 4.0e-2).  That gap is asserted to
    stay at its measured size (bound 5e-2 / 5e-2), and printed."""
    shape = synth.GLM
    T = 4096
    w = synth.make_moe_weights(shape, seed=0, device=gpu, zipf_bias=True)
    x = synth.make_x(shape, T, seed=1, device=gpu)
    layer = M.MoELayer(shape, w, max_tokens=T)
    out = layer.forward(x)
    torch.cuda.synchronize()
    layer.check_error()
    idx, wts, counts = layer.last_routing(T)
    assert counts[: shape.num_experts].sum().item() == T * shape.top_k
    assert counts[shape.num_experts].item() == T
    xf = x.float().cpu().numpy()
    n = oracle.rmsnorm_ref(xf, w["gamma"].cpu().numpy(), shape.eps)
    lg = oracle.moe_gate_ref(n, w["router_w"].cpu().numpy(), w["router_bias"].cpu().numpy())
    oi, _ = oracle.moe_topk_ref(lg, shape.top_k)
    assert np.array_equal(idx.cpu().numpy(), oi)
    sample = np.random.default_rng(0).choice(T, 256, replace=False)
    case = {k_: v for k_, v in w.items()}
    ow = oracle.OracleWeights(shape, case)
    xs = bits(x.cpu()[sample])
    ref, *_ = oracle.moe_ffn_forward(ow, xs, mode=0)
    y = out.cpu()[sample].float().numpy()
    mr, mae = oracle.max_rel_and_mae(y, oracle.bf16_bits_to_f32(ref))
    assert mr <= MAX_REL and mae <= MAE, (mr, mae)
    refm, *_ = oracle.moe_ffn_forward(ow, xs, mode=1)
    mr1, mae1 = oracle.max_rel_and_mae(y, oracle.bf16_bits_to_f32(refm))
    print(f"GLM 256 sampled tokens: vs q mode {mr:.2e}/{mae:.2e}, vs ref mode (fp32 activations) "
          f"{mr1:.2e}/{mae1:.2e}")
    assert mr1 <= 5e-2 and mae1 <= 5e-2, (mr1, mae1)
