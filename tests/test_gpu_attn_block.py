"""The decode attention block (attn_block_decode / _partial) against the
oracle's composition of the same step (oracle.attn_block_partial_ref):
rmsnorm -> FP8 QKV -> partial RoPE + page write -> decode attention -> FP8
o_proj -> sum over TP ranks + residual.  TP ranks are emulated on one GPU by
running each rank's partial and summing them with attn_tp_reduce_residual (the
real multi-GPU reduce is tests/test_gpu_attn_tp.py).  Tolerance: the layer bar
of the spec on bf16 outputs (max |diff| / max |ref| <= 1e-2, MAE <= 2e-3)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from time_b200 import attn as A
from time_b200 import synth

pytestmark = pytest.mark.gpu

PS, D = 16, 128


def np_w(w: dict) -> dict:
    return {k: v.cpu().numpy() for k, v in w.items()}


def setup_case(shape, tp, B, ctx, seed, dev):
    """Whole-model weights, per-rank caches prefilled for positions < ctx[b],
    page tables (disjoint pages), positions = ctx (the new token)."""
    rng = np.random.default_rng(seed)
    w_all = synth.make_attn_weights(shape, seed=seed, device=dev)
    nkv_l = shape.num_kv_heads // tp
    max_pages = max(-(-(c + 1) // PS) for c in ctx) + 1
    num_pages = sum(-(-(c + 1) // PS) for c in ctx) + 3
    perm = rng.permutation(num_pages)
    pt = np.full((B, max_pages), -1, dtype=np.int32)
    o = 0
    for b, c in enumerate(ctx):
        n = -(-(c + 1) // PS)
        pt[b, :n] = perm[o:o + n]
        o += n
    caches = []
    for r in range(tp):
        kc = torch.from_numpy(rng.standard_normal((num_pages, PS, nkv_l, D)).astype(np.float32)).to(torch.bfloat16)
        vc = torch.from_numpy(rng.standard_normal((num_pages, PS, nkv_l, D)).astype(np.float32)).to(torch.bfloat16)
        caches.append((kc.to(dev), vc.to(dev)))
    x = torch.from_numpy(rng.standard_normal((B, shape.hidden)).astype(np.float32)).to(torch.bfloat16).to(dev)
    return w_all, caches, pt, max_pages, x


def oracle_out(shape, tp, w_all, caches, pt, ctx, x):
    nq_l, nkv_l = shape.num_q_heads // tp, shape.num_kv_heads // tp
    xf = x.float().cpu().numpy()
    s = np.zeros_like(xf)
    for r in range(tp):
        wr = np_w(synth.attn_rank_slice(w_all, shape, tp, r))
        kc, vc = (c.float().cpu().numpy() for c in caches[r])
        s = s + O.attn_block_partial_ref(wr, xf, ctx, pt, kc, vc, nq_l, nkv_l, shape.rotary_dim, shape.rope_theta,
                                         shape.eps)
    return O.bf16_round(xf + s)


def check(got: torch.Tensor, ref: np.ndarray):
    g = got.float().cpu().numpy()
    diff = np.abs(g - ref)
    assert diff.max() <= 1e-2 * np.abs(ref).max(), (diff.max(), np.abs(ref).max())
    assert diff.mean() <= 2e-3, diff.mean()


@pytest.mark.parametrize("shape,tp,ctx", [
    (synth.AttnShape(hidden=512, num_q_heads=4, num_kv_heads=1), 1, [5, 40, 100]),
    (synth.AttnShape(hidden=512, num_q_heads=8, num_kv_heads=2), 2, [0, 17, 300, 1023]),
    (synth.AttnShape(hidden=1024, num_q_heads=16, num_kv_heads=2, rotary_dim=128), 2, [64, 65]),
])
def test_block_matches_oracle(gpu, shape, tp, ctx):
    B = len(ctx)
    w_all, caches, pt, max_pages, x = setup_case(shape, tp, B, ctx, seed=tp * 10 + B, dev=gpu)
    ref = oracle_out(shape, tp, w_all, caches, pt, ctx, x)      # before the GPU writes the caches
    pos = torch.tensor(ctx, dtype=torch.int32, device=gpu)
    ptd = torch.from_numpy(pt).to(gpu)
    parts = []
    blocks = []
    for r in range(tp):
        blk = A.AttnBlock(shape, synth.attn_rank_slice(w_all, shape, tp, r), max_batch=B, max_pages_per_seq=max_pages,
                          max_context=max_pages * PS, tp_size=tp, tp_rank=r)
        blocks.append(blk)
        if tp == 1:
            out = blk.decode(x, pos, ptd, *caches[r])
        else:
            parts.append(blk.decode_partial(x, pos, ptd, *caches[r]))
    if tp > 1:
        out = A.tp_reduce_residual(parts, x)
    torch.cuda.synchronize()
    for blk in blocks:
        blk.check_error()
        blk.close()
    check(out, ref)


def test_block_glm_shape_tp8_emulated(gpu):
    """Config 4 per-rank shapes (hidden 5120, 12 query heads and 1 KV head per
    rank, rotary 64 of 128, theta 1e6) for 3 sequences, 8 ranks emulated."""
    shape, tp, ctx = synth.GLM_ATTN, 8, [1024, 1500, 2047]
    B = len(ctx)
    w_all, caches, pt, max_pages, x = setup_case(shape, tp, B, ctx, seed=5, dev=gpu)
    ref = oracle_out(shape, tp, w_all, caches, pt, ctx, x)
    pos = torch.tensor(ctx, dtype=torch.int32, device=gpu)
    ptd = torch.from_numpy(pt).to(gpu)
    parts = []
    for r in range(tp):
        blk = A.AttnBlock(shape, synth.attn_rank_slice(w_all, shape, tp, r), max_batch=64, max_pages_per_seq=max_pages,
                          max_context=max_pages * PS, tp_size=tp, tp_rank=r)
        parts.append(blk.decode_partial(x, pos, ptd, *caches[r]))
        torch.cuda.synchronize()
        blk.check_error()
        blk.close()
    check(A.tp_reduce_residual(parts, x), ref)


@pytest.mark.parametrize("shape,ctx", [
    # more than 64 rows: the projections run on the tcgen05 grouped GEMM
    (synth.AttnShape(hidden=512, num_q_heads=4, num_kv_heads=1), list(np.random.default_rng(2).integers(0, 200, 96))),
    # one GPU's GLM weights (QKV 14336 x 5120, o_proj 5120 x 12288) at a decode batch: grouped GEMM too
    (synth.GLM_ATTN, [100, 517, 1000]),
])
def test_block_grouped_gemm_path(gpu, shape, ctx):
    ctx = [int(c) for c in ctx]
    B = len(ctx)
    w_all, caches, pt, max_pages, x = setup_case(shape, 1, B, ctx, seed=B, dev=gpu)
    ref = oracle_out(shape, 1, w_all, caches, pt, ctx, x)
    blk = A.AttnBlock(shape, synth.attn_rank_slice(w_all, shape, 1, 0), max_batch=max(B, 4),
                      max_pages_per_seq=max_pages, max_context=max_pages * PS)
    out = blk.decode(x, torch.tensor(ctx, dtype=torch.int32, device=gpu), torch.from_numpy(pt).to(gpu), *caches[0])
    torch.cuda.synchronize()
    blk.check_error()
    blk.close()
    check(out, ref)
