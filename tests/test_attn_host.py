"""Host-side checks of the tensor-parallel attention block (no GPU):
the per-rank weight slices reassemble the model, and the TP decomposition
holds across real process ranks -- each `gloo` rank computes its oracle
partial for its heads (oracle.attn_block_partial_ref), the partials are
exchanged over the process group and summed in rank order with the residual,
and the result matches the unsharded oracle step within the bf16 bar."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from time_b200 import synth

SHAPE = synth.AttnShape(hidden=256, num_q_heads=4, num_kv_heads=2)
PS, D = 16, 128


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case(seed=4):
    rng = np.random.default_rng(seed)
    w = synth.make_attn_weights(SHAPE, seed=seed)
    B, ctx = 2, [20, 5]
    pages = 6
    kc = rng.standard_normal((pages, PS, SHAPE.num_kv_heads, D)).astype(np.float32)
    vc = rng.standard_normal((pages, PS, SHAPE.num_kv_heads, D)).astype(np.float32)
    # caches hold bf16 values
    kc = torch.from_numpy(kc).to(torch.bfloat16).float().numpy()
    vc = torch.from_numpy(vc).to(torch.bfloat16).float().numpy()
    pt = np.array([[0, 1], [2, 3]], dtype=np.int32)
    x = torch.from_numpy(rng.standard_normal((B, SHAPE.hidden)).astype(np.float32)).to(torch.bfloat16).float().numpy()
    return w, kc, vc, pt, ctx, x


def _np(w):
    return {k: v.numpy() for k, v in w.items()}


def test_rank_slices_reassemble_the_model():
    w = synth.make_attn_weights(SHAPE, seed=1)
    tp, d = 2, D
    nq, nkv = SHAPE.num_q_heads // tp, SHAPE.num_kv_heads // tp
    parts = [synth.attn_rank_slice(w, SHAPE, tp, r) for r in range(tp)]
    q = torch.cat([p["w_qkv"][:nq * d] for p in parts])
    k = torch.cat([p["w_qkv"][nq * d:(nq + nkv) * d] for p in parts])
    v = torch.cat([p["w_qkv"][(nq + nkv) * d:] for p in parts])
    assert torch.equal(q, w["w_q"]) and torch.equal(k, w["w_k"]) and torch.equal(v, w["w_v"])
    assert torch.equal(torch.cat([p["w_o"] for p in parts], dim=1), w["w_o"])
    assert torch.equal(torch.cat([p["s_o"] for p in parts], dim=1), w["s_o"])
    sq = torch.cat([p["s_qkv"][:nq * d // 128] for p in parts])
    assert torch.equal(sq, w["s_q"])


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from oracle import oracle as O
        w, kc, vc, pt, ctx, x = _case()
        nkv_l = SHAPE.num_kv_heads // world
        wr = _np(synth.attn_rank_slice(w, SHAPE, world, rank))
        # this rank's KV heads of the caches
        kr = np.ascontiguousarray(kc[:, :, rank * nkv_l:(rank + 1) * nkv_l])
        vr = np.ascontiguousarray(vc[:, :, rank * nkv_l:(rank + 1) * nkv_l])
        part = O.attn_block_partial_ref(wr, x, ctx, pt, kr, vr, SHAPE.num_q_heads // world, nkv_l,
                                        SHAPE.rotary_dim, SHAPE.rope_theta, SHAPE.eps)
        parts = [torch.empty(part.shape) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(part))
        s = np.zeros_like(x)
        for p in parts:                       # rank order, fp32
            s = s + p.numpy()
        out = O.bf16_round(x + s)
        full = O.attn_block_partial_ref(_np(synth.attn_rank_slice(w, SHAPE, 1, 0)), x, ctx, pt, kc.copy(), vc.copy(),
                                        SHAPE.num_q_heads, SHAPE.num_kv_heads, SHAPE.rotary_dim, SHAPE.rope_theta,
                                        SHAPE.eps)
        ref = O.bf16_round(x + full)
        diff = np.abs(out - ref)
        assert diff.max() <= 1e-2 * np.abs(ref).max() and diff.mean() <= 2e-3, (diff.max(), diff.mean())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as exc:
        q.put((rank, repr(exc)))


def test_tp_decomposition_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, msg = q.get(timeout=180)
            results[r] = msg
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert all(m == "ok" for m in results.values()), results
