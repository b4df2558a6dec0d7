"""Host side of the expert-parallel exchange on CPU: two `gloo` ranks (no GPU)
route their own tokens, exchange per-expert counts with an all-to-all, plan
both exchanges with the library's moe_ep_plan_host (libkernels.so, C), move
pair ids with gloo all-to-alls split exactly as the plan says, and check the
documented layout:

  * what rank a plans to send to b equals what b plans to receive from a;
  * the rows a rank receives for each local expert, source rank by source
    rank, are that expert's pairs in global (token, slot) order -- the order
    of the single-GPU permutation (moe_permute), so the GEMM rows match;
  * the combine exchange returns every pair's row to its owner at the row the
    dispatch sent it from (the combine reads it there).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _global_routing(T, E, K, seed):
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.choice(E, size=K, replace=False) for _ in range(T)]).astype(np.int32)
    idx[rng.random((T, K)) < 0.02] = -1          # a few invalid slots (NaN logits give -1)
    return idx


def _worker(rank, world, port, T, E, K, seed, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from time_b200 import moe as M
        from time_b200 import synth
        epr = E // world
        idx_all = _global_routing(T, E, K, seed)
        t0, t1 = synth.token_slice(T, world, rank)
        idx = idx_all[t0:t1]
        # dense send order: stable sort of own pairs by global expert (moe_permute_padded, pad 1)
        flat = idx.reshape(-1)
        pairs = np.nonzero(flat >= 0)[0]
        order = pairs[np.argsort(flat[pairs], kind="stable")]
        ecounts = np.bincount(flat[flat >= 0], minlength=E).astype(np.int32)
        recv = torch.empty(E, dtype=torch.int32)
        dist.all_to_all_single(recv, torch.from_numpy(ecounts))
        recv_counts = recv.numpy().reshape(world, epr)
        srows, soff, rrows, roff, stot, rtot = M.ep_plan_host(world, epr, ecounts, recv_counts)
        assert stot == len(order) and rtot == int(recv_counts.sum())
        # plans agree pairwise
        plan = torch.tensor([srows, rrows], dtype=torch.int64)
        plans = [torch.empty_like(plan) for _ in range(world)]
        dist.all_gather(plans, plan)
        for b in range(world):
            assert int(plans[rank][0][b]) == int(plans[b][1][rank])
        # dispatch global pair ids
        gid = torch.from_numpy((t0 * K + order).astype(np.int64))
        got = torch.empty(rtot, dtype=torch.int64)
        dist.all_to_all_single(got, gid, output_split_sizes=list(rrows), input_split_sizes=list(srows))
        got = got.numpy()
        # receiver layout: local expert j = sources 0.. in order, each its (s, j) block
        gflat = idx_all.reshape(-1)
        for j in range(epr):
            e = rank * epr + j
            seg = []
            for s in range(world):
                base = roff[s] + int(recv_counts[s, :j].sum())
                seg.extend(got[base: base + int(recv_counts[s, j])].tolist())
            expect = np.nonzero(gflat == e)[0].tolist()
            assert seg == expect, (rank, j)
        # combine: send each received row back; the owner must find pair p at its send row
        back = torch.empty(stot, dtype=torch.int64)
        dist.all_to_all_single(back, torch.from_numpy(got), output_split_sizes=list(srows),
                               input_split_sizes=list(rrows))
        spos = np.full(flat.size, -1)
        spos[order] = np.arange(len(order))
        for p in range(flat.size):
            if flat[p] >= 0:
                assert int(back[spos[p]]) == t0 * K + p
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as exc:   # report to the parent instead of hanging it
        q.put((rank, repr(exc)))


@pytest.mark.parametrize("world,T,E,K", [(2, 37, 8, 2), (2, 200, 160, 8), (2, 1, 16, 4)])
def test_ep_exchange_gloo(world, T, E, K):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, E, K, 11, q)) for r in range(world)]
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
    assert results == {r: "ok" for r in range(world)}, results


def test_plan_host_rejects_negative_counts():
    from time_b200 import moe as M
    with pytest.raises(M.MoEError):
        M.ep_plan_host(2, 2, [1, 2, -1, 0], [0, 0, 0, 0])


def test_plan_host_offsets():
    from time_b200 import moe as M
    srows, soff, rrows, roff, st, rt = M.ep_plan_host(3, 2, [1, 2, 0, 0, 5, 1], [3, 0, 1, 1, 0, 2])
    assert srows == [3, 0, 6] and soff == [0, 3, 3] and st == 9
    assert rrows == [3, 2, 2] and roff == [0, 3, 5] and rt == 7


def test_balanced_placement_is_even_permutation():
    import random
    from time_b200 import synth
    rng = random.Random(3)
    E, ep = 160, 8
    load = [int(1000 * rng.random() ** 4) for _ in range(E)]
    slot = synth.balanced_placement(load, ep)
    assert sorted(slot) == list(range(E))
    per = E // ep
    rank_load = [sum(load[e] for e in range(E) if slot[e] // per == r) for r in range(ep)]
    contiguous = [sum(load[r * per:(r + 1) * per]) for r in range(ep)]
    assert max(rank_load) <= max(contiguous)
    assert max(rank_load) - min(rank_load) <= max(load)       # LPT bound with equal slot counts
    # within a rank the experts keep ascending order
    for r in range(ep):
        mine = sorted((slot[e], e) for e in range(E) if slot[e] // per == r)
        assert [e for _, e in mine] == sorted(e for _, e in mine)


def test_expert_slice_follows_placement():
    import torch
    from time_b200 import synth
    shape = synth.TINY
    w = synth.make_moe_weights(shape, seed=0)
    slot = [3, 0, 6, 1, 4, 7, 2, 5]                 # expert -> slot, 2 ranks of 4 slots
    for r in range(2):
        ws = synth.expert_slice(w, shape, 2, r, slot_of_expert=slot)
        experts = sorted(range(8), key=lambda e: slot[e])[4 * r:4 * r + 4]
        for j, e in enumerate(experts):
            assert torch.equal(ws["w13"][j], w["w13"][e]) and torch.equal(ws["s2"][j], w["s2"][e])
        assert torch.equal(ws["w13"][4], w["w13"][8])          # shared expert last
