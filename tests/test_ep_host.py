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


def _worker_token_rows(rank, world, port, T, E, K, seed, q):
    """The NVLink peer exchange's layout on gloo ranks: each token travels once
    per destination rank (numbered per destination in token order), every
    pair carries the index of its row in the destination's receive buffer
    (the pair map), and the receiver reading pair i's row through the map
    finds the token of the pair-level exchange's row i."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from time_b200 import synth
        epr = E // world
        idx_all = _global_routing(T, E, K, seed)
        t0, t1 = synth.token_slice(T, world, rank)
        idx = idx_all[t0:t1]
        Tr = t1 - t0
        flat = idx.reshape(-1)
        pairs = np.nonzero(flat >= 0)[0]
        order = pairs[np.argsort(flat[pairs], kind="stable")]          # dense send order
        ecounts = np.bincount(flat[flat >= 0], minlength=E).astype(np.int64)
        srows = [int(ecounts[d * epr:(d + 1) * epr].sum()) for d in range(world)]
        # per-destination numbering of this rank's tokens (ep_unique_kernel)
        uidx = np.full((world, Tr), -1, dtype=np.int64)
        utok = [[] for _ in range(world)]
        for t in range(Tr):
            for d in sorted({int(e) // epr for e in idx[t] if e >= 0}):
                uidx[d, t] = len(utok[d])
                utok[d].append(t)
        ucount = torch.tensor([len(u) for u in utok], dtype=torch.int64)
        table = [torch.empty_like(ucount) for _ in range(world)]            # every rank's row counts
        dist.all_gather(table, ucount)
        U = torch.stack(table).numpy()                                       # U[s][d]
        ubefore = [int(U[:rank, d].sum()) for d in range(world)]            # where my rows land on d
        # rows: one per (destination, token), carrying the global token id
        rows_out = torch.tensor([t0 + t for d in range(world) for t in utok[d]], dtype=torch.int64)
        rrows_u = [int(U[s, rank]) for s in range(world)]
        rows_in = torch.empty(sum(rrows_u), dtype=torch.int64)
        dist.all_to_all_single(rows_in, rows_out, output_split_sizes=rrows_u,
                               input_split_sizes=[len(u) for u in utok])
        # pair map: for every sent pair (send order), its row in the destination's recv
        pmap_out = []
        for r in order:
            d = int(flat[r]) // epr
            pmap_out.append(ubefore[d] + int(uidx[d, r // K]))
        recv = torch.empty(E, dtype=torch.int64)
        dist.all_to_all_single(recv, torch.from_numpy(ecounts))
        rrows = [int(v) for v in recv.view(world, epr).sum(1)]
        pmap_in = torch.empty(sum(rrows), dtype=torch.int64)
        dist.all_to_all_single(pmap_in, torch.tensor(pmap_out, dtype=torch.int64), output_split_sizes=rrows,
                               input_split_sizes=srows)
        # the pair-level exchange of the same pairs, for comparison
        gid = torch.from_numpy((t0 * K + order).astype(np.int64))
        got = torch.empty(sum(rrows), dtype=torch.int64)
        dist.all_to_all_single(got, gid, output_split_sizes=rrows, input_split_sizes=srows)
        pm, rin = pmap_in.numpy(), rows_in.numpy()
        assert (pm >= 0).all() and (pm < len(rin)).all()
        assert np.array_equal(rin[pm], got.numpy() // K), rank
        assert len(rin) <= len(got)                                          # never more rows than pairs
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException as exc:   # report to the parent instead of hanging it
        q.put((rank, repr(exc)))


@pytest.mark.parametrize("world,T,E,K", [(2, 200, 160, 8), (4, 64, 160, 8), (2, 1, 16, 4)])
def test_ep_token_rows_layout_gloo(world, T, E, K):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_token_rows, args=(r, world, port, T, E, K, 13, q)) for r in range(world)]
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
