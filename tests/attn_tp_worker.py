"""One rank of the tensor-parallel decode attention block over real GPUs
(launched by test_gpu_attn_tp.py, or by hand for timing, under
torch.distributed.run, one process per GPU).

Every rank builds the same seeded whole-model weights and keeps its heads,
its own seeded KV cache, and the same tokens; the block runs with the TP sum
over NVLink peer memory.  Check mode: two decode steps; every rank's output
must be bit-identical to rank 0's, and rank 0 recomputes all ranks on its own
GPU (each rank's partial, then attn_tp_reduce_residual in rank order) which
must give the same bits.  Prints ATTN_TP_OK.  Timing mode (--time K): K timed
steps after 3 warm-ups, CUDA events, max over ranks, one JSON line from rank 0.
"""
import argparse
import datetime
import json
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import numpy as np
import torch
import torch.distributed as dist

from time_b200 import attn as A
from time_b200 import synth

PS, D = 16, 128


def rank_cache(rank, num_pages, nkv_l, dev):
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    kc = torch.randn(num_pages, PS, nkv_l, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(num_pages, PS, nkv_l, D, generator=g, device=dev).to(torch.bfloat16)
    return kc, vc


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", choices=["small", "glm"], default="glm")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--ctx-min", type=int, default=1024)
    ap.add_argument("--ctx-max", type=int, default=4096)
    ap.add_argument("--time", type=int, default=0, help="timed steps (0: parity check)")
    ap.add_argument("--graph", action="store_true", help="capture one step in a CUDA graph and replay it")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    shape = synth.GLM_ATTN if a.shape == "glm" else synth.AttnShape(hidden=1024, num_q_heads=16, num_kv_heads=world)
    tp, B = world, a.batch
    nkv_l = shape.num_kv_heads // tp
    rng = np.random.default_rng(7)
    ctx = rng.integers(a.ctx_min, a.ctx_max + 1, size=B)
    steps = 2 if a.time == 0 else 3 + a.time
    max_pages = int(-(-(ctx.max() + steps) // PS))
    pages = (ctx + steps + PS - 1) // PS
    num_pages = int(pages.sum())
    perm = rng.permutation(num_pages)
    pt = np.full((B, max_pages), -1, dtype=np.int32)
    o = 0
    for b in range(B):
        pt[b, :pages[b]] = perm[o:o + pages[b]]
        o += pages[b]
    ptd = torch.from_numpy(pt).to(dev)
    w_all = synth.make_attn_weights(shape, seed=3, device=dev)
    blk = A.AttnBlock(shape, synth.attn_rank_slice(w_all, shape, tp, rank), max_batch=B, max_pages_per_seq=max_pages,
                      max_context=max_pages * PS, tp_size=tp, tp_rank=rank)
    blk.use_peer_memory()
    kc, vc = rank_cache(rank, num_pages, nkv_l, dev)
    gx = torch.Generator(device=dev).manual_seed(11)
    xs = [torch.randn(B, shape.hidden, generator=gx, device=dev).to(torch.bfloat16) for _ in range(2)]
    status = torch.ones(1, device=dev)

    if a.time == 0:
        outs = []
        pos_buf = torch.from_numpy(ctx.astype(np.int32)).to(dev)
        xin = xs[0].clone()
        out_buf = torch.empty_like(xs[0])
        graph = None
        if a.graph:
            # one plain step first (kernel attributes are set outside the capture; it
            # writes the same K/V at the same positions as step 0), then capture one step
            blk.decode(xin, pos_buf, ptd, kc, vc, out=out_buf)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                blk.decode(xin, pos_buf, ptd, kc, vc, out=out_buf)
        for s in range(steps):
            pos_buf.copy_(torch.from_numpy((ctx + s).astype(np.int32)))
            xin.copy_(xs[s % 2])
            if graph is not None:
                graph.replay()
            else:
                blk.decode(xin, pos_buf, ptd, kc, vc, out=out_buf)
            outs.append(out_buf.clone())
        torch.cuda.synchronize()
        blk.check_error()
        got = [torch.empty_like(outs[0]) for _ in range(world)] if rank == 0 else None
        for s in range(steps):
            dist.gather(outs[s], got, dst=0)
            if rank == 0:
                same = all(torch.equal(g.view(torch.int16), outs[s].view(torch.int16)) for g in got)
                if not same:
                    print(f"step {s}: ranks disagree", flush=True)
                    status[0] = 0
        if rank == 0:
            # every rank recomputed here: its partial, then the rank-ordered sum
            blocks = [A.AttnBlock(shape, synth.attn_rank_slice(w_all, shape, tp, r), max_batch=B,
                                  max_pages_per_seq=max_pages, max_context=max_pages * PS, tp_size=tp, tp_rank=r)
                      for r in range(tp)]
            caches = [rank_cache(r, num_pages, nkv_l, dev) for r in range(tp)]
            for s in range(steps):
                pos = torch.from_numpy((ctx + s).astype(np.int32)).to(dev)
                parts = [blocks[r].decode_partial(xs[s % 2], pos, ptd, *caches[r]) for r in range(tp)]
                ref = A.tp_reduce_residual(parts, xs[s % 2])
                if not torch.equal(ref.view(torch.int16), outs[s].view(torch.int16)):
                    d = (ref.float() - outs[s].float()).abs().max().item()
                    print(f"step {s}: differs from the emulated ranks (max {d})", flush=True)
                    status[0] = 0
            for bk in blocks:
                bk.close()
        dist.broadcast(status, src=0)
    else:
        for s in range(3):
            pos = torch.from_numpy((ctx + s).astype(np.int32)).to(dev)
            blk.decode(xs[s % 2], pos, ptd, kc, vc)
        poss = [torch.from_numpy((ctx + 3 + s).astype(np.int32)).to(dev) for s in range(a.time)]
        out = torch.empty_like(xs[0])
        pos_buf = poss[0].clone()
        graph = None
        if a.graph:
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                blk.decode(xs[0], pos_buf, ptd, kc, vc, out=out)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for s in range(a.time):
            if graph is not None:
                pos_buf.copy_(poss[s], non_blocking=True)
                graph.replay()
            else:
                blk.decode(xs[s % 2], poss[s], ptd, kc, vc, out=out)
        e1.record()
        torch.cuda.synchronize()
        dist.barrier()
        blk.check_error()
        t = torch.tensor([e0.elapsed_time(e1) / a.time], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        kv = int(ctx.sum()) * 2 * nkv_l * D * 2
        if rank == 0:
            print(json.dumps({"block": "attention_decode_tp", "tp": tp, "graph": a.graph, "batch": B,
                              "context_tokens": int(ctx.sum()),
                              "ms_per_step": t.item(), "kv_bytes_per_rank": kv,
                              "kv_gbs_per_rank": kv / (t.item() * 1e-3) / 1e9, "split_tokens": blk.split_tokens}),
                  flush=True)
    blk.close()
    dist.barrier()
    dist.destroy_process_group()
    ok = int(status.item()) == 1
    if rank == 0 and ok and a.time == 0:
        print("ATTN_TP_OK", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
