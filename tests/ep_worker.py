"""One rank of the expert-parallel parity check (launched by
test_gpu_ep_nccl.py under torch.distributed.run, one process per GPU), with
the exchange over NCCL or over NVLink peer memory (--exchange).

Every rank builds the same seeded weights and tokens, keeps its expert slice
and token slice, and runs the EP layer over a real NCCL communicator
(ncwCommInitRank).  Rank 0 gathers the outputs and compares them with the
single-GPU layer on its own GPU: they must be bit-identical.  Prints EP_OK on
success; exits non-zero otherwise.
"""
import argparse
import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch
import torch.distributed as dist

from time_b200 import synth
from time_b200 import moe as M


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", choices=["tiny", "glm"], default="tiny")
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--uniform-logits", action="store_true")
    ap.add_argument("--repeats", type=int, default=2)
    ap.add_argument("--exchange", choices=["nccl", "peer"], default="nccl")
    ap.add_argument("--placement", choices=["contiguous", "balanced"], default="contiguous")
    ap.add_argument("--act-planes", type=int, choices=[1, 2], default=1)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    comm = M.nccl_comm(rank, world)
    shape = synth.TINY if a.shape == "tiny" else synth.GLM
    T = a.tokens
    w_all = synth.make_moe_weights(shape, seed=0, device=dev, zipf_bias=True)
    x_all = synth.make_x(shape, T, seed=1, device=dev)
    routing = None
    if a.uniform_logits:
        logits = synth.uniform_routing(T, shape.num_experts, shape.top_k, seed=4, device=dev)
        top = torch.topk(logits, shape.top_k, dim=1)
        routing = (top.indices.to(torch.int32).contiguous(), torch.softmax(top.values, dim=1).contiguous())
    t0, t1 = synth.token_slice(T, world, rank)
    placement = None
    if a.placement == "balanced":
        # load measured on a calibration batch on rank 0, the same table everywhere
        load = M.router_load(shape, w_all, synth.make_x(shape, 1024, seed=9, device=dev)).to(dev)
        dist.broadcast(load, src=0)
        placement = synth.balanced_placement(load.cpu().tolist(), world)
    w = synth.expert_slice(w_all, shape, world, rank, slot_of_expert=placement)
    layer = M.MoELayer(shape, w, max_tokens=-(-T // world), ep_size=world, ep_rank=rank, comm=comm)
    if a.act_planes == 2:
        layer.set_act_planes(2)      # before the peer buffers: packed rows carry both planes
    if placement is not None:
        layer.set_expert_placement(placement)
    if a.exchange == "peer":
        layer.use_peer_memory()
    x = x_all[t0:t1].contiguous()
    r_local = None if routing is None else (routing[0][t0:t1].contiguous(), routing[1][t0:t1].contiguous())
    outs = []
    for _ in range(a.repeats):
        outs.append(layer.forward(x, routing=r_local).clone())
    torch.cuda.synchronize()
    layer.check_error()
    ok = all(torch.equal(outs[0].view(torch.int16), o.view(torch.int16)) for o in outs[1:])
    # gather to rank 0 (pad to the longest slice)
    n_max = -(-T // world)
    pad = torch.zeros(n_max, shape.hidden, dtype=torch.bfloat16, device=dev)
    pad[: t1 - t0].copy_(outs[0])
    got = [torch.empty_like(pad) for _ in range(world)] if rank == 0 else None
    dist.gather(pad, got, dst=0)
    status = torch.tensor([1 if ok else 0], device=dev)
    if rank == 0:
        full = torch.cat([got[r][: synth.token_slice(T, world, r)[1] - synth.token_slice(T, world, r)[0]]
                          for r in range(world)])
        ref_layer = M.MoELayer(shape, w_all, max_tokens=T)
        if a.act_planes == 2:
            ref_layer.set_act_planes(2)
        ref = ref_layer.forward(x_all, routing=routing)
        torch.cuda.synchronize()
        ref_layer.close()
        same = torch.equal(full.view(torch.int16), ref.view(torch.int16))
        if not same:
            diff = (full.float() - ref.float()).abs()
            print(f"rank0: EP output differs from single GPU: max {diff.max().item()} "
                  f"count {(diff > 0).sum().item()}", flush=True)
        status[0] = status[0] * (1 if same else 0)
    dist.broadcast(status, src=0)
    layer.close()
    dist.barrier()
    M.nccl_comm_destroy(comm)
    dist.destroy_process_group()
    if rank == 0 and int(status.item()) == 1:
        print("EP_OK", flush=True)
    return 0 if int(status.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
