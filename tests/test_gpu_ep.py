"""Expert-parallel MoE FFN block on ONE GPU: the ranks of an EP group are
emulated in one process by calling the component entry points of
include/moe_layer.h rank by rank, with the two all-to-alls done as device
copies laid out by moe_ep_plan_host.  Everything the EP forward runs except
NCCL itself is exercised (dense expert-sorted send order, row packing, the
receive plan, the gather, both grouped GEMMs on the rank's expert slice, the
reverse packing and the split combine), and the concatenated output must be
BIT-IDENTICAL to the single-GPU layer: the dispatch carries the exact bytes
the single-GPU GEMM reads and the combine adds in the same order.

The real NCCL path (one process per GPU) is tested in test_gpu_ep_nccl.py.
"""
import numpy as np
import pytest
import torch

from time_b200 import synth
from time_b200 import moe as M

pytestmark = pytest.mark.gpu


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def st():
    return torch.cuda.current_stream().cuda_stream


def single_gpu(shape, w, x, planes=1):
    layer = M.MoELayer(shape, w, max_tokens=x.shape[0])
    if planes == 2:
        layer.set_act_planes(2)
    out = layer.forward(x)
    torch.cuda.synchronize()
    layer.check_error()
    idx, wts, _ = layer.last_routing(x.shape[0])
    layer.close()
    return out, idx


def ep_emulated(shape, w_all, x, ep, routing=None, placement=None, planes=1):
    """The EP forward of every rank, with host-planned device copies for the
    two exchanges.  `placement`: expert -> slot permutation (the send order
    then sorts by slot, as moe_layer_set_expert_placement makes the layer do).
    Returns the concatenated output and each rank's group counts."""
    k = M.libs()["libkernels.so"]
    dev = x.device
    T, H, I, E, K, S = x.shape[0], shape.hidden, shape.intermediate, shape.num_experts, shape.top_k, shape.num_shared
    epr = E // ep
    Tmax = -(-T // ep)
    rb = k.moe_ep_row_bytes(H) + (H if planes == 2 else 0)
    x2 = planes == 2
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    slot_of = None if placement is None else torch.tensor(placement, dtype=torch.int32, device=dev)
    ranks = []
    # ---- source side: norm, route, sort by expert, pack
    for r in range(ep):
        t0, t1 = synth.token_slice(T, ep, r)
        Tr = t1 - t0
        xr = x[t0:t1].contiguous()
        ld = (Tmax + 3) // 4 * 4
        rms = torch.empty(max(Tr, 1), device=dev)
        xq = torch.zeros(max(Tr, 1), H, dtype=torch.uint8, device=dev)
        xql = torch.zeros(max(Tr, 1), H, dtype=torch.uint8, device=dev) if x2 else None
        xs = torch.zeros(H // 128, ld, device=dev)
        if x2:
            M.check("rmsnorm_x2", k.moe_rmsnorm_quant_x2(M.ptr(xr), M.ptr(w_all["gamma"]), Tr, H, shape.eps,
                                                         M.ptr(rms), None, 0, M.ptr(xq), M.ptr(xql), M.ptr(xs), ld,
                                                         st()))
        else:
            M.check("rmsnorm", k.moe_rmsnorm_quant(M.ptr(xr), M.ptr(w_all["gamma"]), Tr, H, shape.eps, M.ptr(rms),
                                                   M.ptr(xq), M.ptr(xs), ld, st()))
        if routing is None:
            idx = torch.empty(max(Tr, 1), K, dtype=torch.int32, device=dev)
            wts = torch.empty(max(Tr, 1), K, device=dev)
            M.check("router", k.moe_router_topk(M.ptr(xr), M.ptr(rms), M.ptr(w_all["gamma"]), M.ptr(w_all["router_w"]),
                                                M.ptr(w_all.get("router_bias")), Tr, H, E, K, None, M.ptr(idx),
                                                M.ptr(wts), st()))
        else:
            idx = routing[0][t0:t1].contiguous()
            wts = routing[1][t0:t1].contiguous()
        P = Tr * K
        sort_ids = idx
        if slot_of is not None:
            sort_ids = torch.full((max(Tr, 1), K), -5, dtype=torch.int32, device=dev)
            M.check("remap", k.moe_ep_remap_experts(M.ptr(idx), P, E, M.ptr(slot_of), M.ptr(sort_ids), st()))
        ecounts = torch.zeros(E, dtype=torch.int32, device=dev)
        estart = torch.zeros(E, dtype=torch.int32, device=dev)
        spos = torch.full((max(P, 1),), -7, dtype=torch.int32, device=dev)
        stok = torch.full((max(P, 1),), -7, dtype=torch.int32, device=dev)
        stotal = torch.zeros(1, dtype=torch.int32, device=dev)
        M.check("permute_padded", k.moe_permute_padded(M.ptr(sort_ids), Tr, K, 0, E, 0, M.ptr(ecounts), M.ptr(estart),
                                                       M.ptr(spos), M.ptr(stok), M.ptr(stotal), P, M.ptr(err), 1,
                                                       st()))
        psend = torch.zeros(max(P, 1), rb, dtype=torch.uint8, device=dev)
        M.check("pack_rows", k.moe_ep_pack_rows_x2(M.ptr(xq), M.ptr(xql), M.ptr(xs), ld, M.ptr(stok),
                                                   M.ptr(stotal), P, H, M.ptr(psend), st()))
        ranks.append(dict(t0=t0, Tr=Tr, x=xr, xq=xq, xql=xql, xs=xs, ld=ld, idx=idx, wts=wts, ecounts=ecounts,
                          spos=spos, psend=psend))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # ---- counts exchange + host plan
    ec = [rk["ecounts"].cpu().numpy() for rk in ranks]
    for r, rk in enumerate(ranks):
        recv_counts = np.stack([ec[s][r * epr:(r + 1) * epr] for s in range(ep)])
        rk["recv_counts"] = torch.from_numpy(recv_counts.astype(np.int32)).to(dev)
        rk["plan"] = M.ep_plan_host(ep, epr, ec[r], recv_counts)
    # ---- dispatch: rank s's block for rank r lands at rank r's offset for s
    recv_cap = ep * Tmax * min(K, epr)
    for r, rk in enumerate(ranks):
        _, _, rrows, roff, _, rtot = rk["plan"]
        assert rtot <= recv_cap
        precv = torch.zeros(max(recv_cap, 1), rb, dtype=torch.uint8, device=dev)
        for s in range(ep):
            srows_s, soff_s = ranks[s]["plan"][0], ranks[s]["plan"][1]
            assert srows_s[r] == rrows[s]
            if rrows[s]:
                precv[roff[s]:roff[s] + rrows[s]].copy_(ranks[s]["psend"][soff_s[r]:soff_s[r] + srows_s[r]])
        rk["precv"] = precv
    # ---- receiving side: plan, gather, GEMMs, pack outputs
    for r, rk in enumerate(ranks):
        wr = synth.expert_slice(w_all, shape, ep, r, slot_of_expert=placement)
        G = epr + S
        R = ((recv_cap + S * Tmax + 16 * G) + 15) // 16 * 16
        counts = torch.zeros(G, dtype=torch.int32, device=dev)
        start = torch.zeros(G, dtype=torch.int32, device=dev)
        total = torch.zeros(1, dtype=torch.int32, device=dev)
        row_src = torch.full((R,), -9, dtype=torch.int32, device=dev)
        recv_dst = torch.full((max(recv_cap, 1),), -9, dtype=torch.int32, device=dev)
        M.check("recv_plan", k.moe_ep_recv_plan(M.ptr(rk["recv_counts"]), ep, epr, rk["Tr"], S, M.ptr(counts),
                                                M.ptr(start), M.ptr(total), M.ptr(row_src), M.ptr(recv_dst), R,
                                                recv_cap, M.ptr(err), st()))
        xp = torch.empty(planes, R, H, dtype=torch.uint8, device=dev)
        xps = torch.empty(H // 128, R, device=dev)
        M.check("ep_gather", k.moe_ep_gather_x2(M.ptr(rk["precv"]), M.ptr(rk["xq"]), M.ptr(rk["xql"]), M.ptr(rk["xs"]),
                                                rk["ld"], M.ptr(row_src), M.ptr(total), R, H, M.ptr(xp[0]),
                                                M.ptr(xp[1]) if x2 else None, M.ptr(xps), R, st()))
        hq = torch.empty(planes, R, I, dtype=torch.uint8, device=dev)
        hs = torch.empty(I // 128, R, device=dev)
        y = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
        # the GEMM form exactly as every rank's layer picks it: from max_tokens x ep_size (the
        # same on every rank), not from the rank's own token count
        # (the down projection takes token-major tiles at decode sizes when H % 256 == 0)
        small = E > 1 and Tmax * ep * K <= 16 * E
        form = M.GEMM_SMALL_TILES if small else M.GEMM_FULL_TILES
        dform = M.GEMM_TOKEN_TILES if small and H % 256 == 0 else form
        if x2:
            form |= M.GEMM_ACT_X2
            dform |= M.GEMM_ACT_X2
        M.grouped_gemm(M.GEMM_GATED_SWIGLU | form, xp, xps, R, wr["w13"], wr["s13"], counts, start, hq, hs, R, H, I,
                       R, error_word=err)
        M.grouped_gemm(M.GEMM_DOWN_BF16 | dform, hq, hs, R, wr["w2"], wr["s2"], counts, start, y, None, 0, I, H, R,
                       error_word=err)
        rtot = rk["plan"][5]
        ysend = torch.zeros(max(rtot, 1), H, dtype=torch.bfloat16, device=dev)
        M.check("pack_y", k.moe_ep_pack_y(M.ptr(y), M.ptr(recv_dst), rtot, H, M.ptr(ysend), st()))
        rk.update(counts=counts, start=start, y=y, ysend=ysend)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # ---- combine exchange + combine
    outs = []
    for s, rk in enumerate(ranks):
        srows, soff, _, _, stot, _ = rk["plan"]
        yrecv = torch.zeros(max(stot, 1), H, dtype=torch.bfloat16, device=dev)
        for r in range(ep):
            rrows_r, roff_r = ranks[r]["plan"][2], ranks[r]["plan"][3]
            if srows[r]:
                yrecv[soff[r]:soff[r] + srows[r]].copy_(ranks[r]["ysend"][roff_r[s]:roff_r[s] + rrows_r[s]])
        out = torch.empty(max(rk["Tr"], 1), H, dtype=torch.bfloat16, device=dev)
        M.check("combine_split", k.moe_combine_split(M.ptr(rk["x"]), M.ptr(yrecv), M.ptr(rk["spos"]), M.ptr(rk["wts"]),
                                                     M.ptr(rk["y"]), M.ptr(rk["start"][epr:]), S, rk["Tr"], K, H,
                                                     M.ptr(out), st()))
        outs.append(out[:rk["Tr"]])
    torch.cuda.synchronize()
    return torch.cat(outs), [rk["counts"].cpu() for rk in ranks]


@pytest.mark.parametrize("ep,T", [(2, 64), (4, 64), (2, 1), (4, 3), (8, 50)])
def test_ep_emulated_tiny_bit_identical(gpu, ep, T):
    shape = synth.TINY
    if shape.num_experts % ep:
        pytest.skip("experts do not split")
    case = synth.make_case(shape, T, seed=3)
    w = {k_: (v.to(gpu) if isinstance(v, torch.Tensor) else v) for k_, v in case.items()}
    x = w.pop("x")
    ref, _ = single_gpu(shape, w, x)
    out, _ = ep_emulated(shape, w, x, ep)
    assert np.array_equal(bits(out), bits(ref))


@pytest.mark.parametrize("ep,T", [(2, 64), (4, 37), (8, 50)])
def test_ep_emulated_two_planes_bit_identical(gpu, ep, T):
    """Two-term activations over expert parallelism: packed rows carry the hi
    and lo planes; the output is bit-identical to the one-GPU two-plane layer."""
    shape = synth.TINY
    case = synth.make_case(shape, T, seed=5)
    w = {k_: (v.to(gpu) if isinstance(v, torch.Tensor) else v) for k_, v in case.items()}
    x = w.pop("x")
    ref, _ = single_gpu(shape, w, x, planes=2)
    out, _ = ep_emulated(shape, w, x, ep, planes=2)
    assert np.array_equal(bits(out), bits(ref))


def test_ep_emulated_two_planes_glm_decode(gpu):
    """configs[2] decode shape (256 tokens, uniform routing) at EP 8 with
    two-term activations: bit-identical to one GPU."""
    shape = synth.GLM
    T = 256
    w = synth.make_moe_weights(shape, seed=0, device=gpu, zipf_bias=False)
    x = synth.make_x(shape, T, seed=1, device=gpu)
    logits = synth.uniform_routing(T, shape.num_experts, shape.top_k, seed=4, device=gpu)
    top = torch.topk(logits, shape.top_k, dim=1)
    routing = (top.indices.to(torch.int32).contiguous(), torch.softmax(top.values, dim=1).contiguous())
    layer = M.MoELayer(shape, w, max_tokens=T)
    layer.set_act_planes(2)
    ref = layer.forward(x, routing=routing).clone()
    torch.cuda.synchronize()
    layer.close()
    out, _ = ep_emulated(shape, w, x, 8, routing=routing, planes=2)
    assert np.array_equal(bits(out), bits(ref))


def test_ep_emulated_all_tokens_one_rank(gpu):
    """Every token routed to experts of rank 1 only: the other ranks receive
    nothing and still run their shared expert."""
    shape = synth.TINY
    T, ep = 40, 4
    case = synth.make_case(shape, T, seed=5)
    w = {k_: (v.to(gpu) if isinstance(v, torch.Tensor) else v) for k_, v in case.items()}
    x = w.pop("x")
    idx = torch.tensor([[2, 3]] * T, dtype=torch.int32, device=gpu)
    wts = torch.tensor([[0.75, 0.25]] * T, dtype=torch.float32, device=gpu)
    layer = M.MoELayer(shape, w, max_tokens=T)
    ref = layer.forward(x, routing=(idx, wts))
    torch.cuda.synchronize()
    layer.close()
    out, counts = ep_emulated(shape, w, x, ep, routing=(idx, wts))
    assert np.array_equal(bits(out), bits(ref))
    assert counts[1][:2].tolist() == [T, T] and int(counts[0][:2].sum()) == 0


@pytest.mark.parametrize("T", [256, 319, 321])
def test_ep_emulated_glm_decode_uniform_logits(gpu, T):
    """256 decode tokens, EP 8 over the GLM shape, routing
    from uniform random logits (top-8 softmax of U(0,1) logits).  319 and 321
    tokens split unevenly over the 8 ranks (40/39 and 41/40 tokens) right at
    the decode-form threshold (16 routed tokens per expert = 320 tokens): the
    ranks must all run the form the one-GPU layer runs."""
    shape = synth.GLM
    ep = 8
    w = synth.make_moe_weights(shape, seed=0, device=gpu)
    x = synth.make_x(shape, T, seed=2, device=gpu)
    logits = synth.uniform_routing(T, shape.num_experts, shape.top_k, seed=4, device=gpu)
    top = torch.topk(logits, shape.top_k, dim=1)
    idx = top.indices.to(torch.int32).contiguous()
    wts = torch.softmax(top.values, dim=1).contiguous()
    layer = M.MoELayer(shape, w, max_tokens=T)
    ref = layer.forward(x, routing=(idx, wts))
    torch.cuda.synchronize()
    layer.close()
    out, counts = ep_emulated(shape, w, x, ep, routing=(idx, wts))
    assert np.array_equal(bits(out), bits(ref))
    hist = torch.cat([c[:shape.num_experts // ep] for c in counts])
    assert int(hist.sum()) == T * shape.top_k


def test_remap_experts_matches_table(gpu):
    k = M.libs()["libkernels.so"]
    E, T, K = 160, 777, 8
    g = torch.Generator().manual_seed(11)
    slot = torch.randperm(E, generator=g).to(torch.int32)
    idx = torch.randint(0, E, (T, K), generator=g, dtype=torch.int32)
    idx[5, 3] = -1                                   # an empty slot of a routed token
    idx[9, 0] = E                                    # out of range: dropped, as the permutation drops it
    d_idx, d_slot = idx.to(gpu), slot.to(gpu)
    vidx = torch.full((T, K), -9, dtype=torch.int32, device=gpu)
    M.check("remap", k.moe_ep_remap_experts(M.ptr(d_idx), T * K, E, M.ptr(d_slot), M.ptr(vidx), st()))
    torch.cuda.synchronize()
    valid = (idx >= 0) & (idx < E)
    ref = torch.where(valid, slot[idx.clamp(0, E - 1).long()], torch.full_like(idx, -1))
    assert torch.equal(vidx.cpu(), ref)


@pytest.mark.parametrize("ep,E,T,K", [(2, 160, 2048, 8), (4, 160, 1024, 8), (8, 160, 512, 8), (8, 160, 2500, 8),
                                      (5, 20, 3000, 4), (6, 162, 777, 8), (64, 128, 100, 8), (3, 9, 0, 2)])
def test_ep_token_rows_numbering(gpu, ep, E, T, K):
    """moe_ep_token_rows (the peer dispatch's one row per token and
    destination rank): for every destination, the tokens with a pair there in
    token order, against a direct count; several 1024-token chunks and more
    than four destinations (several 64-bit scan groups) included."""
    k = M.libs()["libkernels.so"]
    epr = E // ep
    g = torch.Generator().manual_seed(ep * 1000 + T)
    vidx = torch.randint(-1, ep * epr, (T, K), generator=g, dtype=torch.int32)
    if T > 3:
        vidx[0] = 0                                   # every slot on rank 0
        vidx[1] = -1                                  # no valid slot
        vidx[2, :] = ep * epr - 1                     # the last rank only
    d_v = vidx.to(gpu)
    uidx = torch.full((ep, max(T, 1)), -9, dtype=torch.int32, device=gpu)
    utok = torch.full((ep, max(T, 1)), -9, dtype=torch.int32, device=gpu)
    ucnt = torch.full((ep,), -9, dtype=torch.int32, device=gpu)
    M.check("token_rows", k.moe_ep_token_rows(M.ptr(d_v) if T else None, T, K, ep, epr, M.ptr(uidx), M.ptr(utok),
                                              M.ptr(ucnt), st()))
    torch.cuda.synchronize()
    v = vidx.numpy()
    ui, ut, uc = uidx.cpu().numpy(), utok.cpu().numpy(), ucnt.cpu().numpy()
    for d in range(ep):
        has = ((v >= d * epr) & (v < (d + 1) * epr)).any(axis=1) if T else np.zeros(0, bool)
        toks = np.nonzero(has)[0]
        assert uc[d] == len(toks)
        assert np.array_equal(ut[d, :len(toks)], toks)
        ref = np.full(T, -1)
        ref[toks] = np.arange(len(toks))
        assert np.array_equal(ui[d, :T], ref)


@pytest.mark.parametrize("ep,T", [(2, 64), (4, 37)])
def test_ep_emulated_placement_tiny_bit_identical(gpu, ep, T):
    shape = synth.TINY
    case = synth.make_case(shape, T, seed=5)
    w = {kk: (v.to(gpu) if isinstance(v, torch.Tensor) else v) for kk, v in case.items()}
    x = w.pop("x")
    ref, _ = single_gpu(shape, w, x)
    g = torch.Generator().manual_seed(ep)
    placement = torch.randperm(shape.num_experts, generator=g).tolist()
    out, counts = ep_emulated(shape, w, x, ep, placement=placement)
    assert np.array_equal(bits(out), bits(ref))


def test_ep_emulated_placement_glm_balanced(gpu):
    """GLM shape, zipf router bias, 8 emulated ranks: the balanced placement
    computed from a calibration batch evens the ranks' routed rows and keeps
    the output bit-identical."""
    shape, ep, T = synth.GLM, 8, 512
    w = synth.make_moe_weights(shape, seed=0, device=gpu, zipf_bias=True)
    x = synth.make_x(shape, T, seed=1, device=gpu)
    ref, _ = single_gpu(shape, w, x)
    load = M.router_load(shape, w, synth.make_x(shape, 2048, seed=9, device=gpu))
    placement = synth.balanced_placement(load.tolist(), ep)
    out_c, counts_c = ep_emulated(shape, w, x, ep)
    out_b, counts_b = ep_emulated(shape, w, x, ep, placement=placement)
    assert np.array_equal(bits(out_b), bits(ref))
    assert np.array_equal(bits(out_c), bits(ref))
    routed = lambda cs: [int(c[:shape.num_experts // ep].sum()) for c in cs]
    rc, rb = routed(counts_c), routed(counts_b)
    assert sum(rc) == sum(rb) == T * shape.top_k
    assert max(rb) < max(rc)
