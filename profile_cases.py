"""Profiling driver (a tool beside bench.py, not part of the package): small,
self-contained launches of single stages of the MoE FFN block, for
timing with CUDA events and for ncu captures that must stay small (a few
hundred MB on the device, a handful of launches):

    python profile_cases.py router [--tokens 4096] [--iters 3] [--plain]
    python profile_cases.py gemm   [--tokens 4096] [--experts 32] [--iters 3] [--act-planes 1|2]
    python profile_cases.py attention [--batch 64] [--ctx-min 1024] [--ctx-max 32768] [--iters 3]
    python profile_cases.py attn_block [--batch 64] [--ctx-min 1024] [--ctx-max 32768] [--iters 3]
    python profile_cases.py serving [--batch 64] [--prompt 512] [--steps 10] [--layers 92] [--gpus 1]
    python profile_cases.py prefill [--prompts 1] [--prompt 2048] [--iters 3]

`router`: RMSNorm+quant (with the fp32 n rows), the router logits, top-k
over T tokens of the GLM shape (hidden 5120, 160 experts; n is 84 MB at 4096
tokens, larger than L2) -- the layer's column-ordered path (n written in the
router column order, W reordered, `router_logits_rc_kernel`), or with
`--plain` the plain-layout `moe_router_logits`.  `gemm`: the layer forward on
a reduced expert count (weights 23.6 MB per expert) with one or two
activation planes -- the grouped GEMMs are its top kernels.
`attention`: paged decode attention at the per-rank shape of the TP=8
attention block (12 query heads over 1 KV head, head_dim 128, bf16 pages of
16 tokens), one new token per sequence with contexts drawn uniformly from
[ctx-min, ctx-max] (seed 0); its bytes are the K and V pages it must read.
`attn_block`: one TP rank's whole decode step of that block (rmsnorm, FP8
QKV, RoPE + page write, decode, FP8 o_proj, residual) on this GPU.
`serving`: the serving engine (engine.so) on the GLM-4.x shape of config 5
(92 layers, the first 3 dense), one GPU: `batch` requests prefilled with
`prompt` random tokens each, then batched greedy decode steps.  One weight set
per layer kind is shared by all layers of that kind (the whole depth fits one
GPU; each layer still streams its full weights from HBM, far more than L2);
every layer has its own KV pages.  Reports prefill tokens/s (the first step,
which runs every admitted prompt in forwards of up to 2048 rows), decode
tokens/s (wall time of the synchronous engine calls) and the engine's
per-stage device times of one decode step.
`prefill`: attention of prompt rows at that rank shape -- `prompts` prompts
of `prompt` positions in one call -- through the prefill kernel of
attn_paged_rows and, for comparison, through split decode.
Prints one line per stage with the mean CUDA-event time per launch.
"""
from __future__ import annotations

import argparse
import dataclasses
import json

import torch

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

from time_b200 import synth          # noqa: E402
from time_b200 import moe as M       # noqa: E402


def _time(fn, iters: int) -> float:
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def router(tokens: int, iters: int, plain: bool = False) -> dict:
    k = M.libs()["libkernels.so"]
    shape = synth.GLM
    dev = torch.device("cuda", 0)
    T, H, E, K = tokens, shape.hidden, shape.num_experts, shape.top_k
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    gamma = torch.ones(H, device=dev)
    W = torch.randn(E, H, generator=g, device=dev) * 0.02
    bias = synth.zipf_bias(E, seed=0).to(dev)
    rms = torch.empty(T, device=dev)
    n = torch.empty(T, H, device=dev)
    xq = torch.empty(T, H, dtype=torch.uint8, device=dev)
    ld = (T + 3) // 4 * 4
    xs = torch.empty(H // 128, ld, device=dev)
    logits = torch.empty(T, E, device=dev)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, device=dev)
    s = torch.cuda.current_stream().cuda_stream

    wrc = torch.empty_like(W)
    norm_fn = k.moe_rmsnorm_quant_n if plain else k.moe_rmsnorm_quant_rc

    def norm():
        M.check("rmsnorm", norm_fn(M.ptr(x), M.ptr(gamma), T, H, shape.eps, M.ptr(rms), M.ptr(n),
                                   M.ptr(xq), M.ptr(xs), ld, s))

    def logit():
        if plain:
            M.check("router_logits", k.moe_router_logits(M.ptr(n), M.ptr(W), M.ptr(bias), T, H, E, M.ptr(logits), s))
        else:
            M.check("router_columns", k.moe_router_columns(M.ptr(W), M.ptr(wrc), E, H, s))
            M.check("router_logits_rc", k.moe_router_logits_rc(M.ptr(n), M.ptr(wrc), M.ptr(bias), T, H, E,
                                                                 M.ptr(logits), s))

    def topk():
        M.check("topk", k.moe_topk_softmax(M.ptr(logits), T, E, K, M.ptr(idx), M.ptr(w), s))

    out = {"rmsnorm_quant_n_ms": _time(norm, iters), "router_logits_ms": _time(logit, iters),
           "topk_softmax_ms": _time(topk, iters)}
    fl = 2.0 * T * H * E
    out["router_logits_tflops"] = fl / (out["router_logits_ms"] * 1e-3) / 1e12
    out["router_logits_bytes"] = T * H * 4 + E * H * 4 + T * E * 4
    return out


def gemm(tokens: int, experts: int, iters: int, zipf: bool = True, planes: int = 1, form: int = 0) -> dict:
    shape = dataclasses.replace(synth.GLM, num_experts=experts)
    dev = torch.device("cuda", 0)
    w = synth.make_moe_weights(shape, seed=0, device=dev, zipf_bias=zipf)
    x = synth.make_x(shape, tokens, seed=1, device=dev)
    layer = M.MoELayer(shape, w, max_tokens=tokens)
    if planes == 2:
        layer.set_act_planes(2)
    if form:
        layer.set_gemm_form(form)
    out = torch.empty_like(x)
    ms = _time(lambda: layer.forward(x, out), iters)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(M.NUM_STAGES + 1)]
    layer.set_stage_events(ev)
    layer.forward(x, out)
    torch.cuda.synchronize()
    layer.set_stage_events(None)
    names = ["rmsnorm_quant", "router_topk", "permute", "gather", "gemm_gate_up", "gemm_down", "combine"]
    stages = {n: ev[i].elapsed_time(ev[i + 1]) for i, n in enumerate(names)}
    layer.check_error()
    _, _, counts = layer.last_routing(tokens)
    layer.close()
    # algorithmic bytes per launch of each grouped GEMM (the bench's definition)
    H, I = shape.hidden, shape.intermediate
    rows = int(counts.sum())
    touched = int((counts > 0).sum())
    w13 = 2 * I * H + (2 * I // 128) * (H // 128) * 4
    w2 = H * I + (H // 128) * (I // 128) * 4
    gu = touched * w13 + rows * (planes * H + H // 128 * 4) + rows * (planes * I + I // 128 * 4)
    dn = touched * w2 + rows * (planes * I + I // 128 * 4) + rows * H * 2
    return {"layer_forward_ms": ms, "stage_ms": stages, "rows": rows, "touched_groups": touched, "act_planes": planes,
            "gemm_gate_up_bytes": gu, "gemm_down_bytes": dn,
            "gate_up_gbs": gu / (stages["gemm_gate_up"] * 1e-3) / 1e9,
            "down_gbs": dn / (stages["gemm_down"] * 1e-3) / 1e9}


def proj(iters: int) -> dict:
    """The attention block's projections at one GPU's GLM shapes (QKV: N =
    (96 + 16) x 128, K = 5120; o_proj: N = 5120, K = 12288) for a few batch
    sizes, on the split-K mma.sync kernel (fp8_gemm_small) and on the tcgen05
    grouped GEMM with one group."""
    from time_b200 import attn as A
    dev = torch.device("cuda", 0)
    k = A.lib()
    out = {}
    for name, N, K in (("qkv", 112 * 128, 5120), ("o_proj", 5120, 12288)):
        wq = torch.randint(0, 120, (N, K), dtype=torch.uint8, device=dev)
        ws = torch.rand(N // 128, K // 128, device=dev) * 1e-3
        for T in (16, 64, 128, 256, 512):
            ld = (T + 15) // 16 * 16
            a = torch.randint(0, 120, (T, K), dtype=torch.uint8, device=dev)
            asc = torch.rand(K // 128, ld, device=dev)
            o = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
            wsb = int(k.fp8_gemm_small_workspace_bytes(T, N, K))
            wsp = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)

            def small():
                M.check("fp8_gemm_small", k.fp8_gemm_small(M.ptr(a), M.ptr(asc), ld, T, M.ptr(wq), M.ptr(ws), N, K,
                                                           M.ptr(o), M.ptr(wsp), wsb, M.stream_ptr()))
            cnt = torch.tensor([T], dtype=torch.int32, device=dev)
            start = torch.tensor([0], dtype=torch.int32, device=dev)

            def grouped():
                M.grouped_gemm(M.GEMM_DOWN_BF16, a, asc, ld, wq, ws, cnt, start, o, None, 0, K, N, ld)
            out[f"{name}_T{T}"] = {"small_us": _time(small, iters) * 1e3, "grouped_us": _time(grouped, iters) * 1e3,
                                   "weight_mb": N * K / 1e6}
    return out


def attention(batch: int, ctx_min: int, ctx_max: int, split: int, iters: int, nq: int = 12, nkv: int = 1) -> dict:
    import numpy as np
    from time_b200 import attn as A
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    lens = rng.integers(ctx_min, ctx_max + 1, size=batch)
    pages = (lens + A.PAGE - 1) // A.PAGE
    num_pages = int(pages.sum())
    max_pages = int(pages.max())
    perm = rng.permutation(num_pages).astype(np.int32)
    pt = np.full((batch, max_pages), -1, dtype=np.int32)
    o = 0
    for b in range(batch):
        pt[b, :pages[b]] = perm[o:o + pages[b]]
        o += pages[b]
    g = torch.Generator(device=dev).manual_seed(1)
    kc = torch.randn(num_pages, A.PAGE, nkv, A.HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(num_pages, A.PAGE, nkv, A.HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(batch, nq, A.HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    pt_d = torch.from_numpy(pt).to(dev)
    lens_d = torch.from_numpy(lens.astype(np.int32)).to(dev)
    max_splits = -(-max_pages * A.PAGE // split)
    k = A.lib()
    ws = torch.empty(k.attn_decode_workspace_bytes(batch, nq, max_splits), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ms = _time(lambda: A.decode_paged(q, kc, vc, pt_d, lens_d, nq, nkv, 1.0 / 128 ** 0.5, split_tokens=split,
                                      max_splits=max_splits, quant=True, workspace=ws, error_word=err), iters)
    assert int(err.item()) == 0
    kv_bytes = int(lens.sum()) * nkv * A.HEAD_DIM * 2 * 2
    io_bytes = batch * nq * A.HEAD_DIM * (2 + 2 + 1) + nq * batch * 4
    out = {"decode_ms": ms, "kv_bytes": kv_bytes, "algorithmic_bytes": kv_bytes + io_bytes,
           "achieved_gbs": (kv_bytes + io_bytes) / (ms * 1e-3) / 1e9, "context_tokens": int(lens.sum()),
           "split_tokens": split, "max_splits": max_splits}
    return out


def prefill(prompts: int, prompt_len: int, iters: int, nq: int = 12, nkv: int = 1) -> dict:
    """Attention of prefill rows (config-5 rank shape: 12 query heads, 1 KV
    head): `prompts` prompts of `prompt_len` positions, all rows in one call,
    through attn_paged_rows's prefill kernel and, for comparison, through the
    split decode kernel (every row streams its own prefix)."""
    import numpy as np
    from time_b200 import attn as A
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(0)
    pages = (prompt_len + A.PAGE - 1) // A.PAGE
    num_pages = prompts * pages
    pt = rng.permutation(num_pages).astype(np.int32).reshape(prompts, pages)
    g = torch.Generator(device=dev).manual_seed(1)
    kc = torch.randn(num_pages, A.PAGE, nkv, A.HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(num_pages, A.PAGE, nkv, A.HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    R = prompts * prompt_len
    q = torch.randn(R, nq, A.HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    row_seq = torch.arange(prompts, dtype=torch.int32, device=dev).repeat_interleave(prompt_len)
    lens = (torch.arange(prompt_len, dtype=torch.int32, device=dev) + 1).repeat(prompts)
    pt_d = torch.from_numpy(pt).to(dev)
    scale = 1.0 / 128 ** 0.5
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    args = (q, kc, vc, pt_d, row_seq, lens, nq, nkv, scale)
    t_pf = _time(lambda: A.paged_rows(*args, split_tokens=512, prefill_rows=R, quant=True, error_word=err), iters)
    t_dec = _time(lambda: A.paged_rows(*args, split_tokens=512, quant=True, error_word=err), iters)
    assert int(err.item()) == 0
    # causal work: sum over rows of (position + 1) keys, 2 matmuls of 128 x heads
    keys = prompts * prompt_len * (prompt_len + 1) // 2
    flops = 2.0 * 2.0 * keys * nq * A.HEAD_DIM
    kv_unique = num_pages * A.PAGE * nkv * A.HEAD_DIM * 2 * 2
    return {"rows": R, "prompts": prompts, "prompt_len": prompt_len, "prefill_kernel_ms": t_pf,
            "split_decode_ms": t_dec, "speedup": t_dec / t_pf, "attention_flop": flops,
            "prefill_tflops": flops / (t_pf * 1e-3) / 1e12, "kv_bytes_unique": kv_unique,
            "kv_bytes_decode_path": keys * nkv * A.HEAD_DIM * 2 * 2}


def attn_block(batch: int, ctx_min: int, ctx_max: int, iters: int, tp: int = 8, use_graph: bool = False) -> dict:
    """One TP rank's decode step of the config-4 attention block (rank 0's
    weight slice, its own cache) with the rank-local residual add in place of
    the TP sum (tp_size 1 on this GPU)."""
    import numpy as np
    from time_b200 import attn as A
    dev = torch.device("cuda", 0)
    shape = synth.GLM_ATTN
    rng = np.random.default_rng(0)
    ctx = rng.integers(ctx_min, ctx_max + 1, size=batch)
    steps = iters + 3
    pages = (ctx + steps + A.PAGE - 1) // A.PAGE
    num_pages, max_pages = int(pages.sum()), int(pages.max())
    perm = rng.permutation(num_pages).astype(np.int32)
    pt = np.full((batch, max_pages), -1, dtype=np.int32)
    o = 0
    for b in range(batch):
        pt[b, :pages[b]] = perm[o:o + pages[b]]
        o += pages[b]
    nkv = shape.num_kv_heads // tp
    g = torch.Generator(device=dev).manual_seed(1)
    kc = torch.randn(num_pages, A.PAGE, nkv, A.HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(num_pages, A.PAGE, nkv, A.HEAD_DIM, generator=g, device=dev).to(torch.bfloat16)
    x = torch.randn(batch, shape.hidden, generator=g, device=dev).to(torch.bfloat16)
    w_all = synth.make_attn_weights(shape, seed=3, device=dev)
    wr = synth.attn_rank_slice(w_all, shape, tp, 0)
    local = dataclasses.replace(shape, num_q_heads=shape.num_q_heads // tp, num_kv_heads=nkv)
    blk = A.AttnBlock(local, wr, max_batch=batch, max_pages_per_seq=max_pages, max_context=max_pages * A.PAGE)
    ptd = torch.from_numpy(pt).to(dev)
    out = torch.empty_like(x)
    poss = [torch.from_numpy((ctx + i).astype(np.int32)).to(dev) for i in range(steps)]
    pos_buf = poss[0].clone()
    step = [0]
    graph = None
    if use_graph:
        blk.decode(x, pos_buf, ptd, kc, vc, out=out)          # kernel attributes outside the capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            blk.decode(x, pos_buf, ptd, kc, vc, out=out)

    def run():
        pos_buf.copy_(poss[step[0] % steps], non_blocking=True)
        step[0] += 1
        if graph is not None:
            graph.replay()
        else:
            blk.decode(x, pos_buf, ptd, kc, vc, out=out)

    ms = _time(run, iters)
    blk.check_error()
    blk.close()
    kv = int(ctx.sum()) * 2 * nkv * A.HEAD_DIM * 2
    wbytes = sum(v.numel() * v.element_size() for k_, v in wr.items() if k_ != "gamma")
    return {"block_ms": ms, "graph": use_graph, "kv_bytes": kv, "weight_bytes": wbytes,
            "context_tokens": int(ctx.sum()),
            "achieved_gbs": (kv + wbytes) / (ms * 1e-3) / 1e9, "split_tokens": blk.split_tokens}


def serving(batch: int, prompt: int, steps: int, layers: int, max_seq: int, gpus: int = 1) -> dict:
    import time

    import numpy as np

    from time_b200 import engine as EN
    shape = dataclasses.replace(synth.GLM_MODEL, num_layers=layers)
    dev = torch.device("cuda:0")
    w = synth.make_model_weights(shape, seed=0, device=dev, share_layers=True)
    torch.cuda.synchronize()
    eng = EN.NativeEngine.from_weights(shape, w, max_batch=batch, max_seq=max_seq, num_gpus=gpus)
    rng = np.random.default_rng(0)
    prompts = [list(map(int, rng.integers(0, shape.vocab_size, prompt))) for _ in range(batch)]
    states = [eng.prefill(i, p, 0.0, 1.0, 1.0, 1 << 20) for i, p in enumerate(prompts)]
    assert all(s is not None for s in states)
    # the first step runs every admitted prompt (positions 0..prompt-2 of all
    # requests, in forwards of up to 2048 rows) and then one decode row each
    t0 = time.perf_counter()
    eng.batch_decode_raw(states)
    prefill_s = time.perf_counter() - t0
    for _ in range(3):
        eng.batch_decode_raw(states)
    t0 = time.perf_counter()
    for _ in range(steps):
        r = eng.batch_decode_raw(states)
    dt = (time.perf_counter() - t0) / steps
    assert r is not None and not any(d for _, d in r)
    eng.set_timing(True)
    eng.batch_decode_raw(states)
    st = eng.stage_ms()
    eng.check_error()
    weights_gb = (sum(t.numel() * t.element_size() for t in w["layers"][0]["ffn"].values() if t is not None)
                  + sum(t.numel() * t.element_size() for t in w["layers"][-1]["ffn"].values() if t is not None))
    eng.shutdown()
    return {"layers": layers, "gpus": gpus, "batch": batch, "prompt": prompt, "max_seq": max_seq,
            "prefill_tokens_per_s": batch * (prompt - 1) / prefill_s, "prefill_s": prefill_s,
            "decode_ms_per_step": dt * 1e3, "decode_tokens_per_s": batch / dt,
            "context_after": prompt + 4 + steps, "stage_ms_one_step": st,
            "ffn_weight_sets_gb": weights_gb / 1e9}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["router", "gemm", "attention", "attn_block", "serving", "proj", "prefill"])
    ap.add_argument("--prompts", type=int, default=1, help="prefill: prompts in the call")
    ap.add_argument("--gpus", type=int, default=1, help="serving: GPUs of the engine (one process)")
    ap.add_argument("--no-zipf", action="store_true", help="gemm: uniform routing (no router bias)")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--layers", type=int, default=92)
    ap.add_argument("--max-seq", type=int, default=1024)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx-min", type=int, default=1024)
    ap.add_argument("--ctx-max", type=int, default=32768)
    ap.add_argument("--split", type=int, default=512)
    ap.add_argument("--graph", action="store_true", help="attn_block: replay each step from a CUDA graph")
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--experts", type=int, default=32)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--plain", action="store_true", help="router: the plain-layout router")
    ap.add_argument("--act-planes", type=int, choices=[1, 2], default=1, help="gemm: activation planes")
    ap.add_argument("--gemm-form", choices=["rule", "one_sm", "pair", "small", "token"], default="rule",
                    help="gemm: force a grouped-GEMM form on both GEMMs")
    a = ap.parse_args()
    torch.cuda.set_device(0)
    if a.case == "attention":
        res = attention(a.batch, a.ctx_min, a.ctx_max, a.split, a.iters)
    elif a.case == "attn_block":
        res = attn_block(a.batch, a.ctx_min, a.ctx_max, a.iters, use_graph=a.graph)
    elif a.case == "serving":
        res = serving(a.batch, a.prompt, a.steps, a.layers, a.max_seq, a.gpus)
    elif a.case == "proj":
        res = proj(a.iters)
    elif a.case == "prefill":
        res = prefill(a.prompts, a.prompt, a.iters)
    else:
        res = (router(a.tokens, a.iters, a.plain) if a.case == "router"
               else gemm(a.tokens, a.experts, a.iters, not a.no_zipf, a.act_planes,
                         {"rule": 0, "one_sm": M.GEMM_ONE_SM_TILES, "pair": M.GEMM_PAIR_TILES,
                          "small": M.GEMM_SMALL_TILES, "token": M.GEMM_TOKEN_TILES}[a.gemm_form]))
    print(json.dumps({"case": a.case, "tokens": a.tokens, **res}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
