"""Small, self-contained launches of single stages of the MoE FFN block, for
timing with CUDA events and for ncu captures that must stay small (a few
hundred MB on the device, a handful of launches):

    python -m time_b200.profile_cases router [--tokens 4096] [--iters 3]
    python -m time_b200.profile_cases gemm   [--tokens 4096] [--experts 32] [--iters 3]

`router`: RMSNorm+quant (with the fp32 n rows), tiled router logits, top-k
over T tokens of the GLM shape (hidden 5120, 160 experts; n is 84 MB at 4096
tokens, larger than L2).  `gemm`: the layer forward on a reduced expert count
(weights 23.6 MB per expert) -- the grouped GEMMs are its top kernels.
Prints one line per stage with the mean CUDA-event time per launch.
"""
from __future__ import annotations

import argparse
import dataclasses
import json

import torch

from . import synth
from . import moe as M


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


def router(tokens: int, iters: int) -> dict:
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

    def norm():
        M.check("rmsnorm_n", k.moe_rmsnorm_quant_n(M.ptr(x), M.ptr(gamma), T, H, shape.eps, M.ptr(rms), M.ptr(n),
                                                   M.ptr(xq), M.ptr(xs), ld, s))

    def logit():
        M.check("router_logits", k.moe_router_logits(M.ptr(n), M.ptr(W), M.ptr(bias), T, H, E, M.ptr(logits), s))

    def topk():
        M.check("topk", k.moe_topk_softmax(M.ptr(logits), T, E, K, M.ptr(idx), M.ptr(w), s))

    out = {"rmsnorm_quant_n_ms": _time(norm, iters), "router_logits_ms": _time(logit, iters),
           "topk_softmax_ms": _time(topk, iters)}
    fl = 2.0 * T * H * E
    out["router_logits_tflops"] = fl / (out["router_logits_ms"] * 1e-3) / 1e12
    out["router_logits_bytes"] = T * H * 4 + E * H * 4 + T * E * 4
    return out


def gemm(tokens: int, experts: int, iters: int) -> dict:
    shape = dataclasses.replace(synth.GLM, num_experts=experts)
    dev = torch.device("cuda", 0)
    w = synth.make_moe_weights(shape, seed=0, device=dev, zipf_bias=True)
    x = synth.make_x(shape, tokens, seed=1, device=dev)
    layer = M.MoELayer(shape, w, max_tokens=tokens)
    out = torch.empty_like(x)
    ms = _time(lambda: layer.forward(x, out), iters)
    layer.check_error()
    _, _, counts = layer.last_routing(tokens)
    layer.close()
    # algorithmic bytes per launch of each grouped GEMM (the bench's definition)
    H, I = shape.hidden, shape.intermediate
    rows = int(counts.sum())
    touched = int((counts > 0).sum())
    w13 = 2 * I * H + (2 * I // 128) * (H // 128) * 4
    w2 = H * I + (H // 128) * (I // 128) * 4
    return {"layer_forward_ms": ms, "rows": rows, "touched_groups": touched,
            "gemm_gate_up_bytes": touched * w13 + rows * (H + H // 128 * 4) + rows * (I + I // 128 * 4),
            "gemm_down_bytes": touched * w2 + rows * (I + I // 128 * 4) + rows * H * 2}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["router", "gemm"])
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--experts", type=int, default=32)
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()
    torch.cuda.set_device(0)
    res = router(a.tokens, a.iters) if a.case == "router" else gemm(a.tokens, a.experts, a.iters)
    print(json.dumps({"case": a.case, "tokens": a.tokens, **res}), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
