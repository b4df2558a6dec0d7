#!/usr/bin/env python
"""MoE-layer tokens/s on B200 (BASELINE.json metric) for the GLM-4.x-shape MoE
FFN block: hidden 5120, 160 routed experts top-8 + 1 shared expert,
intermediate 1536, SwiGLU, FP8 e4m3 expert weights with 128x128 block scales.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|reference_gpu]
                    [--workload prefill|decode]

prefill (default): one step = one forward of the MoE
FFN block (RMSNorm -> router/top-k -> permute -> gate/up GEMM + SwiGLU ->
down GEMM -> combine + residual) over 4096 tokens with the zipf-skewed router
bias, inputs resident in HBM.
decode: one step = 256 tokens whose routing comes from
uniform random router logits (top-8 softmax of U(0,1) logits, supplied to
the layer's routed forward); the per-expert token histogram is printed.

Activations are two-term e4m3 by default (hi plane + e4m3 residual plane, one
1x128 scale: the format that keeps the layer within the north-star tolerance
of the fp32-activation result); `--act-planes 1` runs one e4m3 plane, and on
one GPU the line also reports the one-plane time of the same layer.

With N > 1 the tokens are split over N expert-parallel ranks (strong
scaling: rank r owns 160/N experts and T/N tokens).  The exchange is the
layer's NVLink peer-memory exchange by default (own kernels: P2P stores with
device-side flags, no host synchronisation), `--exchange nccl` for NCCL
send/recv; rows travel as e4m3 (both planes) + 1x128 scales, outputs return
as bf16.
Rank 0 prints one JSON line with the max-over-ranks time.

`e2e` is the same metric through the public layer call with host buffers:
pinned host x (and, for decode, the routing) -> device, forward, device ->
pinned host output, every step; the copies run on two copy streams so that
one step's input and output copies overlap the neighbouring steps' forwards
(double-buffered device x and out), as a serving loop would run them.  `cpu_baseline` / `--impl reference` time
the CPU restatement of the reference's path (the oracle, fp32 activations --
the reference has no CPU MoE path of its own that builds here) on the host
cores on a bounded sample; the same sample gives the `parity` key: the GPU
output of those tokens against the oracle's fp32-activation result.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/sec at 1/2/4/8 B200 (EP); % of FP8/HBM/NVLink roofline"
UNIT = "tokens/s"
TOKENS = {"prefill": 4096, "decode": 256}
WORKLOAD = {"prefill": "glm4x_moe_ffn_prefill (BASELINE configs[1])",
            "decode": "glm4x_moe_ffn_decode (BASELINE configs[2])"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "reference_gpu"], default="ours",
                    help="reference: the reference's CPU path (oracle port); reference_gpu: the reference's own "
                         "GPU kernels + cuBLAS SGEMM in its MoE call order (the GPU component baseline)")
    ap.add_argument("--workload", choices=["prefill", "decode"], default="prefill")
    ap.add_argument("--act-planes", type=int, choices=[1, 2], default=2,
                    help="expert-GEMM activations: 1 = e4m3, 2 = two-term e4m3 (hi + lo residual, the format "
                         "within the north-star tolerance of the fp32-activation result)")
    ap.add_argument("--tokens", type=int, default=None, help="global tokens per step (default 4096 prefill, 256 decode)")
    ap.add_argument("--experts", type=int, default=160,
                    help="routed experts (profiling captures of a smaller case only; the metric uses 160)")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="expert-parallel exchange for N > 1: NVLink peer memory (own kernels) or NCCL send/recv")
    ap.add_argument("--placement", choices=["balanced", "contiguous"], default=None,
                    help="expert placement for N > 1: load-balanced from a calibration batch (prefill default), "
                         "or contiguous slices (decode default: configs[2] names 160/EP experts per GPU)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="budget of the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    if a.tokens is None:
        a.tokens = TOKENS[a.workload]
    if a.placement is None:
        a.placement = "balanced" if a.workload == "prefill" else "contiguous"
    return a


def decode_routing(shape, T: int, device):
    """configs[2] routing: router logits drawn U(0,1) [T][E] (seeded), the
    top-k by value (equal values do not occur in practice among 160 uniform
    fp32 draws) and softmax weights over the selected logits."""
    import torch
    from time_b200 import synth
    logits = synth.uniform_routing(T, shape.num_experts, shape.top_k, seed=4, device=device)
    top = torch.topk(logits, shape.top_k, dim=1)
    return top.indices.to(torch.int32).contiguous(), torch.softmax(top.values, dim=1).contiguous()


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """SM clock, max clock, power and throttle reasons sampled DURING the timed
    region by an NVML thread every 5 ms (the timed region can be shorter than
    nvidia-smi's loop period); no samples (clocks: null) without NVML."""

    # NVML clocks-event reason bits (nvml.h nvmlClocksEventReason*)
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle", 0x2: "applications_clocks_setting"}

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self._max = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._thread = None
            return self
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    sm = pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM)
                    pw = pynvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                    self.rows.append((float(sm), float(self._max), pw, int(rs)))
                except Exception:
                    pass
                self._stop.wait(0.005)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.rows:
            return None
        reasons = sorted({name for r in self.rows for bit, name in self.REASONS.items()
                          if r[3] & bit and name not in ("gpu_idle", "applications_clocks_setting")})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": max(r[1] for r in self.rows),
                "power_w_max": max(r[2] for r in self.rows), "samples": len(self.rows), "reasons": reasons,
                "source": "nvml, 5 ms"}


# ---------------------------------------------------------------- CPU baseline

def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(shape, weights_cpu, x_cpu, budget_s: float, fixed_tokens: int | None = None, routing=None):
    """The oracle (fp32-activation "ref" mode, OpenMP over tokens, all host
    threads) on a bounded sample of the workload's tokens; tokens/s.  With
    `routing` ((idx, w) host tensors of every token) the experts run on that
    routing (the decode workload's supplied routing).  Also returns the
    sample's output (bf16 bits) for the parity check."""
    import numpy as np
    from oracle import oracle as orc   # CPU-baseline leg: the checker timed as the reference's CPU path
    ow = orc.OracleWeights(shape, weights_cpu)
    xb = x_cpu.contiguous().view(__import__("torch").int16).numpy().view(np.uint16)
    th = cpu_threads()

    def run(n):
        if routing is None:
            return orc.moe_ffn_forward(ow, xb[:n], mode=1, threads=th)[0]
        return orc.moe_ffn_experts(ow, xb[:n], routing[0][:n].numpy(), routing[1][:n].numpy(), mode=1, threads=th)

    if fixed_tokens is None:
        n = min(th, xb.shape[0])
        t0 = time.perf_counter()
        run(n)
        dt = time.perf_counter() - t0
        n = int(max(n, min(xb.shape[0], n * budget_s / max(dt, 1e-3))))
        n = max(th, (n // th) * th)
        n = min(n, xb.shape[0])
    else:
        n = fixed_tokens
    t0 = time.perf_counter()
    out = run(n)
    dt = time.perf_counter() - t0
    what = "full layer" if routing is None else "experts + combine on the supplied routing"
    return {"value": n / dt, "unit": UNIT, "cores": th, "kind": "port",
            "sample": f"{n} of {xb.shape[0]} tokens, {what} incl. all routed + shared experts, "
                      f"oracle ref mode (fp32 activations), {dt:.1f} s"}, n, dt, out


def parity_of(out_gpu, ref_bits, n: int, act_planes: int = 1):
    """The north-star tolerance metrics of the GPU output's first n tokens
    against the oracle's fp32-activation ("ref" mode) result."""
    import numpy as np
    from oracle import oracle as orc
    y = out_gpu[:n].float().cpu().numpy()
    mr, mae = orc.max_rel_and_mae(y, orc.bf16_bits_to_f32(ref_bits))
    return {"tokens": n, "against": "oracle ref mode: fp32 activations, dequantised e4m3 weights, fp32 router",
            "max_rel": mr, "mae": mae, "bar": {"max_rel": 1e-2, "mae": 2e-3},
            "within_bar": bool(mr <= 1e-2 and mae <= 2e-3),
            "note": ("two-term e4m3 activations (hi + lo residual, one 1x128 scale): about 7 significant bits "
                     "per activation" if act_planes == 2 else
                     "one e4m3 plane per activation (1x128 scales): 3 mantissa bits give ~3.6% RMS relative "
                     "rounding per activation, which this gap measures")}


# ---------------------------------------------------------------- algorithmic work

def algorithmic(shape, counts, T, planes: int = 1):
    """Bytes / FLOPs the layer must move or do, from the actual routing.  With
    two-term activations (planes = 2) each e4m3 activation row is read or
    written twice (hi and lo planes); the FLOPs are the layer's arithmetic
    (the tensor cores do `planes` times the MMA work of it)."""
    H, I, E, S, k = shape.hidden, shape.intermediate, shape.num_experts, shape.num_shared, shape.top_k
    counts = [int(c) for c in counts]
    touched = [c > 0 for c in counts]
    rows = sum(counts)
    w13 = 2 * I * H + (2 * I // 128) * (H // 128) * 4
    w2 = H * I + (H // 128) * (I // 128) * 4
    g1_bytes = sum(w13 for t in touched if t) + rows * (planes * H + H // 128 * 4) + rows * (planes * I + I // 128 * 4)
    g2_bytes = sum(w2 for t in touched if t) + rows * (planes * I + I // 128 * 4) + rows * H * 2
    g1_flops = 2.0 * rows * H * 2 * I
    g2_flops = 2.0 * rows * I * H
    layer_bytes = sum(w13 + w2 for t in touched if t) + T * H * 2 * 2 + E * H * 4
    layer_flops = g1_flops + g2_flops + 2.0 * T * H * E
    return {"gemm_gate_up": (g1_bytes, g1_flops), "gemm_down": (g2_bytes, g2_flops),
            "layer": (layer_bytes, layer_flops), "rows": rows}


def load_traffic(kernel: str, planes: int = 1):
    """ncu DRAM bytes per full launch of `kernel` (profiles/traffic.json; keys
    with a "_x2" suffix for two-term activations), or None."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(kernel + ("_x2" if planes == 2 else ""))
    except Exception:
        return None


# ---------------------------------------------------------------- arms

def run_reference(args):
    """--impl reference: the reference's CPU path (the oracle restatement; the
    reference's Futhark/Terra CPU builds are not available), bounded samples."""
    import torch
    from time_b200 import synth
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    shape = synth.GLM
    decode = args.workload == "decode"
    torch.manual_seed(0)
    w = synth.make_moe_weights(shape, seed=0, device="cpu", zipf_bias=not decode)
    x = synth.make_x(shape, args.tokens, seed=1, device="cpu")
    routing = decode_routing(shape, args.tokens, "cpu") if decode else None
    th = cpu_threads()
    # size one step to ~budget/steps seconds so the whole run stays within minutes
    per_step = max(2.0, min(20.0, 120.0 / max(1, args.steps + args.warmup)))
    _, n, _, _ = cpu_baseline(shape, w, x, per_step, routing=routing)
    from oracle import oracle as orc
    import numpy as np
    ow = orc.OracleWeights(shape, w)
    xb = x[:n].contiguous().view(torch.int16).numpy().view(np.uint16)
    times = []
    for i in range(args.warmup + args.steps):
        t1 = time.perf_counter()
        if decode:
            orc.moe_ffn_experts(ow, xb, routing[0][:n].numpy(), routing[1][:n].numpy(), mode=1, threads=th)
        else:
            orc.moe_ffn_forward(ow, xb, mode=1, threads=th)
        dt = time.perf_counter() - t1
        if i >= args.warmup:
            times.append(dt)
    ms = 1000.0 * sum(times) / len(times)
    value = n / (ms / 1000.0)
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD[args.workload], "tokens": args.tokens, "hidden": shape.hidden,
                       "experts": shape.num_experts, "top_k": shape.top_k, "intermediate": shape.intermediate,
                       "shared_experts": shape.num_shared,
                       "router": ("top-8 softmax of U(0,1) logits (supplied routing)" if decode
                                  else "softmax top-k, zipf(1.1) bias"),
                       "sample_tokens_per_step": n},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": th, "kind": "port",
                             "sample": f"{n} tokens per step of the {args.tokens}-token workload, oracle ref mode"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_reference_gpu(args):
    """--impl reference_gpu: the reference's own GPU components, the "beat this"
    number.  The reference's csrc/kernels.cu and csrc/cublas_wrappers.cu, built
    unmodified for sm_100 into oracle/_ref/, driven with ctypes in the call
    order of its MoE branch (src/terra/engine.t:1317-1347): launch_rms_norm ->
    launch_moe_gate (fp32 router) -> launch_moe_topk -> per expert:
    launch_fp8_dequantize + cbwSgemm (gate), the same for up, launch_swiglu,
    launch_fp8_dequantize + cbwSgemm (down) -> launch_moe_combine ->
    launch_add_residual (shared expert, residual).  The reference runs each of
    its top_k slots with the layer's single expert weight (its MoE path never
    indexes an expert); here each routed expert's own e4m3 weights are
    substituted and its rows gathered, so the FLOPs and weight bytes are the
    layer's.  Glue that the reference has no kernel for runs in torch inside
    the timed region: the zipf router bias add, the per-expert row order and
    counts (one host read per step, as a host loop over experts needs), the
    row gather and the scatter back to slot order.  The reference's dequantise
    has no block scales, so this arm is timed, not compared.  One GPU,
    rank 0 only; prefill only."""
    import ctypes
    import torch
    from time_b200 import synth
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    base = {"metric": METRIC, "impl": "reference_gpu"}
    libk = ROOT / "oracle" / "_ref" / "libref_kernels.so"
    libc = ROOT / "oracle" / "_ref" / "libref_cublas.so"
    if args.workload != "prefill" or not (libk.exists() and libc.exists()):
        why = ("prefill only" if args.workload != "prefill"
               else "oracle/_ref/ lacks the reference's kernels or cuBLAS wrapper (build() needs the reference sources)")
        print(json.dumps({**base, "unavailable": why}), flush=True)
        return 0
    K = ctypes.CDLL(str(libk))
    C = ctypes.CDLL(str(libc))
    vp, i32, sz, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float
    K.launch_rms_norm.argtypes = [vp, vp, vp, i32, i32, f32, vp]
    K.launch_moe_gate.argtypes = [vp, vp, vp, i32, i32, i32, i32, vp]
    K.launch_moe_topk.argtypes = [vp, vp, vp, i32, i32, i32, vp]
    K.launch_fp8_dequantize.argtypes = [vp, vp, sz, vp]
    K.launch_swiglu.argtypes = [vp, vp, vp, sz, vp]
    K.launch_moe_combine.argtypes = [vp, vp, vp, i32, i32, i32, vp]
    K.launch_add_residual.argtypes = [vp, vp, sz, vp]
    for f in (K.launch_rms_norm, K.launch_moe_gate, K.launch_moe_topk, K.launch_fp8_dequantize,
              K.launch_swiglu, K.launch_moe_combine, K.launch_add_residual):
        f.restype = None
    C.cbwCreate.argtypes = [ctypes.POINTER(vp)]
    C.cbwSetStream.argtypes = [vp, vp]
    C.cbwDestroy.argtypes = [vp]
    C.cbwSgemm.argtypes = [vp, i32, i32, i32, i32, i32, ctypes.POINTER(f32), vp, i32, vp, i32,
                           ctypes.POINTER(f32), vp, i32]
    for f in (C.cbwCreate, C.cbwSetStream, C.cbwDestroy, C.cbwSgemm):
        f.restype = i32

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = synth.GLM
    H, E, k, I, S, T = (shape.hidden, shape.num_experts, shape.top_k, shape.intermediate,
                        shape.num_shared, args.tokens)
    w = synth.make_moe_weights(shape, seed=0, device=dev, zipf_bias=True)
    x = synth.make_x(shape, T, seed=1, device=dev).float()        # the reference's hidden state is fp32
    gamma, router_w, bias = w["gamma"], w["router_w"].contiguous(), w["router_bias"]
    w13, w2 = w["w13"], w["w2"]                                    # [G][2I][H], [G][H][I] e4m3 bytes
    f = dict(dtype=torch.float32, device=dev)
    norm_out = torch.empty(T, H, **f)
    logits = torch.empty(T, E, **f)
    idx = torch.empty(T, k, dtype=torch.int32, device=dev)
    ew = torch.empty(T, k, **f)
    mlp = torch.empty(I * H, **f)                                   # handle.mlp_buffer: one dequantised matrix
    ein = torch.empty(T * k, H, **f)
    gate_o = torch.empty(T * k, I, **f)
    up_o = torch.empty(T * k, I, **f)
    eout = torch.empty(T * k, H, **f)
    slots = torch.empty(T * k, H, **f)                              # combine's [t][slot][H] layout
    sh_gate = torch.empty(T, I, **f)
    sh_up = torch.empty(T, I, **f)
    sh_out = torch.empty(T, H, **f)
    out = torch.empty(T, H, **f)
    stream = torch.cuda.current_stream(dev)
    st = vp(stream.cuda_stream)
    h = vp()
    if C.cbwCreate(ctypes.byref(h)) != 0 or C.cbwSetStream(h, st) != 0:
        raise RuntimeError("cbwCreate / cbwSetStream failed")
    one, zero = f32(1.0), f32(0.0)
    launches = [0]

    def P(t, off=0):
        return vp(t.data_ptr() + off)

    def sgemm(m, n, kk, A, lda, B, ldb, Cm, ldc):
        # engine.t:1328-1345: cbwSgemm(handle, N, N, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc)
        if C.cbwSgemm(h, 0, 0, m, n, kk, ctypes.byref(one), A, lda, B, ldb, ctypes.byref(zero), Cm, ldc) != 0:
            raise RuntimeError("cbwSgemm failed")
        launches[0] += 1

    def expert(g, rows, n, x_in, go, uo, yo):
        """One expert's MLP over n rows, engine.t:1326-1345 (gate, up, swiglu, down)."""
        K.launch_fp8_dequantize(P(w13[g]), P(mlp), I * H, st)
        sgemm(I, n, H, P(mlp), I, P(x_in, rows * H * 4), H, P(go, rows * I * 4), I)
        K.launch_fp8_dequantize(P(w13[g], I * H), P(mlp), I * H, st)
        sgemm(I, n, H, P(mlp), I, P(x_in, rows * H * 4), H, P(uo, rows * I * 4), I)
        K.launch_swiglu(P(go, rows * I * 4), P(uo, rows * I * 4), P(go, rows * I * 4), n * I, st)
        K.launch_fp8_dequantize(P(w2[g]), P(mlp), H * I, st)
        sgemm(H, n, I, P(mlp), H, P(go, rows * I * 4), I, P(yo, rows * H * 4), H)
        launches[0] += 4

    def step():
        K.launch_rms_norm(P(x), P(gamma), P(norm_out), H, T, shape.eps, st)
        K.launch_moe_gate(P(norm_out), P(router_w), P(logits), H, E, T, 0, st)
        logits.add_(bias)                                           # the benchmark's zipf skew (glue)
        K.launch_moe_topk(P(logits), P(idx), P(ew), E, k, T, st)
        flat = idx.view(-1).long()
        order = torch.argsort(flat, stable=True)                    # slot positions t*k+j, expert-major
        counts = torch.bincount(flat, minlength=E).tolist()         # host loop bounds
        torch.index_select(norm_out, 0, order // k, out=ein)
        row = 0
        for e in range(E):
            n = counts[e]
            if n:
                expert(e, row, n, ein, gate_o, up_o, eout)
            row += n
        slots.index_copy_(0, order, eout)
        K.launch_moe_combine(P(slots), P(ew), P(out), H, k, T, st)
        for s in range(S):
            expert(E + s, 0, T, norm_out, sh_gate, sh_up, sh_out)
            K.launch_add_residual(P(out), P(sh_out), T * H, st)
        K.launch_add_residual(P(out), P(x), T * H, st)
        launches[0] += 5 + S

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    launches[0] = 0
    times = []
    with ClockSampler(0) as clk:
        for _ in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            step()
            b.record(stream)
            b.synchronize()
            times.append(a.elapsed_time(b))
    C.cbwDestroy(h)
    ms = sum(times) / len(times)
    line = {**base, "value": T / (ms / 1000.0), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD["prefill"], "tokens": T, "hidden": H, "experts": E, "top_k": k,
                       "intermediate": I, "shared_experts": S, "router": "softmax top-k, zipf(1.1) bias",
                       "path": "reference csrc/kernels.cu + cuBLAS SGEMM (cbwSgemm), engine.t:1317-1347 order, "
                               "per-expert weights substituted", "l2": "weights (1.3 GB e4m3) exceed L2"},
            "reference_launches_per_step": launches[0] // max(1, args.steps),
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    return 0


NVLINK_GBS = 770.0   # measured peer copy per direction on this pool's B200s (no NVLink figure in MEASURED_PEAKS.json)


def run_ours(args):
    import torch
    import torch.distributed as dist
    from time_b200 import synth
    from time_b200 import moe as M

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        comm = M.nccl_comm(rank, world)

    decode = args.workload == "decode"
    shape = synth.GLM
    if args.experts != shape.num_experts:
        import dataclasses
        shape = dataclasses.replace(shape, num_experts=args.experts)
    if shape.num_experts % world:
        raise SystemExit(f"{shape.num_experts} experts do not split over {world} ranks")
    T = args.tokens
    w_all = synth.make_moe_weights(shape, seed=0, device=dev, zipf_bias=not decode)
    placement = None
    if world > 1 and args.placement == "balanced":
        # per-expert load measured on a calibration batch (not the timed tokens), the same table on every rank
        load = M.router_load(shape, w_all, synth.make_x(shape, 4096, seed=9, device=dev)).to(dev)
        dist.broadcast(load, src=0)
        placement = synth.balanced_placement(load.cpu().tolist(), world)
    w = synth.expert_slice(w_all, shape, world, rank, slot_of_expert=placement) if world > 1 else w_all
    del w_all
    x_all = synth.make_x(shape, T, seed=1, device=dev)
    t0, t1 = synth.token_slice(T, world, rank)
    x = x_all[t0:t1].contiguous()
    del x_all
    routing = None
    hist = None
    if decode:
        idx_all, w_all_r = decode_routing(shape, T, dev)         # the same draw on every rank
        hist = torch.bincount(idx_all.flatten().long(), minlength=shape.num_experts).tolist()
        routing = (idx_all[t0:t1].contiguous(), w_all_r[t0:t1].contiguous())
        del idx_all, w_all_r
    Tr = t1 - t0
    max_tokens = -(-T // world)
    out = torch.empty_like(x)
    layer = M.MoELayer(shape, w, max_tokens=max_tokens, ep_size=world, ep_rank=rank, comm=comm)
    act_planes = args.act_planes
    if act_planes == 2:
        layer.set_act_planes(2)
    if placement is not None:
        layer.set_expert_placement(placement)
    if world > 1 and args.exchange == "peer":
        layer.use_peer_memory()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(3, args.warmup)):
        layer.forward(x, out, routing=routing)
    torch.cuda.synchronize()
    layer.check_error()
    idx, _, counts = layer.last_routing(Tr)
    if decode:
        idx = routing[0].cpu()

    # ---- device-resident timed region with per-stage events
    K = args.steps
    stage_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(M.NUM_STAGES + 1)] for _ in range(K)]
    for evs in stage_ev:            # create the CUDA events outside the timed loop
        for e in evs:
            e.record(stream)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gate = torch.zeros(1, device=dev)

    def device_gate():
        # the timed region starts when every GPU has left one tiny all-reduce
        # queued on the stream, so a rank whose host starts late (NVML start-up
        # of the clock sampler, Python) does not charge its delay to the others
        if world > 1:
            dist.all_reduce(gate)

    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        device_gate()
        start.record(stream)
        for i in range(K):
            layer.set_stage_events(stage_ev[i])
            layer.forward(x, out, routing=routing)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    layer.set_stage_events(None)
    layer.check_error()
    ms_per_step = max_over_ranks(start.elapsed_time(end) / K)
    stages = {}
    for s_, name in enumerate(M.STAGE_NAMES):
        stages[name] = statistics.mean(stage_ev[i][s_].elapsed_time(stage_ev[i][s_ + 1]) for i in range(K))
    clocks = clk.summary()
    stages_max = stages
    if world > 1:
        t = torch.tensor([stages[n] for n in M.STAGE_NAMES], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        stages_max = dict(zip(M.STAGE_NAMES, t.tolist()))

    # ---- end to end through the public call with host buffers.  Every step
    # copies its input from pinned host memory and its output back to pinned
    # host memory, as a serving loop does: the copies of one step run on their
    # own streams (copy engines) while the forward of the previous step runs,
    # with two device buffers for x and out.  The timed region starts before
    # the first step's input copy and ends after the last step's output copy.
    x_host = x.cpu().pin_memory()
    out_host = [torch.empty(x_host.shape, dtype=x_host.dtype).pin_memory() for _ in range(2)]
    x_dev = [torch.empty_like(x) for _ in range(2)]
    out_dev = [torch.empty_like(out) for _ in range(2)]
    r_host = None
    r_dev = [None, None]
    if decode:
        r_host = tuple(t_.cpu().pin_memory() for t_ in routing)
        r_dev = [tuple(torch.empty_like(t_) for t_ in routing) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]     # input copy into buffer b done
    ev_fw = [torch.cuda.Event() for _ in range(2)]     # forward on buffer b done
    ev_out = [torch.cuda.Event() for _ in range(2)]    # output copy of buffer b done
    for b in range(2):
        ev_fw[b].record(stream)
        ev_out[b].record(stream)

    def e2e_step(i):
        b = i % 2
        s_in.wait_event(ev_fw[b])                  # the forward two steps back has read x_dev[b]
        with torch.cuda.stream(s_in):
            x_dev[b].copy_(x_host, non_blocking=True)
            if decode:
                for d_, h_ in zip(r_dev[b], r_host):
                    d_.copy_(h_, non_blocking=True)
        ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[b])               # out_dev[b] has been copied out
        layer.forward(x_dev[b], out_dev[b], routing=r_dev[b])
        ev_fw[b].record(stream)
        s_out.wait_event(ev_fw[b])
        with torch.cuda.stream(s_out):
            out_host[b].copy_(out_dev[b], non_blocking=True)
        ev_out[b].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    device_gate()
    e_start.record(stream)
    s_in.wait_event(e_start)
    for i in range(K):
        e2e_step(i)
    for b in range(2):
        stream.wait_event(ev_out[b])
    e_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end) / K)
    e2e_ok = bool(torch.equal(out_host[(K - 1) % 2], out.cpu()))   # same input, same output
    h2d = x.numel() * x.element_size() + (sum(t_.numel() * t_.element_size() for t_ in routing) if decode else 0)
    d2h = out.numel() * out.element_size()

    # ---- roofline of the dominant kernel (this rank) and of the layer
    peaks = load_peaks()
    G_local = shape.num_experts // world
    local_shape = shape
    if world > 1:
        import dataclasses
        local_shape = dataclasses.replace(shape, num_experts=G_local)
    work = algorithmic(local_shape, counts.tolist(), Tr, act_planes)
    dom = max(("gemm_gate_up", "gemm_down"), key=lambda n: stages[n])
    dom_bytes, dom_flops = work[dom]
    dom_s = stages[dom] / 1000.0
    achieved_gbs = dom_bytes / dom_s / 1e9
    roofline = {"kernel": dom, "bound": "hbm", "achieved": achieved_gbs, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": achieved_gbs / peaks["hbm_gbs"],
                "traffic": load_traffic(dom, act_planes) if not decode else None,
                "peak_source": peaks["source"], "algorithmic_bytes": dom_bytes,
                "tensor_tflops": dom_flops / dom_s / 1e12}
    lb, lf = work["layer"]
    if decode:
        lb -= shape.num_experts * shape.hidden * 4                  # the router does not run: routing is supplied
        lf -= 2.0 * Tr * shape.hidden * shape.num_experts
    elif world > 1:
        lb += (shape.num_experts - G_local) * shape.hidden * 4      # router weights are replicated
        lf += 2.0 * Tr * shape.hidden * (shape.num_experts - G_local)
    idx_h = idx.flatten().tolist()
    owner = [(placement[e] if placement else e) // G_local for e in range(shape.num_experts)]
    own_local = sum(1 for e in idx_h if e >= 0 and owner[e] == rank)
    sent_remote = sum(1 for e in idx_h if e >= 0) - own_local
    routed_rows = int(sum(counts[:G_local].tolist()))
    recv_remote = routed_rows - own_local
    rows_max = rows_mean = routed_rows
    if world > 1:
        t = torch.tensor([routed_rows, routed_rows], dtype=torch.float64, device=dev)
        tm = t.clone()
        dist.all_reduce(t[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(tm[1:], op=dist.ReduceOp.SUM)
        rows_max, rows_mean = int(t[0].item()), float(tm[1].item()) / world
    # the dispatch moves one packed row per (token, remote rank that owns at
    # least one of its experts) -- the peer exchange sends each token once per
    # destination; the return moves one bf16 row per remote pair
    rb = M.libs()["libkernels.so"].moe_ep_row_bytes(shape.hidden) + (shape.hidden if act_planes == 2 else 0)
    a2a_bytes = 0
    if world > 1:
        K_ = shape.top_k
        rows_to = [0] * world
        for t_ in range(len(idx_h) // K_):
            for d_ in {owner[e] for e in idx_h[t_ * K_:(t_ + 1) * K_] if e >= 0}:
                rows_to[d_] += 1
        got = torch.tensor(rows_to, dtype=torch.float64, device=dev)
        dist.all_reduce(got, op=dist.ReduceOp.SUM)
        uniq_sent = sum(rows_to) - rows_to[rank]
        uniq_recv = int(got[rank].item()) - rows_to[rank]
        a2a_bytes = max(uniq_sent * rb + recv_remote * shape.hidden * 2,
                        uniq_recv * rb + sent_remote * shape.hidden * 2)
    fp8_peak = 2 * peaks["bf16_tflops"]
    t_hbm = lb / (peaks["hbm_gbs"] * 1e9)
    t_fp8 = lf / (fp8_peak * 1e12)
    t_nvl = a2a_bytes / (NVLINK_GBS * 1e9)
    t_roof = max(t_hbm, t_fp8, t_nvl)
    t_roof = max_over_ranks(t_roof)
    layer_s = ms_per_step / 1000.0
    layer_roofline = {"bound": ("hbm", "tensor", "nvlink")[[t_hbm, t_fp8, t_nvl].index(max(t_hbm, t_fp8, t_nvl))],
                      "t_roof_us": t_roof * 1e6, "t_us": layer_s * 1e6, "frac": t_roof / layer_s,
                      "bytes_rank0": lb, "flops_rank0": lf, "a2a_bytes_per_direction_rank0": a2a_bytes,
                      "fp8_peak_tflops_assumed": fp8_peak, "nvlink_gbs_assumed": NVLINK_GBS,
                      "note": "per rank, max over ranks; fp8 peak = 2x measured bf16 (no fp8 measurement "
                              "in MEASURED_PEAKS.json); nvlink = measured peer copy per direction"}

    cpu = parity = None
    if not args.no_cpu_baseline and world == 1:
        wc = {k_: (v.cpu() if isinstance(v, torch.Tensor) else v) for k_, v in w.items()}
        rc_ = tuple(t_.cpu() for t_ in routing) if decode else None
        layer.forward(x, out, routing=routing)
        torch.cuda.synchronize()
        cpu, n_s, _, ref_bits = cpu_baseline(shape, wc, x.cpu(), args.cpu_seconds, routing=rc_)
        parity = parity_of(out, ref_bits, n_s, act_planes)

    # our kernels per forward: rmsnorm, router logits, top-k, 3 permutation kernels (count, scan,
    # scatter), gather, 2 GEMMs, combine = 10 (8 with supplied routing); EP replaces gather/combine
    # and adds (NCCL) row pack, receive plan, gather, output pack, split combine = 13 or (peer memory)
    # per-destination token numbering, counts, dispatch, 2 signal/waits, receive plan, gather, output
    # send, split combine = 17; the
    # expert placement adds its remap kernel.  NCCL's own kernels are not counted.
    # (The prefill router is three launches since the router reads column-ordered inputs: the
    # reorder of W, the logits, the top-k; the decode workload supplies its routing.)
    router_launches = 0 if decode else 3
    launches_per_step = (1 + router_launches + 3 + 1 + 2 + 1 if world == 1 else
                         1 + router_launches + (10 if args.exchange == "nccl" else 14) + (1 if placement else 0))

    # ---- the one-plane activation format on the same layer and inputs, for comparison
    one_plane = None
    if act_planes == 2 and world == 1:
        layer.set_act_planes(1)
        for _ in range(3):
            layer.forward(x, out, routing=routing)
        torch.cuda.synchronize()
        s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s1.record(stream)
        for _ in range(K):
            layer.forward(x, out, routing=routing)
        e1.record(stream)
        torch.cuda.synchronize()
        layer.check_error()
        ms1 = s1.elapsed_time(e1) / K
        one_plane = {"ms_per_step": ms1, "value": T * 1000.0 / ms1, "unit": UNIT,
                     "note": "moe_layer_set_act_planes(1): one e4m3 plane per activation (as FP8 serving stacks "
                             "run it) -- outside the north-star tolerance of the fp32-activation result at this "
                             "shape (max-rel ~3.3e-2, MAE ~4.0e-2 on the CPU oracle)"}
        layer.set_act_planes(2)
    if decode:
        launches_per_step -= 2
    dispatch = None
    if world > 1:
        dispatch = ("fp8 rows + 1x128 scales (5,280 B per row and plane at H = 5120; BASELINE configs[2] names "
                    "bf16 hidden states -- a deviation: the GEMM reads e4m3 rows, so sending them halves the bytes), "
                    "combine bf16, " + ("NVLink peer-memory stores from own kernels, no host sync, one row per "
                                        "(token, destination rank) however many of its experts live there"
                                        if args.exchange == "peer"
                                        else "NCCL send/recv, one host sync, one row per (token, expert) pair"))
    line = {"metric": METRIC, "value": T * 1000.0 / ms_per_step, "unit": UNIT, "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": ("e4m3 weights x two-term e4m3 activations (hi + lo, one 1x128 scale) -> f32, bf16 in/out"
                      if act_planes == 2 else "e4m3 x e4m3 -> f32 (bf16 in/out)"),
            "data": "synthetic",
            "config": {"workload": WORKLOAD[args.workload], "tokens": T,
                       "tokens_per_rank": max_tokens,
                       "hidden": shape.hidden, "experts": shape.num_experts, "top_k": shape.top_k,
                       "intermediate": shape.intermediate, "shared_experts": shape.num_shared,
                       "router": ("top-8 softmax of U(0,1) logits (supplied to the routed forward)" if decode
                                  else "fp32 softmax top-k in the reference's summation order, zipf(1.1) bias"),
                       "parallelism": f"ep{world}",
                       "expert_placement": ((args.placement + (" (greedy by routed pairs of a separate 4096-token "
                                                                "calibration batch)" if placement else ""))
                                            if world > 1 else None),
                       "dispatch": dispatch,
                       "l2": "inputs larger than L2: %.1f GB of expert weights streamed per step per rank"
                             % (sum(v.numel() for k_, v in w.items() if k_ in ("w13", "w2")) / 1e9)},
            "e2e": {"value": T * 1000.0 / e2e_ms, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "copies": "every step: pinned host -> device input, device -> pinned host output, on two copy "
                              "streams overlapping the neighbouring steps' forwards (double-buffered)",
                    "output_matches_device_run": e2e_ok},
            "roofline": roofline, "layer_roofline": layer_roofline,
            "stages_ms_rank0": stages, "rows_rank0": work["rows"],
            "stages_ms_max_over_ranks": stages_max,
            "routed_rows_per_rank": {"max": rows_max, "mean": rows_mean},
            "expert_tokens_rank0": {"max": int(counts[:G_local].max()), "min": int(counts[:G_local].min()),
                                    "mean": float(counts[:G_local].float().mean())},
            "gpu_launches": K * launches_per_step, "clocks": clocks, "cpu_baseline": cpu, "parity": parity,
            "act_planes": act_planes, "one_plane_activations": one_plane}
    if hist is not None:
        line["expert_histogram"] = hist
    if rank == 0:
        print(json.dumps(line), flush=True)
    layer.close()
    if world > 1:
        barrier()
        M.nccl_comm_destroy(comm)
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "reference_gpu":
        return run_reference_gpu(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
