"""moe_router_topk_noalloc: the router for callers that cannot give this
library any device memory beyond their inputs and outputs (an engine that
plans all of its device memory up front, or a C / FFI host that must not call
cudaMalloc on its hot path).  Its [T][E] logits live in a fixed array inside
libkernels.so instead of a caller buffer.

Checked through the C-ABI against the two-call path (moe_router_logits into a
caller buffer, then moe_topk_softmax): identical indices and weights, on two
calls in a row with different sizes (the second call finds the first call's
logits still in the shared array), and a clear refusal above the array's
size.  This file is collected last on purpose; it also passes alone.
"""
import numpy as np
import pytest
import torch

from time_b200 import synth
from time_b200 import moe as M

pytestmark = pytest.mark.gpu

MAX_LOGITS = 1 << 20      # T * E limit of the fixed array


def _inputs(T, H, E, seed, dev):
    g = torch.Generator().manual_seed(seed)
    n = (torch.randn(T, H, generator=g) * torch.exp(0.3 * torch.randn(T, 1, generator=g))).float().to(dev)
    W = (torch.randn(E, H, generator=g) * 0.02).to(dev)
    b = synth.zipf_bias(E, seed=seed).to(dev)
    return n, W, b


def _two_call_path(k, n, W, b, T, H, E, K, dev):
    logits = torch.empty(T, E, device=dev)
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    M.check("moe_router_logits", k.moe_router_logits(M.ptr(n), M.ptr(W), M.ptr(b), T, H, E, M.ptr(logits), s))
    M.check("moe_topk_softmax", k.moe_topk_softmax(M.ptr(logits), T, E, K, M.ptr(idx), M.ptr(w), s))
    return idx, w


def _noalloc(k, n, W, b, T, H, E, K, dev):
    idx = torch.full((T, K), -7, dtype=torch.int32, device=dev)
    w = torch.full((T, K), -1.0, device=dev)
    s = torch.cuda.current_stream().cuda_stream
    M.check("moe_router_topk_noalloc",
            k.moe_router_topk_noalloc(M.ptr(n), M.ptr(W), M.ptr(b), T, H, E, K, M.ptr(idx), M.ptr(w), s))
    return idx, w


def test_noalloc_router_matches_two_call_path_twice(gpu):
    k = M.libs()["libkernels.so"]
    # first call: the GLM router shape at the array's full size (4096 x 256 would
    # be the limit; 4096 x 160 is the bench's shape); second call: a smaller,
    # different problem, so stale logits of the first call sit past its end
    for (T, H, E, K, seed) in [(4096, 5120, 160, 8, 1), (300, 1024, 64, 4, 2)]:
        n, W, b = _inputs(T, H, E, seed, gpu)
        ref_idx, ref_w = _two_call_path(k, n, W, b, T, H, E, K, gpu)
        idx, w = _noalloc(k, n, W, b, T, H, E, K, gpu)
        torch.cuda.synchronize()
        assert torch.equal(idx, ref_idx)
        # the same kernels run on the same logits: bit-identical weights
        assert np.array_equal(w.cpu().numpy().view(np.uint32), ref_w.cpu().numpy().view(np.uint32))


def test_noalloc_router_refuses_beyond_fixed_size(gpu):
    k = M.libs()["libkernels.so"]
    T, H, E, K = 8192, 256, 160, 8          # 8192 * 160 logits > 1,048,576
    assert T * E > MAX_LOGITS
    n, W, b = _inputs(16, H, E, 3, gpu)     # never read: the call must refuse before launching
    idx = torch.full((16, K), -7, dtype=torch.int32, device=gpu)
    w = torch.full((16, K), -1.0, device=gpu)
    s = torch.cuda.current_stream().cuda_stream
    rc = k.moe_router_topk_noalloc(M.ptr(n), M.ptr(W), M.ptr(b), T, H, E, K, M.ptr(idx), M.ptr(w), s)
    torch.cuda.synchronize()
    assert rc == 6                          # MOE_ERR_WORKSPACE
    assert k.moe_status_string(rc).decode().startswith("workspace too small")
    assert (idx == -7).all() and (w == -1.0).all()
