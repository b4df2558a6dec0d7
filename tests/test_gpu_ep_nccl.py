"""Expert-parallel MoE FFN block across real GPUs, one process per GPU
(tests/ep_worker.py under torch.distributed.run), with the exchange over NCCL
and over NVLink peer memory: the EP output must be bit-identical to the
single-GPU layer.  Needs at least 2 GPUs; skipped on a
1-GPU box (the single-GPU emulation in test_gpu_ep.py covers every EP kernel
there)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def n_gpus() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def launch(nproc: int, *args: str, extra_env=None) -> subprocess.CompletedProcess:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TIME_B200_EP_TIMEOUT_MS="60000", **(extra_env or {}))
    for _ in range(3):
        cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
               str(ROOT / "tests" / "ep_worker.py"), *args]
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=str(ROOT))
        # the rendezvous port can be taken between choosing it and binding it: choose again
        if r.returncode == 0 or "EADDRINUSE" not in r.stderr:
            return r
    return r


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("args", [("--shape", "tiny", "--tokens", "64", "--repeats", "3"),
                                  ("--shape", "tiny", "--tokens", "3"),
                                  ("--shape", "glm", "--tokens", "4096"),
                                  ("--shape", "glm", "--tokens", "256", "--uniform-logits")])
def test_ep_bit_identical(gpu, args, exchange):
    n = n_gpus()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    nproc = 8 if n >= 8 else (4 if n >= 4 else 2)
    r = launch(nproc, *args, "--exchange", exchange)
    assert r.returncode == 0 and "EP_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])


@pytest.mark.parametrize("fused", ["1", "0"])
@pytest.mark.parametrize("args", [("--shape", "glm", "--tokens", "4096", "--act-planes", "2"),
                                  ("--shape", "glm", "--tokens", "64", "--repeats", "3")])
def test_ep_peer_return_forms_bit_identical(gpu, args, fused):
    """The peer exchange's two return paths: the copy kernel after the GEMM
    (default) and the down GEMM storing each output row into its owner's
    buffer (TIME_B200_EP_FUSED_RETURN=1, token-major down form)."""
    n = n_gpus()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    nproc = 8 if n >= 8 else (4 if n >= 4 else 2)
    r = launch(nproc, *args, "--exchange", "peer", extra_env={"TIME_B200_EP_FUSED_RETURN": fused})
    assert r.returncode == 0 and "EP_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("args", [("--shape", "tiny", "--tokens", "64"), ("--shape", "glm", "--tokens", "4096")])
def test_ep_two_planes_bit_identical(gpu, args, exchange):
    """Two-term activations (moe_layer_set_act_planes(2)) over real ranks: the
    packed rows carry both planes; same output bits as the one-GPU layer."""
    n = n_gpus()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    nproc = 8 if n >= 8 else (4 if n >= 4 else 2)
    r = launch(nproc, *args, "--exchange", exchange, "--act-planes", "2")
    assert r.returncode == 0 and "EP_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_ep_balanced_placement_bit_identical(gpu, exchange):
    """Load-aware expert placement (moe_layer_set_expert_placement): same
    output bits as the single-GPU layer."""
    n = n_gpus()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    nproc = 8 if n >= 8 else (4 if n >= 4 else 2)
    r = launch(nproc, "--shape", "glm", "--tokens", "2048", "--placement", "balanced", "--exchange", exchange)
    assert r.returncode == 0 and "EP_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])
