"""Tensor-parallel decode attention block across real GPUs (tests/attn_tp_worker.py
under torch.distributed.run, one process per GPU, TP sum over NVLink peer
memory): every rank's output bit-identical to every other rank's and to all
ranks recomputed on one GPU, with plain calls and with each step replayed
from a CUDA graph.  Needs at least 2 GPUs; the one-GPU emulation is
tests/test_gpu_attn_block.py."""
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


@pytest.mark.parametrize("args", [("--shape", "small", "--batch", "3", "--ctx-min", "0", "--ctx-max", "300"),
                                  ("--shape", "glm", "--batch", "8"),
                                  ("--shape", "glm", "--batch", "8", "--graph")])
def test_attn_tp_bit_identical(gpu, args):
    n = n_gpus()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    nproc = 8 if n >= 8 else 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TIME_B200_EP_TIMEOUT_MS="20000")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           str(ROOT / "tests" / "attn_tp_worker.py"), *args]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=str(ROOT))
    assert r.returncode == 0 and "ATTN_TP_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])
