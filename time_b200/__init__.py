"""B200-native (sm_100a) MoE decoder-layer forward for the GLM-4.x-FP8 engine
of kollarsandor/time.

The product is the C-ABI shared libraries in ``time_b200/lib`` (built by
``python -m time_b200.build``), drop-in replacements for the reference's
libcudawrap / libncclwrap / libcublaswrap / libkernels / engine.so plus the
MoE, attention and loader entry points of ``include/``.  This Python package only loads them
(:func:`load`) and mirrors the reference's ctypes-driver style for tests and
benchmarks (:mod:`time_b200.moe`).  There is no CPU fallback: if the libraries
are missing, :func:`load` raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_DIR = Path(__file__).resolve().parent / "lib"
LIB_NAMES = ("libcudawrap.so", "libncclwrap.so", "libcublaswrap.so", "libkernels.so", "engine.so")

_loaded: dict[str, ctypes.CDLL] = {}


def lib_path(name: str) -> Path:
    return LIB_DIR / name


def load() -> dict[str, ctypes.CDLL]:
    """Load (once) and return the libraries keyed by file name.

    Raises RuntimeError if any is missing -- the CUDA path is the only path.
    """
    if _loaded:
        return _loaded
    missing = [n for n in LIB_NAMES if not lib_path(n).exists()]
    if missing:
        raise RuntimeError(
            f"time_b200 native libraries missing: {', '.join(missing)} in {LIB_DIR}; "
            "run `python -m time_b200.build` (needs nvcc)")
    try:
        # torch's CUDA library resolves its NCCL symbols at import; loading the
        # system NCCL globally (through libncclwrap) first would shadow them
        import torch  # noqa: F401
    except ImportError:
        pass
    for n in LIB_NAMES:
        _loaded[n] = ctypes.CDLL(str(lib_path(n)), mode=ctypes.RTLD_GLOBAL)
    return _loaded


__all__ = ["LIB_DIR", "LIB_NAMES", "load", "lib_path"]
