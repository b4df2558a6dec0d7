"""The C-ABI boundary: the libraries load (no GPU needed to load) and export
every entry point include/*.h declares, including the full symbol sets of the
reference's headers (csrc/kernels.h:12-31, cublas_wrappers.h:51-67,
nccl_wrappers.h:47-61, cuda_wrappers.h:24-45) and the engine.so functions the
reference's server binds (src/server/engine_wrapper.py:64-98).  No compute
calls here."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
INCLUDE = ROOT / "include"

# which library implements each header
HEADER_LIB = {
    "cuda_wrappers.h": "libcudawrap.so",
    "nccl_wrappers.h": "libncclwrap.so",
    "cublas_wrappers.h": "libcublaswrap.so",
    "kernels.h": "libkernels.so",
    "moe_layer.h": "libkernels.so",
    "attn_block.h": "libkernels.so",
    "st_loader.h": "libkernels.so",
    "engine.h": "engine.so",
}

# the reference's exported symbol counts per header
REFERENCE_COUNTS = {"kernels.h": ("launch_", 20), "cublas_wrappers.h": ("cbw", 17),
                    "nccl_wrappers.h": ("ncw", 15), "cuda_wrappers.h": ("cw", 22)}
REFERENCE_NEW = {"cublas_wrappers.h": {"cbwFp8BlockScaledGroupedGemm", "cbwFp8BlockScaledGroupedGemmRowOut"},
                 "nccl_wrappers.h": {"ncwAllToAllv", "ncwCommInitRankTimeout", "ncwCommGetAsyncError",
                                     "ncwCommAbort", "ncwStreamSynchronizeTimeout"}}


def declared_functions(header: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", " ", header.read_text(), flags=re.S)
    text = "\n".join(l for l in text.splitlines() if not l.lstrip().startswith("#"))
    text = text.replace('extern "C" {', " ")
    text = re.sub(r"typedef[^;]*?\{.*?\}[^;]*;", " ", text, flags=re.S)   # struct/enum typedefs
    names = []
    for stmt in text.split(";"):
        s = " ".join(stmt.replace("}", " ").split())
        if not s or s.startswith("typedef"):
            continue
        m = re.match(r"^(?:const\s+)?[\w\s\*]+?\b(\w+)\s*\(", s)
        if m:
            names.append(m.group(1))
    return names


def exported(lib: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


@pytest.fixture(scope="module")
def libdir():
    import time_b200
    for n in time_b200.LIB_NAMES:
        assert time_b200.lib_path(n).exists(), f"{n} not built (python -m time_b200.build)"
    return time_b200.LIB_DIR


@pytest.mark.parametrize("header", sorted(HEADER_LIB))
def test_header_symbols_exported(libdir, header):
    names = declared_functions(INCLUDE / header)
    assert names, header
    syms = exported(libdir / HEADER_LIB[header])
    missing = [n for n in names if n not in syms]
    assert not missing, f"{HEADER_LIB[header]} lacks {missing}"


@pytest.mark.parametrize("header", sorted(REFERENCE_COUNTS))
def test_reference_symbol_sets_complete(header):
    prefix, count = REFERENCE_COUNTS[header]
    names = [n for n in declared_functions(INCLUDE / header) if n.startswith(prefix)]
    names = [n for n in names if n not in REFERENCE_NEW.get(header, set())]
    assert len(names) == count, (header, names)


def test_libraries_load_without_gpu(libdir):
    import time_b200
    libs = time_b200.load()
    assert set(libs) == set(time_b200.LIB_NAMES)
    k = libs["libkernels.so"]
    k.moe_status_string.restype = ctypes.c_char_p
    assert k.moe_status_string(4) == b"device-side wait timed out"
    c = libs["libcudawrap.so"]
    c.cwGetErrorString.restype = ctypes.c_char_p
    assert c.cwGetErrorString(2) == b"Out of memory"


# the engine.so functions src/server/engine_wrapper.py:64-98 binds
ENGINE_WRAPPER_SYMBOLS = ["init_engine", "prefill_opaque", "decode_step_opaque", "free_request_opaque", "free_engine",
                          "get_engine_info", "run_batch_decode_ext"]


def test_engine_wrapper_symbols(libdir):
    syms = exported(libdir / "engine.so")
    assert all(n in syms for n in ENGINE_WRAPPER_SYMBOLS), [n for n in ENGINE_WRAPPER_SYMBOLS if n not in syms]
    names = declared_functions(INCLUDE / "engine.h")
    assert names[:7] == ENGINE_WRAPPER_SYMBOLS, names[:7]
