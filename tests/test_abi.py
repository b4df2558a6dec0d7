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


def test_row_entry_points_refuse_bad_arguments_without_launching(libdir):
    """moe_scatter_rows_x2 and moe_ep_token_rows check every argument before
    any CUDA call, so a refused call returns MOE_ERR_INVALID_ARGUMENT (1) on
    a machine without a GPU; none of these pointers is ever dereferenced."""
    import time_b200
    k = time_b200.load()["libkernels.so"]
    vp, ci = ctypes.c_void_p, ctypes.c_int
    k.moe_scatter_rows_x2.argtypes = [vp, vp, vp, ci, vp, ci, ci, vp, ci, vp, vp, ci, ci, vp, vp, vp, ci, vp]
    k.moe_ep_token_rows.argtypes = [vp, ci, ci, ci, ci, vp, vp, vp, vp]
    fake = 0x1000                                     # 16-byte aligned, never dereferenced

    def scatter(**over):
        a = dict(xq=fake, xq_lo=None, xs=fake, xs_ld=64, pos=fake, T=64, k=8, shared=fake, ns=1, rowtok=fake,
                 total=fake, cap=1024, H=512, xp=fake, xp_lo=None, xps=fake, xps_ld=1024)
        a.update(over)
        return k.moe_scatter_rows_x2(a["xq"], a["xq_lo"], a["xs"], a["xs_ld"], a["pos"], a["T"], a["k"], a["shared"],
                                     a["ns"], a["rowtok"], a["total"], a["cap"], a["H"], a["xp"], a["xp_lo"], a["xps"],
                                     a["xps_ld"], None)
    assert scatter(k=17) == 1                          # more slots than a token can have
    assert scatter(k=0) == 1
    assert scatter(ns=3) == 1                          # at most two shared experts
    assert scatter(H=500) == 1                         # H % 128
    assert scatter(xps_ld=1000) == 1                   # scale rows shorter than the layout
    assert scatter(xq=fake + 8) == 1                   # misaligned rows
    assert scatter(xq_lo=fake) == 1                    # one lo pointer without the other
    assert scatter(shared=None) == 1                   # shared rows without their starts
    assert scatter(cap=0) == 0                         # nothing to write: no launch

    def token_rows(ep, epr=20, T=64, K=8, ptrs=True):
        p = fake if ptrs else None
        return k.moe_ep_token_rows(p, T, K, ep, epr, p, p, fake, None)
    assert token_rows(65) == 1                         # more ranks than the numbering supports
    assert token_rows(0) == 1
    assert token_rows(8, epr=0) == 1
    assert token_rows(8, ptrs=False) == 1              # T > 0 needs vidx, uidx, utok
