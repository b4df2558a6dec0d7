"""Build the C-ABI libraries of this package in-tree for sm_100a.

    python -m time_b200.build            # incremental
    python -m time_b200.build --force

Outputs (time_b200/lib/):
    libcudawrap.so    csrc/cuda_wrappers.cu                       (reference libcudawrap)
    libncclwrap.so    csrc/nccl_wrappers.cu                       (reference libncclwrap)
    libcublaswrap.so  csrc/cublas_wrappers.cu + csrc/moe_gemm.cu  (reference libcublaswrap + grouped GEMM)
    libkernels.so     csrc/kernels.cu + csrc/moe_prep.cu + csrc/moe_ep.cu + csrc/moe_layer.cu
                      + csrc/attn.cu + csrc/attn_block.cu + csrc/gemm_small.cu + csrc/st_loader.cpp
                      (reference libkernels + the MoE layer, the attention block and the
                      checkpoint loader; links the two above)
    engine.so         csrc/engine.cpp + csrc/engine_kernels.cu
                      (reference engine.so: the serving engine; links libkernels)

Every library links the shared CUDA runtime so that device pointers and streams
handed over by a host framework are the same objects on both sides.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "lib"
OBJ = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-cudart", "shared",
              f"-I{INCLUDE}", f"-I{CSRC}"] + ARCH

LIBS = {
    "libcudawrap.so": (["cuda_wrappers.cu"], ["-lcudart"], []),
    "libncclwrap.so": (["nccl_wrappers.cu"], ["-lcudart", "-lnccl"], []),
    "libcublaswrap.so": (["cublas_wrappers.cu", "moe_gemm.cu"], ["-lcudart", "-lcublas", "-lcublasLt"], []),
    "libkernels.so": (["kernels.cu", "moe_prep.cu", "moe_ep.cu", "moe_layer.cu", "attn.cu", "attn_block.cu", "gemm_small.cu",
                       "st_loader.cpp"], ["-lcudart"], ["libcublaswrap.so", "libncclwrap.so"]),
    "engine.so": (["engine.cpp", "engine_kernels.cu"], ["-lcudart", "-lcublas"],
                  ["libkernels.so", "libcublaswrap.so", "libncclwrap.so"]),
}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def _newest_header() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, force: bool) -> str:
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _newest_header()):
        return f"up to date {obj.name}"
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return f"compiled {src.name}"


def build(force: bool = False, verbose: bool = False) -> None:
    LIB.mkdir(exist_ok=True)
    OBJ.mkdir(exist_ok=True)
    jobs = {}
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for srcs, _, _ in LIBS.values():
            for s in srcs:
                src = CSRC / s
                obj = OBJ / (src.stem + ".o")
                jobs[ex.submit(_compile, src, obj, force)] = s
        for fut in cf.as_completed(jobs):
            msg = fut.result()
            if verbose:
                print(msg)
    order = ["libcudawrap.so", "libncclwrap.so", "libcublaswrap.so", "libkernels.so", "engine.so"]
    for name in order:
        srcs, links, deps = LIBS[name]
        out = LIB / name
        objs = [OBJ / (Path(s).stem + ".o") for s in srcs]
        dep_paths = [LIB / d for d in deps]
        newest = max(o.stat().st_mtime for o in objs + dep_paths)
        if not force and out.exists() and out.stat().st_mtime >= newest:
            continue
        cmd = [nvcc(), "-shared", *ARCH, "-cudart", "shared", "-o", str(out), *map(str, objs),
               f"-L{LIB}", *[f"-l:{d}" for d in deps], *links, "-Xlinker", "-rpath=$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed for {name}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"linked {name}")


def reference_dir() -> Path | None:
    """The reference checkout whose own kernels oracle/_ref/ is built from: the
    REF_DIR environment variable, else a `reference` directory beside this
    repository's directory; None when neither exists (the GPU box has no
    reference sources and uses the prebuilt oracle/_ref/)."""
    env = os.environ.get("REF_DIR")
    if env:
        return Path(env)
    sibling = PKG.parent.parent / "reference"
    return sibling if sibling.is_dir() else None


def build_oracle(verbose: bool = False) -> None:
    """Build the CPU oracle (test infrastructure) and, when the reference
    sources are present, the reference's own kernels into oracle/_ref/."""
    odir = PKG.parent / "oracle"
    r = subprocess.run(["make", "-C", str(odir)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    ref = reference_dir()
    if ref is not None and (ref / "csrc" / "kernels.cu").exists():
        r = subprocess.run(["make", "-C", str(odir), "ref", f"REF_DIR={ref}"], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference kernel build failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print("oracle built")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    build(force=a.force, verbose=a.verbose)
    return 0


if __name__ == "__main__":
    sys.exit(main())
