"""Build libmoe_b200.so (CUDA kernels + C ABI) and libmoe_layer.so (the C++
drop-in layer classes) in-tree for sm_100a.

    python accelerating-moe-inference_b200/build.py [-v]

nvcc cross-compiles without a GPU.  Objects go to ``_build/`` beside this
file; the shared libraries land next to this file, where the Python binding
and the C++ tests look for them.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = CSRC / "host"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libmoe_b200.so"
LAYER_LIB = PKG / "libmoe_layer.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("MOE_CXX", "/usr/bin/g++")
CUDA_HOME = Path(NVCC).resolve().parent.parent

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                     "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(str(c) for c in cmd[:3])} ...")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    sources = sorted(CSRC.glob("*.cu"))
    objs = []
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _newer(obj, [src] + headers) or ptxas_info:
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs.append([NVCC] + NVCC_FLAGS + extra + ["-c", src, "-o", obj])
    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for f in [ex.submit(_run, j, verbose or ptxas_info) for j in jobs]:
            f.result()
    if jobs or not LIB.exists():
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs, verbose)

    # C++ drop-in layer (Tensor / ModelLoader / Linear / PhiMLP / PhiMoE) over the C ABI.
    host_srcs = sorted(HOST.glob("*.cpp"))
    if host_srcs:
        host_hdrs = [INCLUDE / n for n in ("tensor.h", "model_loader.h", "layer.h", "moe_b200.h")
                     if (INCLUDE / n).exists()]
        if _newer(LAYER_LIB, host_srcs + host_hdrs + [LIB]):
            # No implicit contraction: the reference-order arithmetic (the
            # router's FMA chain, layer_norm's unfused variance) is spelled out.
            _run([CXX, "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-fopenmp",
                  "-Wall", "-I",
                  INCLUDE, *host_srcs, "-o", LAYER_LIB, f"-L{PKG}", "-lmoe_b200",
                  "-Wl,-rpath,$ORIGIN"], verbose)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="rebuild all with -Xptxas -v")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_info))
