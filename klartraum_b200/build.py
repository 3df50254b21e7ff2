"""Build the renderer's shared library ``klartraum_b200/libkt_gs.so`` for sm_100a.

Every CUDA source is compiled by nvcc for ``sm_100a`` only. ``project.cu`` (projection and
bin counting) is compiled with ``-fmad=false`` so that its float results are the correctly
rounded values of the shader's operation sequence; the host code uses
``-ffp-contract=off`` for the camera matrix products for the same reason.

Usage: ``python -m klartraum_b200.build`` (or ``klartraum_b200.build.build()``).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libkt_gs.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
          "-I", INCLUDE, "-I", CSRC]

# source -> extra flags
SOURCES = {
    "project.cu": ["-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false"],
    "binning.cu": [],
    "place.cu": [],
    "keys.cu": [],
    "sort.cu": [],
    "raster.cu": [],
    "sort_static.cu": [],
    "api.cpp": [],
    "spz.cpp": [],
    "ply.cpp": [],
}


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _deps(src: str) -> list[str]:
    hdrs = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    return [os.path.join(CSRC, src), os.path.join(INCLUDE, "kt_gs.h"), __file__] + hdrs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _compile(src: str, extra: list[str], verbose: bool) -> str:
    obj = os.path.join(BUILD, src.rsplit(".", 1)[0] + ".o")
    if not _stale(obj, _deps(src)):
        return obj
    lang = ["-x", "cu"] if src.endswith(".cu") else []
    cmd = [nvcc(), *ARCH, *COMMON, *extra, *lang, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compile the CUDA library in place and return its path."""
    os.makedirs(BUILD, exist_ok=True)
    extra_info = ["-Xptxas", "-v"] if ptxas_info else []
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda kv: _compile(kv[0], kv[1] + (extra_info if kv[0].endswith(".cu") else []),
                                               verbose or ptxas_info), SOURCES.items()))
    if _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB + ".tmp", *objs, "-lcudart_static", "-lrt", "-ldl", "-lz",
               "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
