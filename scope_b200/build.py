"""Builds libscope_b200.so in-tree with nvcc for sm_100a.

    python -m scope_b200.build          # or scope_b200.build.build()

Every .cu under scope_b200/csrc is compiled for
``-gencode arch=compute_100a,code=sm_100a`` (no other architecture; the
kernels use tcgen05/TMA instructions that exist only there) into one shared
library with a plain C ABI (include/scope_b200.h).  fp32 division and square
root stay IEEE (no --use_fast_math) so the mask builder's float steps match
the reference bit for bit; the mask builder is compiled with FMA contraction
off for the same reason.
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
OUT = os.path.join(PKG, "libscope_b200.so")
BUILD = os.path.join(ROOT, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NO_FMA = {"mask_build.cu"}


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def build(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    inc = ["-I", os.path.join(ROOT, "include")]
    common = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"] + inc
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]

    def compile_one(src):
        obj = os.path.join(BUILD, src[:-3] + ".o")
        flags = list(common)
        if src in NO_FMA:
            flags += ["-fmad=false"]
        cmd = [nvcc] + flags + ["-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose or ptxas_verbose:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}")
        return obj

    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(compile_one, srcs))
    tmp = OUT + ".tmp"
    cmd = [nvcc] + ARCH + ["-shared", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link failed")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv))
