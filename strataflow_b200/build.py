"""Build libsfk.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m strataflow_b200.build          # or __graft_entry__.build()

Output: strataflow_b200/_lib/libsfk.so.  The library is a plain C-ABI shared
object (include/sfk.h); it links the CUDA runtime statically and has no
dependency on PyTorch.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(OUT_DIR, "libsfk.so")
OBJ_DIR = os.path.join(ROOT, "_build", "sfk")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "-I", CSRC, "-I", os.path.join(ROOT, "include")] + ARCH
# per-file extra flags: the synthetic generator must round exactly as written
EXTRA = {"sfk_synth.cu": ["-fmad=false"]}
SOURCES = ["sfk_kernels.cu", "sfk_mega.cu", "sfk_tc.cu", "sfk_prefill.cu", "sfk_sample.cu", "sfk_synth.cu", "sfk_api.cu", "sfk_noalloc.cu",
           "sfk_strata.cpp", "sfk_tier.cpp"]
HEADERS = ["sfk_device.cuh", "sfk_act.cuh", "sfk_dequant.cuh", "sfk_kernels.cuh", "sfk_route.cuh", "sfk_mega.cuh",
           "sfk_tc.cuh", "sfk_prefill.cuh", "sfk_sample.cuh", "sfk_tier.h"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "sfk.h")]
    objs = []
    for src in SOURCES:
        sp = os.path.join(CSRC, src)
        obj = os.path.join(OBJ_DIR, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        if force or ptxas_info or _stale(obj, [sp] + hdrs + [__file__]):
            cmd = [nvcc()] + COMMON + EXTRA.get(src, []) + (["-Xptxas", "-v"] if ptxas_info else []) + \
                  ["-c", sp, "-o", obj]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", LIB] + objs + ["-lcudart_static", "-lrt",
                                                                                     "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
