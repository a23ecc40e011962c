"""Build libqwantize_b200.so in-tree with nvcc for sm_100a.

    python -m qwantize_b200.build [-j N] [--force]

Each translation unit compiles to _build/<name>.o with its own flags (the
quantization kernels need -fmad=false for bit-exact arithmetic), then one
shared library is linked next to this file.  Rebuilds only what changed.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libqwantize_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "-I", os.path.join(ROOT, "include"), "--expt-relaxed-constexpr"]
# per-unit extra flags
UNITS = {
    "qz_quantize.cu": ["-fmad=false"],
    "qz_elementwise.cu": ["-fmad=false"],
    "qz_int.cu": ["-fmad=false"],
    "qz_abi.cu": [],
    "qz_gemm.cu": [],
}


def _deps(src):
    return [src] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))] + \
        [os.path.join(ROOT, "include", "qwantize_b200.h")]


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(jobs: int = 4, force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    objs, todo = [], []
    for unit, extra in UNITS.items():
        src = os.path.join(CSRC, unit)
        obj = os.path.join(BUILD, unit.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, _deps(src)):
            todo.append([NVCC, *ARCH, *COMMON, *extra, "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({cmd[-3]}):\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with ThreadPoolExecutor(max(1, jobs)) as ex:
        for err in ex.map(run, todo):
            if err.strip() and verbose:
                print(err)
    if todo or not os.path.exists(LIB) or _stale(LIB, objs):
        run([NVCC, *ARCH, "-shared", "-o", LIB, *objs])
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(a.j, a.force, a.v))
    sys.exit(0)
