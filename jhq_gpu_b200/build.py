"""Build libjhq_b200.so in-tree: nvcc for the sm_100a CUDA sources, g++ for the
host C++ (with -ffp-contract=off so the CPU training steps match the
reference's cpu/ bit for bit). Incremental on file modification times.

    python -m jhq_gpu_b200.build [--verbose-ptxas] [--force]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libjhq_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr", f"-I{INCLUDE}"]
CXX_FLAGS = ["-O3", "-fPIC", "-std=c++17", "-ffp-contract=off", f"-I{INCLUDE}"]


def _nvcc() -> str:
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _cuda_home() -> str:
    return os.path.dirname(os.path.dirname(os.path.realpath(_nvcc())))


def _headers():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))] + \
        [os.path.join(INCLUDE, "jhq.h")]


def _stale(obj: str, src: str, headers) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + list(headers))


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = _nvcc()
    headers = _headers()
    objs, changed = [], False
    for f in sorted(os.listdir(CSRC)):
        src = os.path.join(CSRC, f)
        if f.endswith(".cu"):
            obj = os.path.join(OUT_DIR, f[:-3] + ".o")
            cmd = [nvcc] + ARCH + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else []) + \
                ["-c", src, "-o", obj]
        elif f.endswith(".cpp"):
            obj = os.path.join(OUT_DIR, f[:-4] + ".o")
            cmd = ["g++"] + CXX_FLAGS + [f"-I{_cuda_home()}/include", "-c", src, "-o", obj]
        else:
            continue
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, src, headers):
            print("[build]", " ".join(os.path.basename(c) if c == src else c for c in cmd[:1] + [f]),
                  flush=True)
            subprocess.run(cmd, check=True)
            changed = True
    if changed or force or not os.path.exists(LIB):
        cmd = [nvcc] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas))


if __name__ == "__main__":
    sys.exit(main())
