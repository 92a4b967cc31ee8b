"""Builds libt0b.so (all CUDA kernels + the C ABI) in-tree for sm_100a.

nvcc cross-compiles without a GPU, so this runs on any machine with the CUDA
toolkit.  Usage: python -m t0_web_b200.build  (or build() from Python).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libt0b.so")
OBJ = os.path.join(HERE, "_build")
# the checked build: every T0B_CHECK index check compiled in (a failed check
# records T0B_DEVERR_BOUNDS and skips the access); used by the tests only
LIB_CHECKED = os.path.join(HERE, "libt0b_checked.so")
OBJ_CHECKED = os.path.join(HERE, "_build_checked")

CU_SOURCES = ["t0b_model.cu", "k_gemm_small.cu", "k_gemm_tc.cu", "k_misc.cu"]
CPP_SOURCES = ["gguf_host.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or os.path.exists(c)):
            return c
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False, checked: bool = False) -> str:
    """Builds libt0b.so (checked=True: libt0b_checked.so with -DT0B_CHECKED)."""
    obj_dir, lib_path = (OBJ_CHECKED, LIB_CHECKED) if checked else (OBJ, LIB)
    defs = ["-DT0B_CHECKED"] if checked else []
    os.makedirs(obj_dir, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(ROOT, "include", "t0b.h"))
    objs = []
    nvcc = _nvcc()
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(obj_dir, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-ffp-contract=off", "-rdc=false",
                   *defs, "-I", CSRC, "-I", os.path.join(ROOT, "include"), "-c", s, "-o", o]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd))
            subprocess.run(cmd, check=True)
    for src in CPP_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(obj_dir, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            subprocess.run(["g++", "-O2", "-fPIC", "-ffp-contract=off", "-std=c++17", "-I", CSRC, "-c", s, "-o", o],
                           check=True)
    if force or _stale(lib_path, objs):
        subprocess.run([nvcc, *ARCH, "-shared", "-o", lib_path, *objs, "-lcudart"], check=True)
    return lib_path


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv, checked="--checked" in sys.argv))
