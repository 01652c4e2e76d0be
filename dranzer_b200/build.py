"""Builds dranzer_b200/libdz_cuda.so in-tree: the sm_100a CUDA shim (nvcc) and
the plain-C host library (gcc), linked with the static CUDA runtime.

    python -m dranzer_b200.build        # or __graft_entry__.build()
"""
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libdz_cuda.so")

NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"]
CC_FLAGS = ["-O2", "-fPIC", "-std=c11", "-Wall", "-Wextra", "-fno-fast-math", "-ffp-contract=off",
            f"-I{INCLUDE}"]

CUDA_SOURCES = ["dz_cuda.cu", "qmvi.cu", "seqgen.cu", "attn.cu", "pfattn.cu"]
C_SOURCES = ["dz_host.c"]


def _nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _deps():
    out = []
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".cu", ".cuh", ".c", ".h")):
                out.append(os.path.join(d, f))
    return out


def build(verbose=False, force=False):
    os.makedirs(BUILD, exist_ok=True)
    deps = _deps() + [os.path.abspath(__file__)]
    objs = []
    run = (lambda cmd: subprocess.run(cmd, check=True)) if verbose else \
        (lambda cmd: subprocess.run(cmd, check=True, stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    for src in CUDA_SOURCES:
        obj = os.path.join(BUILD, src + ".o")
        if force or _newer(obj, deps):
            try:
                run([_nvcc(), *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj])
            except subprocess.CalledProcessError as e:
                sys.stderr.write(e.stdout.decode() if e.stdout else "")
                raise
        objs.append(obj)
    for src in C_SOURCES:
        obj = os.path.join(BUILD, src + ".o")
        if force or _newer(obj, deps):
            try:
                run(["gcc", *CC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj])
            except subprocess.CalledProcessError as e:
                sys.stderr.write(e.stdout.decode() if e.stdout else "")
                raise
        objs.append(obj)
    if force or _newer(LIB, objs):
        run([_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs,
             "-cudart", "static", "-lm", "-lpthread", "-ldl", "-lrt"])
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
