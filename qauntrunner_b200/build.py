"""Builds libqrmoe.so (the C-ABI library of include/qrmoe.h) in-tree.

    python -m qauntrunner_b200.build [--ptxas-v]

Every translation unit is compiled for sm_100a only.  The quantiser unit
(synth.cu) is compiled with -fmad=false so its float expressions are exactly
the reference quantiser's operations; the kernels that must reproduce the
reference bit for bit (routing, combine) use explicit _rn intrinsics instead.
"""
import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib", "libqrmoe.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"),
          "--expt-relaxed-constexpr"]
UNITS = [("qrmoe.cu", []), ("umma.cu", []), ("qwfile.cu", []), ("synth.cu", ["-fmad=false"])]


def nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources_newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(ptxas_verbose=False, force=False, quiet=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    headers.append(os.path.join(ROOT, "include", "qrmoe.h"))
    objs = []
    for src, extra in UNITS:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or ptxas_verbose or sources_newer(o, [s, __file__] + headers):
            cmd = [nvcc()] + ARCH + COMMON + extra + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", s, "-o", o]
            if not quiet:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or sources_newer(LIB, objs):
        # NCCL (expert parallelism): libnccl.so.2 resolves at load time; in a
        # process that imported torch it is the copy torch already loaded
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lnccl", "-lpthread"]
        if not quiet:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build(ptxas_verbose=a.ptxas_v, force=a.force)
    print(LIB)
    sys.exit(0)
