"""Build the in-tree CUDA library pingala8_llm_b200/libpingala8_b200.so for sm_100a (nvcc, no JIT cache).

usage: python -m pingala8_llm_b200.build  [--verbose-ptxas]
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libpingala8_b200.so")
SOURCES = ["p8_host.cpp", "p8_gguf.cpp", "p8_api.cu", "p8_kernels.cu", "p8_noalloc.cu", "p8_tp.cu", "p8_encode.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or os.path.exists(c)):
            return c
    return "nvcc"


def build(verbose_ptxas=False, out=LIB, csrc=None, bdir=None):
    csrc = csrc or CSRC
    objs = []
    bdir = bdir or os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)
    for s in SOURCES:
        src = os.path.join(csrc, s)
        obj = os.path.join(bdir, s + ".o")
        cmd = [nvcc(), "-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-O2,-Wall", "-c", src, "-o", obj,
               "-I", csrc, "-I", os.path.join(os.path.dirname(HERE), "include")]
        if s.endswith(".cu") and verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
        print("+", " ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    cmd = [nvcc(), "-shared", *ARCH, *objs, "-o", out, "-lcudart"]
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    build(a.verbose_ptxas)
    sys.exit(0)
