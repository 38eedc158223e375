"""Build recipe for the oracles (TEST INFRASTRUCTURE ONLY).

1. oracle/libp8oracle.so  -- our plain-C restatement (oracle/p8_oracle.c). Always built.
2. oracle/_ref/            -- the reference's OWN CPU core compiled from the patch text where it lies:
     patches/llama_cpu_vs_7ac59a6.patch  ggml/src/ggml-cpu/vr-native-cpu-core.h  (CP:144-1027)
     patches/llama_cuda_vs_7ac59a6.patch ggml/include/ggml-vr-native.h           (CU:1-51)
     patches/llama_cuda_vs_7ac59a6.patch src/llama-vr3.h                         (CU:3621-3661)
   The new-file hunks are written out (leading '+' stripped) into oracle/_ref/ and compiled with oracle/ref_harness.c
   into two shared objects, one per ISA level, so the box that runs the tests can pick what its CPU supports:
     oracle/_ref/libp8ref_vnni.so (-mavx2 -mfma -mf16c -mavxvnni)   oracle/_ref/libp8ref_avx2.so (-mavx2 -mfma -mf16c)
   Needs the reference checkout (P8_REFERENCE; present only in the build container); when it is absent the step is skipped and the
   prebuilt oracle/_ref/ (git-ignored, shipped with the working tree) is used as is.
3. oracle/_ref/libp8ref_gpu.so -- the reference's OWN batch-1 GEMV kernels (k_vr, k_vr_qx_real) cut from vr49.cuh by
   line markers (GPU_CUTS below) and compiled for sm_100a with the launcher oracle/ref_gpu_harness.cu: the same-box
   GPU comparison arm of bench.py --impl reference and of tests/test_gpu_ref_kernels.py.

Usage: python oracle/build_ref.py [--reference PATH]
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

# (patch file, path of the new file inside the patch, output name)
SOURCES = [
    ("patches/llama_cpu_vs_7ac59a6.patch", "ggml/src/ggml-cpu/vr-native-cpu-core.h", "vr-native-cpu-core.h"),
    ("patches/llama_cuda_vs_7ac59a6.patch", "ggml/include/ggml-vr-native.h", "ggml-vr-native.h"),
    ("patches/llama_cuda_vs_7ac59a6.patch", "src/llama-vr3.h", "llama-vr3.h"),
]


def extract_new_file(patch_path, inner):
    """Return the text of a file ADDED by a unified diff (its single '@@ -0,0 +1,N @@' hunk)."""
    lines = open(patch_path, encoding="utf-8", errors="replace").read().split("\n")
    hdr = f"diff --git a/{inner} b/{inner}"
    i = lines.index(hdr)
    while not lines[i].startswith("@@"):
        i += 1
    out = []
    i += 1
    while i < len(lines) and not lines[i].startswith("diff --git"):
        ln = lines[i]
        if ln.startswith("+"):
            out.append(ln[1:])
        elif ln.startswith("\\") or (ln == "" and i == len(lines) - 1):
            pass
        else:
            raise RuntimeError(f"unexpected line in new-file hunk of {inner}: {ln[:40]!r}")
        i += 1
    return "\n".join(out) + "\n"


def run(cmd):
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_oracle():
    out = os.path.join(HERE, "libp8oracle.so")
    run(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-Wall", "-Wextra",
         "-Wno-unused-function", os.path.join(HERE, "p8_oracle.c"), "-o", out, "-lm"])
    return out


def build_ref(reference):
    if not os.path.isdir(os.path.join(reference, "patches")):
        print(f"build_ref: {reference} not present; keeping prebuilt oracle/_ref", flush=True)
        return False
    os.makedirs(REF_DIR, exist_ok=True)
    for patch, inner, name in SOURCES:
        txt = extract_new_file(os.path.join(reference, patch), inner)
        with open(os.path.join(REF_DIR, name), "w") as f:
            f.write(txt)
    common = ["gcc", "-O2", "-std=gnu11", "-fPIC", "-shared", "-fopenmp", "-Wno-unused-function", "-Wno-unused-variable",
              "-I", REF_DIR, os.path.join(HERE, "ref_harness.c")]
    run(common + ["-mavx2", "-mfma", "-mf16c", "-mavxvnni", "-o", os.path.join(REF_DIR, "libp8ref_vnni.so"), "-lm"])
    run(common + ["-mavx2", "-mfma", "-mf16c", "-o", os.path.join(REF_DIR, "libp8ref_avx2.so"), "-lm"])
    return True


# The reference's shipped batch-1 GEMV kernels, cut from vr49.cuh (a new file of patches/llama_cuda_vs_7ac59a6.patch,
# CU:2514-3260) between these line markers (start line included, end line excluded):
#   vr49_kvr.cuh  CU:2537-2729  format constants, vr_args, vr_run / vr_load helpers and k_vr<RL, V, NWP, NS>
#   vr49_qx.cuh   CU:2950-3018  Hadamard sign copies, warp FWHT and k_vr_qx_real (FWHT256 + int8 quant per 128)
# The rest of vr49.cuh is ggml glue (pool, registry, tensor prepare) that oracle/ref_gpu_harness.cu replaces.
GPU_CUTS = [
    ("vr49_kvr.cuh", "__host__ __device__ constexpr int vrW1(int c)",
     "// ------------------------------------------------------------------------- independent per-weight reference decoder"),
    ("vr49_qx.cuh", "__constant__ float c_vr_sgn[256];", "// R51b fix (b): un-permute by gather"),
]


def cut_between(txt, start, end):
    """The lines of txt from the first line starting with `start` up to (not including) the next line starting with
    `end`; both markers must be present exactly once."""
    lines = txt.split("\n")
    i = [k for k, ln in enumerate(lines) if ln.startswith(start)]
    j = [k for k, ln in enumerate(lines) if ln.startswith(end)]
    if len(i) != 1 or len(j) != 1 or j[0] <= i[0]:
        raise RuntimeError(f"markers not found once each in order: {start[:40]!r} .. {end[:40]!r}")
    return "\n".join(lines[i[0]:j[0]]) + "\n"


def build_ref_gpu(reference):
    """oracle/_ref/libp8ref_gpu.so: the reference's own k_vr + k_vr_qx_real (cut from the patch text) behind the small
    launcher oracle/ref_gpu_harness.cu, for sm_100a. Needs the reference checkout; skipped (prebuilt kept) without it."""
    patch = os.path.join(reference, "patches/llama_cuda_vs_7ac59a6.patch")
    if not os.path.exists(patch):
        print(f"build_ref: {patch} not present; keeping prebuilt oracle/_ref/libp8ref_gpu.so", flush=True)
        return False
    os.makedirs(REF_DIR, exist_ok=True)
    vr49 = extract_new_file(patch, "ggml/src/ggml-cuda/vr49.cuh")
    for name, start, end in GPU_CUTS:
        with open(os.path.join(REF_DIR, name), "w") as f:
            f.write(cut_between(vr49, start, end))
    if not os.path.exists(os.path.join(REF_DIR, "ggml-vr-native.h")):
        with open(os.path.join(REF_DIR, "ggml-vr-native.h"), "w") as f:
            f.write(extract_new_file(patch, "ggml/include/ggml-vr-native.h"))
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    run([nvcc, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-shared",
         "-cudart", "shared", "-Xcompiler", "-fPIC", "-I", REF_DIR, "-diag-suppress", "177,550", os.path.join(HERE, "ref_gpu_harness.cu"),
         "-o", os.path.join(REF_DIR, "libp8ref_gpu.so")])
    return True


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("P8_REFERENCE", "/root/reference"))
    a = ap.parse_args()
    build_oracle()
    build_ref(a.reference)
    build_ref_gpu(a.reference)


if __name__ == "__main__":
    sys.exit(main())
