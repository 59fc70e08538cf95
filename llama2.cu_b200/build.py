"""Builds libb200_sampler.so in-tree with nvcc for sm_100a.

Usage: python llama2.cu_b200/build.py [--verbose]
The library is written next to this file (llama2.cu_b200/libb200_sampler.so).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libb200_sampler.so")
SOURCES = ["sampler_kernels.cu", "row_stream.cu", "classifier_gemm.cu", "sampler_api.cu", "noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def build(verbose=False, force=False):
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(ROOT, "include", "b200_sampler.h"))
    if not force and os.path.exists(LIB):
        lib_t = os.path.getmtime(LIB)
        if all(os.path.getmtime(d) <= lib_t for d in deps):
            return LIB
    objs = []
    for src in srcs:
        obj = os.path.join(CSRC, os.path.basename(src) + ".o")
        cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
               "-I" + os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
        objs.append(obj)
    cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", LIB, *objs, "-ldl"]
    subprocess.run(cmd, check=True)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
