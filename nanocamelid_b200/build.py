"""Builds libncm.so in-tree (nanocamelid_b200/libncm.so) for sm_100a.

nvcc compiles the CUDA sources with -fmad=false so that f32 expressions round as the
reference's unfused Rust arithmetic does; the host GGUF writer is compiled with
-ffp-contract=off for the same reason.  Parallel, incremental (object files are
rebuilt only when a source or header is newer).
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libncm.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["kernels.cu", "engine.cu"]
CPP_SOURCES = ["gguf.cpp", "libm_table.cpp"]


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(os.path.dirname(HERE), "include", "ncm.h"))
    return hs


def _stale(obj, src):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src] + _headers())


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(verbose=False, ptxas_info=False):
    os.makedirs(BUILD, exist_ok=True)
    jobs = []
    objs = []
    for f in CU_SOURCES:
        src, obj = os.path.join(CSRC, f), os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if _stale(obj, src) or ptxas_info:
            cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC,-ffp-contract=off",
                   "-c", src, "-o", obj]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    for f in CPP_SOURCES:
        src, obj = os.path.join(CSRC, f), os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if _stale(obj, src):
            jobs.append(["g++", "-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-fno-fast-math",
                         "-I/usr/local/cuda/include", "-c", src, "-o", obj])
    if jobs:
        with ThreadPoolExecutor(max_workers=len(jobs)) as ex:
            outs = list(ex.map(_run, jobs))
        if verbose:
            for o in outs:
                sys.stdout.write(o)
    if jobs or not os.path.exists(LIB):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-ldl", "-lpthread",
              "-Xlinker", "-rpath,/usr/local/cuda/lib64"])
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
