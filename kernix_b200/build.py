"""Build kernix_b200/libkernix.so: the .knx runtime (C) and its sm_100a CUDA kernels.

    python -m kernix_b200.build [--force] [--verbose]

nvcc compiles every .cu for sm_100a only (-gencode arch=compute_100a,code=sm_100a), gcc compiles the host C;
the shared library links the CUDA runtime statically, so it loads on a machine without a GPU (calls then fail
with "no CUDA device") and needs only the driver's libcuda at run time. Objects go to kernix_b200/_build/.
"""
import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libkernix.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
                     "-I" + INCLUDE, "-I" + CSRC]
CC_FLAGS = ["-std=gnu11", "-O2", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra", "-Wno-unused-parameter",
            "-I" + INCLUDE, "-I" + CSRC, "-I" + os.path.join(CUDA_HOME, "include")]

CU_SOURCES = ["kx_gemm.cu", "kx_ops.cu", "kx_noalloc.cu", "kx_attn.cu", "kx_tensor.cu", "kx_mlp.cu"]
C_SOURCES = ["knx_load.c", "knx_model.c", "knx_nccl.c"]
HEADERS = ["kx_sm100.cuh", "kx_act.cuh", "kx_pdl.cuh", "kx_internal.h"]


def _newer(src_list, dst):
    if not os.path.exists(dst):
        return True
    t = os.path.getmtime(dst)
    return any(os.path.getmtime(s) > t for s in src_list)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)
    return r


def build(force=False, verbose=False, ptxas_info=False):
    """Compile the library if any source changed. Returns the path of libkernix.so."""
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, h) for h in os.listdir(INCLUDE)]
    objs = []
    for f in CU_SOURCES:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if force or _newer([src] + hdrs, obj):
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            r = _run([NVCC] + NVCC_FLAGS + extra + ["-c", src, "-o", obj], verbose)
            if ptxas_info:
                sys.stderr.write(r.stderr)
    for f in C_SOURCES:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f + ".o")
        objs.append(obj)
        if force or _newer([src] + hdrs, obj):
            _run(["gcc"] + CC_FLAGS + ["-c", src, "-o", obj], verbose)
    if force or _newer(objs, LIB):
        tmp = LIB + ".tmp"
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs + ["-ldl", "-lrt", "-lpthread"], verbose)
        os.replace(tmp, LIB)
    return LIB


def clean():
    shutil.rmtree(BUILD, ignore_errors=True)
    if os.path.exists(LIB):
        os.remove(LIB)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose, a.ptxas_info))
