"""Build the C-ABI library libsam3cuda.so in-tree for sm_100a.

CUDA sources are compiled by nvcc with ``-gencode arch=compute_100a,
code=sm_100a -lineinfo``; the C host layer by gcc; the CUDA runtime is
linked statically so the library does not depend on the runtime that the
loading process (e.g. torch) brings. Rebuilds only what changed.

    python i.sam3.opencl_b200/build.py [--force] [--verbose]
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INC = os.path.join(ROOT, "include")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsam3cuda.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

CU = ["gemm_tc.cu", "attn_tc.cu", "attn_simt.cu", "attn_decoder.cu", "elementwise.cu", "attn_noalloc.cu",
      "decoder.cu", "neck.cu", "input.cu",
      "detector.cu"]
C = ["cuda_backend.c", "sam3_ops.c", "sam3_encoder.c", "sam3_decoder.c", "sam3_neck.c", "sam3_input.c",
     "synth.c"]
HEADERS = ["tc_ptx.cuh", "tmap.cuh", "pdl.cuh", "kernels.h", "backend_internal.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
              "-Xptxas", "-warn-spills", "-I" + INC, "-I" + CSRC] + ARCH
CC_FLAGS = ["-std=gnu11", "-O2", "-fPIC", "-fopenmp", "-Wall", "-Wno-unused-function",
            "-I" + INC, "-I" + CSRC, "-I" + os.path.join(CUDA, "include")]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def build(force=False, verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    deps_common = [os.path.join(CSRC, h) for h in HEADERS] + \
        [os.path.join(INC, h) for h in os.listdir(INC) if h.endswith(".h")]
    objs = []
    for f in CU:
        src = os.path.join(CSRC, f)
        obj = os.path.join(OBJ, f + ".o")
        if force or _newer(obj, [src] + deps_common):
            _run([NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj], verbose)
        objs.append(obj)
    for f in C:
        src = os.path.join(CSRC, f)
        obj = os.path.join(OBJ, f + ".o")
        if force or _newer(obj, [src] + deps_common):
            _run(["gcc"] + CC_FLAGS + ["-c", src, "-o", obj], verbose)
        objs.append(obj)
    if force or _newer(LIB, objs + [os.path.join(CSRC, "exports.map")]):
        _run([NVCC, "-shared"] + ARCH + ["-o", LIB] + objs +
             ["-cudart", "static", "-Xcompiler", "-fopenmp", "-lgomp",
              "-Xlinker", "--version-script=" + os.path.join(CSRC, "exports.map")],
             verbose)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB)
