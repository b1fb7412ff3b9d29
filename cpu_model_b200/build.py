"""Build recipe for libmxq.so (sm_100a), in-tree next to this file.

    python -m cpu_model_b200.build

nvcc compiles the CUDA sources for sm_100a only and links a shared library
with a plain C-ABI (include/mxq.h); no torch headers are involved.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SOURCES = ["mxq_api.cu", "mxq_quant.cu", "mxq_gemv.cu", "mxq_rgemv.cu", "mxq_bgemv.cu", "mxq_gemm.cu", "mxq_moe.cu",
           "mxq_ops.cu", "mxq_decoder_kernels.cu", "mxq_decoder.cu", "mxq_cogemv.cu",
           "mxq_tp.cu"]
LIB = os.path.join(HERE, "libmxq.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I" + os.path.join(ROOT, "include"),
]


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc"))]
    deps.append(os.path.join(ROOT, "include", "mxq.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False, ptxas_v=False):
    if not force and not needs_build():
        return LIB
    objs = []
    for src in SOURCES:
        obj = os.path.join(HERE, "csrc", src.replace(".cu", ".o"))
        cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if ptxas_v else []) + [
            "-c", os.path.join(HERE, "csrc", src), "-o", obj]
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.check_call([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
                           "-o", tmp] + objs)
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="--ptxas-v" in sys.argv)
    print(LIB)
