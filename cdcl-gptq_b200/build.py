"""Build the sm_100a CUDA library (libcdclq_cuda.so) in-tree.

    python cdcl-gptq_b200/build.py [--verbose]

nvcc cross-compiles for sm_100a without a GPU.  Flags that matter for the numerics:
  -fmad=false   no implicit a*b+c contraction: the reference (Rust) never contracts, so every rounding outside
                the explicit __fmaf_rn / __fma_rn of the fixed GEMM order must stay a separate multiply and add;
  no --use_fast_math (IEEE division, square root and f16 conversion).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "cdclq", "libcdclq_cuda.so")
SOURCES = ["engine.cu", "prep.cu", "gptq.cu", "repair.cu", "gemm.cu", "pack.cu", "syrk.cu", "noalloc.cu"]
HEADERS = ["common.cuh", "gemm_core.cuh", "kernels.h"]


def nvcc_path():
    for p in (os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"):
        if p and os.path.exists(os.path.join(p, "bin", "nvcc")):
            return os.path.join(p, "bin", "nvcc")
    return "nvcc"


def needs_rebuild():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [os.path.join(ROOT, "include", "cdclq.h"),
                                                                   os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(verbose=False, force=False):
    if not force and not needs_rebuild():
        return OUT
    cmd = [
        nvcc_path(),
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-std=c++17", "-lineinfo", "-fmad=false",
        "-Xcompiler", "-fPIC", "-shared",
        "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
        "-o", OUT,
    ] + [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stdout.write(r.stdout)
        sys.stderr.write(r.stderr)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed building %s" % OUT)
    return OUT


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True)
    print(OUT)
