"""Build the sm_100a CUDA library (libcdclq_cuda.so) in-tree.

    python cdcl-gptq_b200/build.py [--verbose] [--force]

nvcc cross-compiles for sm_100a without a GPU.  Each .cu file is compiled to an object in parallel (objects
are reused while neither the source nor a header it includes changed), then linked into the shared library.
Flags that matter for the numerics:
  -fmad=false   no implicit a*b+c contraction: the reference (Rust) never contracts, so every rounding outside
                the explicit __fmaf_rn / __fma_rn of the fixed GEMM order must stay a separate multiply and add;
  no --use_fast_math (IEEE division, square root and f16 conversion).
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "cdclq", "libcdclq_cuda.so")
SOURCES = ["engine.cu", "prep.cu", "gptq.cu", "repair.cu", "repair_bm64.cu", "repair_bm128.cu", "gemm.cu", "pack.cu",
           "syrk.cu", "noalloc.cu", "io.cu", "model_io.cu", "runtime.cu", "model.cu"]
HEADERS = ["common.cuh", "gemm_core.cuh", "kernels.h", "repair_core.cuh", "model_io.h", "runtime.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC"]


def nvcc_path():
    for p in (os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"):
        if p and os.path.exists(os.path.join(p, "bin", "nvcc")):
            return os.path.join(p, "bin", "nvcc")
    return "nvcc"


def _includes(path, seen):
    """Local headers a file includes, transitively (quoted includes found in csrc/ or include/)."""
    try:
        text = open(path).read()
    except OSError:
        return seen
    for line in text.splitlines():
        line = line.strip()
        if line.startswith("#include \""):
            name = line.split('"')[1]
            for d in (CSRC, os.path.join(ROOT, "include")):
                h = os.path.join(d, name)
                if os.path.exists(h) and h not in seen:
                    seen.add(h)
                    _includes(h, seen)
                    break
    return seen


def _deps_mtime(src=None):
    """Newest modification time among the headers `src` includes (all shared headers when src is None)."""
    if src is None:
        deps = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "cdclq.h")]
    else:
        deps = sorted(_includes(os.path.join(CSRC, src), set()))
    deps.append(os.path.abspath(__file__))
    return max(os.path.getmtime(d) for d in deps if os.path.exists(d))


def _obj(src):
    return os.path.join(OBJ, src.replace(".cu", ".o"))


def _stale(src):
    o = _obj(src)
    if not os.path.exists(o):
        return True
    t = os.path.getmtime(o)
    return os.path.getmtime(os.path.join(CSRC, src)) > t or _deps_mtime(src) > t


def needs_rebuild():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(_stale(s) for s in SOURCES) or any(os.path.getmtime(_obj(s)) > t for s in SOURCES)


def _compile(src, verbose):
    cmd = [nvcc_path()] + ARCH + FLAGS + ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "-c",
                                          os.path.join(CSRC, src), "-o", _obj(src)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, r


def build(verbose=False, force=False):
    if not force and not needs_rebuild():
        return OUT
    os.makedirs(OBJ, exist_ok=True)
    todo = [s for s in SOURCES if force or _stale(s)]
    failed = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 4))) as ex:
        for src, r in ex.map(lambda s: _compile(s, verbose), todo):
            if verbose or r.returncode != 0:
                sys.stdout.write(r.stdout)
                sys.stderr.write(r.stderr)
            if r.returncode != 0:
                failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed on %s" % ", ".join(failed))
    cmd = [nvcc_path()] + ARCH + ["-shared", "-o", OUT] + [_obj(s) for s in SOURCES] + ["-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stdout.write(r.stdout)
        sys.stderr.write(r.stderr)
        raise RuntimeError("nvcc link failed building %s" % OUT)
    return OUT


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force="--force" in sys.argv)
    print(OUT)
