"""Build the sm_100a shared library ``blitzgs_b200/lib/libblitzgs_b200.so``.

nvcc compiles every ``csrc/*.cu`` for ``arch=compute_100a,code=sm_100a`` with
``-O3 -lineinfo`` and no fast-math (bit-exact culling depends on IEEE divide,
sqrt and the reference's FMA contraction pattern), then links one shared
library with the C ABI of ``include/blitzgs_b200.h``.  The CUDA runtime is
linked statically so the library does not depend on which libcudart the
host process (PyTorch) ships.  Cross-compiles without a GPU.

Usage: python -m blitzgs_b200.build [--force] [--jobs N]
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(OUT_DIR, "libblitzgs_b200.so")
OBJ_DIR = os.path.join(ROOT, "_build", "obj")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC]


def nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build blitzgs_b200")
    return cand


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, force):
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + ".o")
    if not force and not _stale(obj, [src] + headers() + [__file__]):
        return obj
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force=False, jobs=None, verbose=True):
    """Compile and link the library if any source is newer than it.  Returns its path."""
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = sources()
    if not force and not _stale(LIB, srcs + headers() + [__file__]):
        return LIB
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", tmp] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print(f"[blitzgs_b200] built {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args()
    build(force=a.force, jobs=a.jobs)
    sys.exit(0)
