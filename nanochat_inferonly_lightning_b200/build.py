"""Builds libnanochat_attn_sm100.so in-tree with nvcc for sm_100a.

Each csrc/*.cu compiles to an object under _build/ (in parallel), then nvcc links the shared
library next to this file.  cudart is linked statically; the driver's cuTensorMapEncodeTiled
is fetched at run time through cudaGetDriverEntryPoint, so there is no -lcuda dependency.
Rebuilds only what is older than its sources or the shared headers.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libnanochat_attn_sm100.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-Wall", "--expt-relaxed-constexpr"]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h*"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=True, jobs=4):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = _headers()
    objs = []
    todo = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            todo.append((s, o))

    def compile_one(so):
        s, o = so
        cmd = ["nvcc"] + NVCC_FLAGS + ["-c", s, "-o", o]
        if verbose:
            print("[build]", " ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s}:\n{r.stdout}\n{r.stderr}")
        return o

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(compile_one, todo))
    if force or todo or _stale(LIB, objs):
        cmd = ["nvcc"] + ARCH + ["-shared", "-o", LIB] + objs
        if verbose:
            print("[build]", " ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
