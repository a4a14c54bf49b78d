"""TEST INFRASTRUCTURE ONLY: rebuild the reference's kernels for sm_100a.

Compiles kernels/rope.cu, kernels/flash_attention.cu, kernels/rmsnorm.cu and kernels/ops.cu of
the reference project from where they lie (never copied) through oracle/ref_shim.cu, with the
namespace renamed to nanochat_ref, into oracle/_ref/libref_attn.so.  The output is git-ignored but travels to the
GPU box with the working tree; the reference tree itself is only needed for this build.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "libref_attn.so")


def reference_root():
    """The reference project's source tree: $NC_REFERENCE_ROOT, else the `reference_path` that
    BASELINE.json at the repository root records, else None."""
    env = os.environ.get("NC_REFERENCE_ROOT")
    if env:
        return env
    import json

    bj = os.path.join(os.path.dirname(HERE), "BASELINE.json")
    try:
        with open(bj) as f:
            return json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None


def build(ref_root=None, force=False, verbose=True):
    ref_root = ref_root or reference_root()
    if not ref_root:
        if verbose:
            print("[oracle] no reference tree given (set NC_REFERENCE_ROOT); keeping existing "
                  f"{OUT}")
        return os.path.exists(OUT)
    kdir = os.path.join(ref_root, "kernels")
    sdir = os.path.join(ref_root, "src")
    srcs = [os.path.join(kdir, "rope.cu"), os.path.join(kdir, "flash_attention.cu"),
            os.path.join(kdir, "rmsnorm.cu"), os.path.join(kdir, "ops.cu"),
            os.path.join(HERE, "ref_shim.cu")]
    if not all(os.path.exists(s) for s in srcs[:4]):
        if verbose:
            print(f"[oracle] reference tree not found at {ref_root}; keeping existing {OUT}")
        return os.path.exists(OUT)
    if not force and os.path.exists(OUT):
        newest = max(os.path.getmtime(s) for s in srcs)
        if os.path.getmtime(OUT) >= newest:
            return True
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
           "-Dnanochat=nanochat_ref", "-I" + kdir, "-I" + sdir, "-Xcompiler", "-fPIC",
           "-shared", "-lineinfo", "-o", OUT, os.path.join(HERE, "ref_shim.cu")]
    if verbose:
        print("[oracle]", " ".join(cmd))
    subprocess.run(cmd, check=True)
    return True


if __name__ == "__main__":
    ok = build(force="--force" in sys.argv)
    sys.exit(0 if ok else 1)
