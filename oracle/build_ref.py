"""TEST INFRASTRUCTURE ONLY: rebuild the reference's kernels and engine for sm_100a.

1. oracle/_ref/libref_attn.so: kernels/rope.cu, kernels/flash_attention.cu, kernels/rmsnorm.cu
   and kernels/ops.cu of the reference project, compiled from where they lie (never copied)
   through oracle/ref_shim.cu with the namespace renamed to nanochat_ref.
2. The reference's host engine, unmodified (src/model.cpp, src/engine.cpp with
   kernels/rmsnorm.cu, kernels/ops.cu and kernels/gemm.cu; gemm.cu needs CUTLASS headers: the
   reference pins v3.4.1, which cannot be fetched offline, so the CUTLASS 4.5 headers vendored
   with the flashinfer package are used), plus oracle/ref_model_shim.cpp, linked twice:
     oracle/_ref/libref_model_ref.so  with the reference's own rope.cu and flash_attention.cu;
     oracle/_ref/libref_model_nc.so   against libnanochat_attn_sm100.so instead (the link-level
                                      drop-in of this library's nanochat:: entry points).
The outputs are git-ignored but travel to the GPU box with the working tree; the reference
tree itself is only needed for this build.
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


def cutlass_include():
    """CUTLASS headers for the reference's kernels/gemm.cu: $NC_CUTLASS_INCLUDE, else the copy
    vendored with the installed flashinfer package."""
    env = os.environ.get("NC_CUTLASS_INCLUDE")
    if env:
        return env
    import sysconfig

    cand = os.path.join(sysconfig.get_paths()["purelib"], "flashinfer", "data", "cutlass",
                        "include")
    return cand if os.path.isdir(os.path.join(cand, "cutlass")) else None


MODEL_REF = os.path.join(OUT_DIR, "libref_model_ref.so")
MODEL_NC = os.path.join(OUT_DIR, "libref_model_nc.so")


def build_model(ref_root=None, force=False, verbose=True, jobs=4):
    """The reference engine linked with its own attention kernels and with this library's."""
    import concurrent.futures as cf

    ref_root = ref_root or reference_root()
    cutlass = cutlass_include()
    pkg = os.path.join(os.path.dirname(HERE), "nanochat_inferonly_lightning_b200")
    nc_lib = os.path.join(pkg, "libnanochat_attn_sm100.so")
    if not ref_root or not os.path.exists(os.path.join(ref_root, "src", "model.cpp")):
        if verbose:
            print("[oracle] reference tree not found; keeping existing reference engine builds")
        return os.path.exists(MODEL_REF) and os.path.exists(MODEL_NC)
    if not cutlass:
        if verbose:
            print("[oracle] CUTLASS headers not found (set NC_CUTLASS_INCLUDE); reference engine "
                  "not built")
        return False
    sdir, kdir = os.path.join(ref_root, "src"), os.path.join(ref_root, "kernels")
    common = [os.path.join(sdir, "model.cpp"), os.path.join(sdir, "engine.cpp"),
              os.path.join(kdir, "rmsnorm.cu"), os.path.join(kdir, "ops.cu"),
              os.path.join(kdir, "gemm.cu"), os.path.join(HERE, "ref_model_shim.cpp")]
    attn = [os.path.join(kdir, "rope.cu"), os.path.join(kdir, "flash_attention.cu")]
    srcs = common + attn
    if not force and os.path.exists(MODEL_REF) and os.path.exists(MODEL_NC):
        newest = max(os.path.getmtime(x) for x in srcs)
        if min(os.path.getmtime(MODEL_REF), os.path.getmtime(MODEL_NC)) >= newest:
            return True
    obj_dir = os.path.join(OUT_DIR, "obj")
    os.makedirs(obj_dir, exist_ok=True)
    flags = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
             "-DNDEBUG", "-I" + sdir, "-I" + cutlass, "-Xcompiler", "-fPIC", "-w"]

    def obj(src):
        o = os.path.join(obj_dir, os.path.basename(src).replace(".", "_") + ".o")
        cmd = flags + ["-x", "cu", "-c", src, "-o", o]
        if verbose:
            print("[oracle]", " ".join(cmd))
        subprocess.run(cmd, check=True)
        return o

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(obj, srcs))
    common_o, attn_o = objs[:len(common)], objs[len(common):]
    link = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-shared"]
    subprocess.run(link + ["-o", MODEL_REF] + common_o + attn_o, check=True)
    subprocess.run(link + ["-o", MODEL_NC] + common_o +
                   ["-L" + pkg, "-l:libnanochat_attn_sm100.so",
                    "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN/../../nanochat_inferonly_lightning_b200"],
                   check=True)
    return os.path.exists(nc_lib)


if __name__ == "__main__":
    ok = build(force="--force" in sys.argv)
    ok = build_model(force="--force" in sys.argv) and ok
    sys.exit(0 if ok else 1)
