"""TEST INFRASTRUCTURE ONLY: build the C oracle (oracle/nc_oracle.c -> oracle/libnc_oracle.so).

Plain gcc, baseline x86-64 (no -march=native: the library is built here and run on the GPU
box's host), -O3 without fast-math so float results follow the written expression order,
OpenMP over attention rows.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "nc_oracle.c")
OUT = os.path.join(HERE, "libnc_oracle.so")


def build(force=False, verbose=True):
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    cmd = ["gcc", "-O3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared",
           "-Wall", "-o", OUT, SRC, "-lm"]
    if verbose:
        print("[oracle]", " ".join(cmd))
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv)
