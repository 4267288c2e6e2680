"""Build libg1env.so (the sm_100a fused rollout + its C-ABI) in-tree with nvcc.

    python g1.cu_b200/build.py [--force]

The library is the product: no CPU fallback exists, and g1env.py refuses to run without it.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libg1env.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--shared", "-diag-suppress", "550"]


def sources():
    srcs = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    srcs.append(os.path.join(HERE, "..", "include", "g1env.h"))
    return srcs


def build(force=False, verbose=False, extra=()):
    if not force and os.path.exists(LIB):
        t = os.path.getmtime(LIB)
        if all(os.path.getmtime(s) <= t for s in sources()) and os.path.getmtime(__file__) <= t:
            return LIB
    cmd = ["nvcc"] + ARCH + FLAGS + list(extra) + [os.path.join(CSRC, "g1_env.cu"), "-o", LIB]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose:
        print(r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
