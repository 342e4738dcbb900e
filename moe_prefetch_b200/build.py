"""Build libmoeb200.so in-tree with nvcc for sm_100a (B200).

    python -m moe_prefetch_b200.build            # build if sources changed
    python -m moe_prefetch_b200.build --force

The library links the CUDA runtime statically, so it loads without a
libcudart on the library path; it shares the device's primary context with
PyTorch, so device pointers and streams pass between them freely.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libmoeb200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-shared",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def deps():
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.h")) +
                              glob.glob(os.path.join(CSRC, "*.cuh")) +
                              [os.path.join(INCLUDE, "moeb200.h")])


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in deps())


def build(force=False, verbose=False):
    if not force and up_to_date():
        return LIB
    cmd = [NVCC] + ARCH + FLAGS + ["-I", INCLUDE, "-I", CSRC, "-o", LIB] + sources()
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
