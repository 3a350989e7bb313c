"""Builds libca_b200.so (the sm_100a kernels behind the C ABI) in-tree.

    python cpu-attention_b200/build.py [--force] [--verbose]

One nvcc invocation: csrc/ca_abi.cu (which includes every kernel) and
csrc/ca_noalloc.cu (the allocation-free decode entry) ->
cpu_attention/libca_b200.so, compiled for sm_100a only, with line info, static
CUDA runtime. Rebuilds only when a source or this script is newer than the
library. nvcc cross-compiles, so this runs on a machine without a GPU.
"""

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "cpu_attention", "libca_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-DNDEBUG"]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found (CUDA 12.8+ is needed for sm_100a)")
    return exe


def sources():
    files = glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    files.append(os.path.join(ROOT, "include", "cpu_attention_b200.h"))
    files.append(os.path.abspath(__file__))
    return files


def stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(f) > t for f in sources())


def build(force=False, verbose=False):
    """Compile the library if needed; returns its path."""
    if not force and not stale():
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *ARCH, *FLAGS, "-o", tmp, os.path.join(CSRC, "ca_abi.cu"), os.path.join(CSRC, "ca_noalloc.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    sys.exit(0)
