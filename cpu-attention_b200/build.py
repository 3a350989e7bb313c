"""Builds libca_b200.so (the sm_100a kernels behind the C ABI) in-tree.

    python cpu-attention_b200/build.py [--force] [--verbose]

One nvcc process per translation unit, in parallel: csrc/ca_abi.cu (the C ABI,
the store and prefill kernels), csrc/decode_bf16.cu and csrc/decode_f32.cu (the
decode kernel's instantiations) and csrc/ca_noalloc.cu (the allocation-free
decode entry), objects under cpu-attention_b200/_build/, linked into
cpu_attention/libca_b200.so; sm_100a only, with line info, static CUDA runtime. Rebuilds only when a source or this script is newer than the
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


UNITS = ["ca_abi.cu", "ca_noalloc.cu", "decode_bf16.cu", "decode_f32.cu"]


def build(force=False, verbose=False):
    """Compile the library if needed; returns its path. Each translation unit
    compiles in its own nvcc process (in parallel), then one link."""
    if not force and not stale():
        return OUT
    from concurrent.futures import ThreadPoolExecutor

    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    flags = [f for f in FLAGS if f != "-shared"]

    def compile_unit(unit):
        obj = os.path.join(objdir, unit.replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, *flags, "-c", "-o", obj, os.path.join(CSRC, unit)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        return obj

    with ThreadPoolExecutor(max_workers=len(UNITS)) as pool:
        objs = list(pool.map(compile_unit, UNITS))
    tmp = OUT + ".tmp"
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs], check=True)
    os.replace(tmp, OUT)
    return OUT


FAST_SRC = os.path.join(CSRC, "fastpath.cpp")


def fastpath_out():
    import sysconfig

    return os.path.join(HERE, "cpu_attention", "_fastpath" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_fastpath(force=False, verbose=False):
    """Compile cpu_attention/_fastpath (the decode host path in C++, a torch
    extension linked against libca_b200.so) if needed; returns its path."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension

    out = fastpath_out()
    deps = [FAST_SRC, OUT, os.path.join(ROOT, "include", "cpu_attention_b200.h"), os.path.abspath(__file__)]
    if not force and os.path.exists(out) and all(os.path.getmtime(f) <= os.path.getmtime(out) for f in deps):
        return out
    gxx = shutil.which("g++") or "g++"
    incs = cpp_extension.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    libdirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [gxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_fastpath", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{d}" for d in incs], FAST_SRC, "-o", out + ".tmp",
           *[f"-L{d}" for d in libdirs], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
           f"-L{os.path.dirname(OUT)}", "-lca_b200", "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{d}" for d in libdirs]]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    print(build_fastpath(a.force, a.verbose))
    sys.exit(0)
