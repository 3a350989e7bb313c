"""TEST INFRASTRUCTURE ONLY. ctypes access to ``ca_oracle.c`` -- the C
restatement of the reference's CPU kernel -- over numpy arrays or CPU torch
tensors, and its build.

The library is compiled for three x86-64 levels (v4: AVX-512, v3: AVX2+FMA,
baseline) so the copy that travels to another host runs there; ``load()`` picks
the best one this CPU supports. Threads: all host cores unless told otherwise.
"""

import ctypes
import os
import shutil
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ca_oracle.c")
LIBDIR = os.path.join(HERE, "lib")
LEVELS = [("v4", "x86-64-v4", {"avx512f", "avx512bw", "avx512vl", "avx512dq"}),
          ("v3", "x86-64-v3", {"avx2", "fma", "bmi2"}),
          ("base", "x86-64", set())]


def lib_path(level):
    return os.path.join(LIBDIR, f"liboracle_{level}.so")


def build(force=False):
    """Compile ca_oracle.c for every level (skipped when up to date)."""
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler for the oracle")
    os.makedirs(LIBDIR, exist_ok=True)
    for level, march, _ in LEVELS:
        out = lib_path(level)
        if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(SRC):
            continue
        subprocess.run([cc, "-O3", f"-march={march}", "-fopenmp", "-fPIC", "-shared", "-o", out + ".tmp", SRC,
                        "-lm"], check=True)
        os.replace(out + ".tmp", out)


def cpu_flags():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


_LIB = []


def load():
    if _LIB:
        return _LIB[0]
    if not all(os.path.exists(lib_path(level)) for level, _, _ in LEVELS):
        build()
    flags = cpu_flags()
    level = next(lv for lv, _, need in LEVELS if need <= flags)
    lib = ctypes.CDLL(lib_path(level))
    P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
    PI64 = ctypes.POINTER(ctypes.c_int64)
    lib.oracle_store.argtypes = [P, P, I64, P, P, I64, P, I64, I64, I64, I64, I32]
    lib.oracle_store.restype = None
    lib.oracle_decode.argtypes = [P, I64, P, P, I64, P, P, I64, P, P, P, I64, P, I64, I64, I64, I64, I32, F, I32]
    lib.oracle_decode.restype = None
    lib.oracle_flash.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, PI64, PI64, PI64, F, I32, I32, I32]
    lib.oracle_flash.restype = None
    _LIB.append(lib)
    _LIB.append(level)
    return lib


def level():
    load()
    return _LIB[1]


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        assert x.flags.c_contiguous or x.ndim == 0
        return x.ctypes.data
    return x.data_ptr()  # a CPU torch tensor


def _dtype_code(x):
    name = str(x.dtype)
    if name in ("uint16", "torch.bfloat16", "torch.int16"):
        return 1
    if name in ("float32", "torch.float32"):
        return 0
    raise TypeError(f"oracle: unsupported dtype {x.dtype}")


def _nan():
    return float("nan")


def store(key, value, k_cache, v_cache, slots):
    """reshape_and_cache on CPU tensors/arrays (caches mutated in place)."""
    lib = load()
    n, heads, hd = key.shape
    stride = key.strides[0] // key.itemsize if isinstance(key, np.ndarray) else key.stride(0)
    lib.oracle_store(_ptr(key), _ptr(value), stride, _ptr(k_cache), _ptr(v_cache), k_cache.shape[0], _ptr(slots),
                     n, heads, hd, k_cache.shape[2], _dtype_code(key))


def decode(q, k_cache, v_cache, lens, page_table, out, k_new=None, v_new=None, slots=None, scale=None,
           threads=0):
    """Paged decode on CPU tensors (the `_C.decode` contract); q/out [B, H, E]
    rows with any sequence stride for q, out contiguous."""
    lib = load()
    b, heads, hd = q.shape[0], q.shape[-2], q.shape[-1]
    qstride = q.stride(0) if not isinstance(q, np.ndarray) else q.strides[0] // q.itemsize
    kvs = 0
    if k_new is not None:
        kvs = k_new.stride(0) if not isinstance(k_new, np.ndarray) else k_new.strides[0] // k_new.itemsize
    lib.oracle_decode(_ptr(q), qstride, _ptr(k_cache), _ptr(v_cache), k_cache.shape[0], _ptr(k_new), _ptr(v_new),
                      kvs, _ptr(slots), _ptr(lens), _ptr(page_table), page_table.shape[1], _ptr(out), b, heads, hd,
                      k_cache.shape[2], _dtype_code(q), _nan() if scale is None else float(scale), threads)


def flash(q, k, v, out, scale=None, causal=False, threads=0):
    """flash_attn_func on CPU torch tensors (any batch/token/head strides, dim
    stride 1); out contiguous [B, Lq, H, E]."""
    lib = load()
    b, lq, heads, hd = q.shape
    arr = [(ctypes.c_int64 * 3)(*x.stride()[:3]) for x in (q, k, v)]
    lib.oracle_flash(_ptr(q), _ptr(k), _ptr(v), _ptr(out), b, lq, k.shape[1], heads, hd, *arr,
                     _nan() if scale is None else float(scale), int(bool(causal)), _dtype_code(q), threads)
