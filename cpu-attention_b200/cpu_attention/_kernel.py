"""Loads the B200 kernel library and keeps its per-stream workspace.

Replaces the reference's loader (`cpu_attention/_kernel.py:1-220`): instead of
one Mojo extension per CPU ISA tier, TensorImpl offset calibration and a
per-thread CPU workspace, there is one sm_100a shared object,
``libca_b200.so``, whose C ABI (``include/cpu_attention_b200.h``) takes plain
device pointers, sizes and strides. ``CPU_ATTENTION_SO`` points at another
build of it. There is no CPU fallback: without the library, or without a CUDA
device, every compute call raises.

``module()`` returns the native entries with the reference's call shapes
(``decode``, ``store``, ``flash``; `_C.mojo:24-33`), so engine code written
against ``K.module().decode(K.runtime(), ...)`` (`examples/ops.py:19-31`) runs
unchanged.
"""

import ctypes
import os
import threading

import torch

DTYPES = {torch.float32: 0, torch.bfloat16: 1}  # `_kernel.py:17`
HEAD_DIMS = (32, 64, 128)  # `_kernel.py:18`
_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libca_b200.so"

# return codes and device status bits (include/cpu_attention_b200.h)
OK, EDTYPE, EHEADDIM, EPAGE, ESHAPE, ELAYOUT, ENULL, EWORKSPACE, ECUDA, EUNSUPPORTED, ESCRATCH = (
    0, -1, -2, -3, -4, -5, -6, -7, -8, -9, -10)
STATUS_LENS, STATUS_TABLE, STATUS_SLOT, STATUS_TIMEOUT = 1, 2, 4, 8

# Every exported symbol the header declares, with its ctypes signature.
_P, _I64, _I32, _F, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
_PI64 = ctypes.POINTER(ctypes.c_int64)
_I64X3 = ctypes.c_int64 * 3
SIGNATURES = {
    "ca_store": (_I32, [_P, _P, _I64, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _I32, _P, _P]),
    "ca_decode_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64, _I32, _I32]),
    "ca_decode": (_I32, [_P, _I64, _P, _P, _I64, _P, _P, _I64, _P, _P, _P, _I64, _P,
                         _I64, _I64, _I64, _I64, _I32, _F, _P, _SZ, _P]),
    "ca_decode_append": (_I32, [_P, _I64, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _P, _P, _I64, _P,
                                _I64, _I64, _I64, _I64, _I32, _F, _P, _SZ, _P]),
    "ca_decode_ex": (_I32, [_P, _I64, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _P, _P,
                            _I64, _I64, _I64, _I64, _I64, _I32, _F, _P, _SZ, _P]),
    "ca_flash_ex": (_I32, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _PI64, _PI64, _PI64, _P, _P,
                           _I64, _I64, _F, _I32, _I32, _P, _P]),
    "ca_decode_noalloc": (_I32, [_P, _I64, _P, _P, _I64, _P, _P, _I64, _P, _P, _P, _I64, _P,
                                 _I64, _I64, _I64, _I64, _I32, _F, _P]),
    "ca_flash": (_I32, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _PI64, _PI64, _PI64, _F, _I32, _I32, _P,
                        _P]),
    "ca_status": (_I32, [_P, _I32, _P]),
    "ca_set_wait_limit_ns": (None, [ctypes.c_uint64]),
    "ca_last_cuda_error": (ctypes.c_char_p, []),
    "ca_build_info": (ctypes.c_char_p, []),
}

_LOCK = threading.Lock()
_LIB = []


def library_path():
    return os.environ.get("CPU_ATTENTION_SO") or os.path.join(_DIR, LIB_NAME)


def library():
    """The loaded ``libca_b200.so`` (RuntimeError when it is not built)."""
    if _LIB:
        return _LIB[0]
    with _LOCK:
        if not _LIB:
            path = library_path()
            if not os.path.exists(path):
                raise RuntimeError("cpu_attention: the CUDA kernel library is not built; run "
                                   "`python cpu-attention_b200/build.py`")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = res, args
            _LIB.append(lib)
    return _LIB[0]


def i64x3(values):
    """Three int64 strides as the ``const int64_t[3]`` the ABI takes."""
    return _I64X3(*values)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def current_stream(device):
    """The raw cudaStream_t (as an int) of ``device``'s current stream; torch's
    raw accessor when it has one (no Stream object is built)."""
    if _raw_stream is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


class on_device:
    """Makes ``device`` current for the C calls (kernels launch on the current
    device), at no cost when it already is."""

    def __init__(self, device):
        self.index = device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


def cuda_error():
    return library().ca_last_cuda_error().decode()


# ---- per-(device, stream) workspace -----------------------------------------
# The decode kernel keeps split-merge partials and per-(sequence, head) tickets
# there, and every kernel ORs value errors into its first word. Tickets must be
# zero between calls (the kernel leaves them so), so a workspace is zero-filled
# when it is made. Calls on one stream are ordered, so they may share one.
_WS = {}
_WS_LOCK = threading.Lock()
_MIN_WS = 1 << 16


_FAST = None


def fastpath():
    """The decode host path in C++ (``cpu_attention._fastpath``, built beside
    the kernel library and linked to it), or None when it is not built or
    CPU_ATTENTION_SO selects another kernel library."""
    global _FAST
    if _FAST is None:
        _FAST = False
        if not os.environ.get("CPU_ATTENTION_SO"):
            library()  # the extension resolves the kernel library already loaded
            try:
                from . import _fastpath
                _FAST = _fastpath
            except ImportError:
                _FAST = False
    return _FAST or None


def workspace(device, stream, nbytes=0):
    """The workspace tensor of (device, stream), at least ``nbytes`` long (the
    C++ host path's registry when it is built, so both paths share one)."""
    fast = fastpath()
    if fast is not None:
        index = device.index if device.index is not None else torch.cuda.current_device()
        return fast.workspace(index, int(stream), nbytes)
    key = (device.index if device.index is not None else torch.cuda.current_device(), int(stream))
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        with _WS_LOCK:
            ws = _WS.get(key)
            if ws is None or ws.numel() < nbytes:
                size = max(nbytes, _MIN_WS, 0 if ws is None else 2 * ws.numel())
                ws = torch.zeros(size, dtype=torch.uint8, device=device)
                _WS[key] = ws
    return ws


_WS_BYTES = {}


def decode_workspace_bytes(batch, heads, head_dim, page, dtype_code, device_index):
    """ca_decode_workspace_bytes, remembered per shape (a pure function of its
    arguments and the device)."""
    key = (batch, heads, head_dim, page, dtype_code, device_index)
    n = _WS_BYTES.get(key)
    if n is None:
        n = int(library().ca_decode_workspace_bytes(*key))
        if len(_WS_BYTES) < 4096:
            _WS_BYTES[key] = n
    return n


def status(device=None, stream=None, reset=True):
    """The CA_STATUS_* bits the kernels raised on (device, stream) since the last
    reset; synchronises that stream."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    stream = torch.cuda.current_stream(device).cuda_stream if stream is None else stream
    ws = workspace(device, stream)
    rc = library().ca_status(ws.data_ptr(), int(reset), stream)
    if rc < 0:
        raise RuntimeError(f"cpu_attention: {cuda_error()}")
    return rc


_STATUS_TEXT = [
    (STATUS_LENS, ValueError, "cpu_attention: cache_seqlens exceed the page table's capacity"),
    (STATUS_SLOT, ValueError, "cpu_attention: slot_mapping points past the end of the cache"),
    (STATUS_TABLE, ValueError, "cpu_attention: page_table points past the end of the cache"),
    (STATUS_TIMEOUT, RuntimeError, "cpu_attention: a device wait timed out"),
]

CHECK = os.environ.get("CPU_ATTENTION_CHECK", "0") not in ("", "0")
"""With CPU_ATTENTION_CHECK=1 every call synchronises and raises the value errors
the device found (the reference raises them in the call); by default they are
recorded on the device and read with ``status()`` / ``raise_status()``."""


def raise_status(device=None, stream=None):
    """Raise the error for value problems the kernels found (and clear them)."""
    bits = status(device, stream, reset=True)
    for bit, exc, text in _STATUS_TEXT:
        if bits & bit:
            raise exc(text)


def runtime():
    """The reference passes a runtime-config address to every native entry
    (`_kernel.py:167-207`); this build needs none. Kept so engine code keeps its
    call shape."""
    return 0


def module():
    """The native entries: ``decode``, ``store``, ``flash`` (see `_native`)."""
    from . import _native
    library()
    return _native


__all__ = ["DTYPES", "HEAD_DIMS", "library", "module", "runtime", "workspace", "status", "raise_status",
           "CHECK"]
