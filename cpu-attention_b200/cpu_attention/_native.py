"""The native entries, one per op, over torch tensors: the counterpart of the
reference's Mojo extension `_C` (`_mojo/src/_C.mojo:87-316`).

Each entry checks the tensors' metadata (device, dtype, sizes, strides), picks
the launch arguments and calls the C ABI of ``libca_b200.so`` on the tensors'
device and its current stream. Like `_C`, it returns ``None`` for anything it
does not take -- a wrong shape or dtype, a layout that needs a copy, a tensor
on another device -- and the public API then raises the precise error or
copies and calls again. A CUDA failure raises RuntimeError.
"""

import torch

from . import _kernel as K


_DEVICES = {}


def _cuda(*ts):
    """The common CUDA device of the given tensors, or None. (Device indices are
    compared as ints: building a torch.device per tensor costs more than the
    rest of the host path.)"""
    idx = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            return None
        d = t.get_device()
        if idx is None:
            idx = d
        elif d != idx:
            return None
    if idx is None:
        return None
    dev = _DEVICES.get(idx)
    return dev if dev is not None else _DEVICES.setdefault(idx, torch.device("cuda", idx))


def _plain_tensors(*ts):
    return all(type(t) is torch.Tensor for t in ts)


def _plain_or_none(*ts):
    return all(t is None or type(t) is torch.Tensor for t in ts)


def _rows_ok(t, hd):
    """Heads and dims contiguous; any token stride (`_C.mojo:68-71`)."""
    return t.stride(-1) == 1 and t.stride(-2) == hd


def _caches_ok(kc, vc, dtype, heads, hd):
    """[blocks, heads, page, dim], contiguous, matching, page % 16 == 0 (`_C.mojo:74-80`)."""
    if kc.dim() != 4 or vc.shape != kc.shape:
        return False
    return (kc.dtype == dtype and vc.dtype == dtype and kc.shape[1] == heads and kc.shape[3] == hd
            and kc.shape[2] > 0 and kc.shape[2] % 16 == 0 and kc.is_contiguous() and vc.is_contiguous())


def _int_vector(t, dtype, n):
    return (isinstance(t, torch.Tensor) and t.dim() == 1 and t.dtype == dtype and t.shape[0] == n
            and t.is_contiguous())


def _check_rc(rc):
    if rc == K.ECUDA:
        raise RuntimeError(f"cpu_attention: {K.cuda_error()}")
    return rc == K.OK


def _scale(scale):
    return float("nan") if scale is None else float(scale)


def decode(rt, q, k_cache, v_cache, k, v, slots, lens, page_table, scale, dst):
    """Paged decode of q ``[seqs, (1,) heads, dim]`` (MHA). With k/v, each
    sequence's new token is stored first: at ``slots`` (then ``lens`` is the
    length after the store), or appended at ``lens`` (the length before). k/v
    of shape ``[seqs, n, heads, dim]`` with n > 1 append n tokens at ``lens``
    in the same launch (``ca_decode_append``). Writes ``dst`` when given, else a
    new tensor; returns it, or None (`_C.mojo:87-171`)."""
    del rt
    fast = K.fastpath()
    if fast is not None and _plain_tensors(q, k_cache, v_cache, lens, page_table) and _plain_or_none(k, v, slots, dst):
        # the same checks and call in C++ (cpu_attention/_fastpath)
        out = fast.decode(q, k_cache, v_cache, k, v, slots, lens, page_table, None if scale is None else float(scale),
                          dst)
        if out is not None and K.CHECK:
            K.raise_status(out.device, K.current_stream(out.device))
        return out
    dev = _cuda(q, k_cache, v_cache, k, v, slots, lens, page_table, dst)
    if dev is None or not isinstance(q, torch.Tensor):
        return None
    nd = q.dim()
    if nd not in (3, 4) or (nd == 4 and q.shape[1] != 1):
        return None
    b, heads, hd = q.shape[0], q.shape[-2], q.shape[-1]
    dt = K.DTYPES.get(q.dtype)
    if dt is None or hd not in K.HEAD_DIMS or not _rows_ok(q, hd):
        return None
    if not _caches_ok(k_cache, v_cache, q.dtype, heads, hd):
        return None
    page = k_cache.shape[2]
    if (page_table.dim() != 2 or page_table.dtype != torch.int32 or page_table.shape[0] != b
            or not page_table.is_contiguous()):
        return None
    if not _int_vector(lens, torch.int32, b):
        return None
    store = k is not None
    n_new = 1
    if store:
        multi = (nd == 4 and slots is None and k.dim() == 4 and k.shape[0] == b and k.shape[1] > 1
                 and tuple(k.shape[2:]) == (heads, hd))
        if v is None or (k.shape != q.shape and not multi) or v.shape != k.shape or v.stride() != k.stride():
            return None
        if k.dtype != q.dtype or v.dtype != q.dtype or not _rows_ok(k, hd):
            return None
        if multi:
            n_new = k.shape[1]
    elif v is not None:
        return None
    if slots is not None and not (store and _int_vector(slots, torch.int64, b)):
        return None
    if dst is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=dev)
    else:
        out = dst
        if out.shape != q.shape or out.dtype != q.dtype or not out.is_contiguous():
            return None
    if b == 0:
        return out
    lib = K.library()
    stream = K.current_stream(dev)
    need = K.decode_workspace_bytes(b, heads, hd, page, dt, dev.index)
    if need == 0:
        return None
    ws = K.workspace(dev, stream, need)
    with K.on_device(dev):
        if n_new > 1:
            rc = lib.ca_decode_append(
                q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
                k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), n_new, lens.data_ptr(),
                page_table.data_ptr(), page_table.shape[1], out.data_ptr(), b, heads, hd, page, dt,
                _scale(scale), ws.data_ptr(), ws.numel(), stream)
        else:
            rc = lib.ca_decode(
                q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
                k.data_ptr() if store else None, v.data_ptr() if store else None, k.stride(0) if store else 0,
                slots.data_ptr() if slots is not None else None, lens.data_ptr(), page_table.data_ptr(),
                page_table.shape[1], out.data_ptr(), b, heads, hd, page, dt, _scale(scale), ws.data_ptr(),
                ws.numel(), stream)
    if not _check_rc(rc):
        return None
    if K.CHECK:
        K.raise_status(dev, stream)
    return out


def store(rt, key, value, k_cache, v_cache, slots):
    """``reshape_and_cache``: token i of key/value ``[tokens, heads, dim]`` goes
    to slot ``slots[i]`` (int64; negative skips it). True, or None
    (`_C.mojo:174-213`)."""
    del rt
    dev = _cuda(key, value, k_cache, v_cache, slots)
    if dev is None or key.dim() != 3 or value.dim() != 3:
        return None
    n, heads, hd = key.shape
    dt = K.DTYPES.get(key.dtype)
    if dt is None or hd not in K.HEAD_DIMS or value.dtype != key.dtype or not _rows_ok(key, hd):
        return None
    if value.shape != key.shape or value.stride() != key.stride():
        return None
    if not _caches_ok(k_cache, v_cache, key.dtype, heads, hd) or not _int_vector(slots, torch.int64, n):
        return None
    if n == 0:
        return True
    stream = K.current_stream(dev)
    ws = K.workspace(dev, stream)
    with K.on_device(dev):
        rc = K.library().ca_store(key.data_ptr(), value.data_ptr(), key.stride(0), k_cache.data_ptr(),
                                  v_cache.data_ptr(), k_cache.shape[0], slots.data_ptr(), n, heads, hd,
                                  k_cache.shape[2], dt, ws.data_ptr(), stream)
    if not _check_rc(rc):
        return None
    if K.CHECK:
        K.raise_status(dev, stream)
    return True


def flash(rt, q, k, v, scale, causal):
    """flash_attn_func over q/k/v ``[batch, seq, heads, dim]`` (MHA, dims
    contiguous). Returns the output, or None (`_C.mojo:232-316`)."""
    del rt
    fast = K.fastpath()
    if fast is not None and _plain_tensors(q, k, v) and (causal is True or causal is False):
        # the same checks and call in C++ (cpu_attention/_fastpath)
        out = fast.flash(q, k, v, None if scale is None else float(scale), causal)
        if out is not None and K.CHECK:
            K.raise_status(out.device, K.current_stream(out.device))
        return out
    dev = _cuda(q, k, v)
    if dev is None or q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        return None
    b, sq, heads, hd = q.shape
    sk = k.shape[1]
    dt = K.DTYPES.get(q.dtype)
    if dt is None or hd not in K.HEAD_DIMS or sq < 1 or sk < 1:
        return None
    if k.shape[0] != b or k.shape[2] != heads or k.shape[3] != hd or k.dtype != q.dtype or v.dtype != q.dtype:
        return None
    if v.shape != k.shape or q.stride(3) != 1 or k.stride(3) != 1 or v.stride(3) != 1:
        return None
    if causal is not True and causal is not False:
        return None
    out = torch.empty((b, sq, heads, hd), dtype=q.dtype, device=dev)
    if b == 0:
        return out
    stream = K.current_stream(dev)
    arr = (K.i64x3(q.stride()[:3]), K.i64x3(k.stride()[:3]), K.i64x3(v.stride()[:3]))
    ws = K.workspace(dev, stream)
    with K.on_device(dev):
        rc = K.library().ca_flash(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, sq, sk, heads, hd,
                                  *arr, _scale(scale), int(causal), dt, ws.data_ptr(), stream)
    if not _check_rc(rc):
        return None
    return out
