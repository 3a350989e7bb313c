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


def _lse_ok(lse, shape, dev):
    return (lse is None or (isinstance(lse, torch.Tensor) and lse.dtype == torch.float32 and lse.is_cuda
                            and lse.get_device() == dev.index and tuple(lse.shape) == shape
                            and lse.is_contiguous()))


def decode(rt, q, k_cache, v_cache, k, v, slots, lens, page_table, scale, dst, lse=None):
    """Paged decode of q ``[seqs, (1,) heads, dim]`` against caches of
    ``kv_heads`` heads (``heads % kv_heads == 0``: query head h reads KV head
    ``h // (heads // kv_heads)``). With k/v (``kv_heads`` heads), each
    sequence's new token is stored first: at ``slots`` (then ``lens`` is the
    length after the store), or appended at ``lens`` (the length before). k/v
    of shape ``[seqs, n, kv_heads, dim]`` with n > 1 append n tokens at
    ``lens`` in the same launch. Writes ``dst`` when given, else a new tensor,
    and each row's log-sum-exp into ``lse`` (float32 ``[seqs, heads]``) when
    given; returns the output, or None (`_C.mojo:87-171`)."""
    del rt
    fast = K.fastpath()
    if (fast is not None and _plain_tensors(q, k_cache, v_cache, lens, page_table)
            and _plain_or_none(k, v, slots, dst, lse)):
        # the same checks and call in C++ (cpu_attention/_fastpath)
        out = fast.decode(q, k_cache, v_cache, k, v, slots, lens, page_table, None if scale is None else float(scale),
                          dst, lse)
        if out is not None and K.CHECK:
            K.raise_status(out.device, K.current_stream(out.device))
        return out
    dev = _cuda(q, k_cache, v_cache, k, v, slots, lens, page_table, dst, lse)
    if dev is None or not isinstance(q, torch.Tensor):
        return None
    nd = q.dim()
    if nd not in (3, 4) or (nd == 4 and q.shape[1] != 1):
        return None
    b, heads, hd = q.shape[0], q.shape[-2], q.shape[-1]
    dt = K.DTYPES.get(q.dtype)
    if dt is None or hd not in K.HEAD_DIMS or not _rows_ok(q, hd) or k_cache.dim() != 4:
        return None
    kvh = k_cache.shape[1]
    if kvh < 1 or heads % kvh or not _caches_ok(k_cache, v_cache, q.dtype, kvh, hd):
        return None
    page = k_cache.shape[2]
    if (page_table.dim() != 2 or page_table.dtype != torch.int32 or page_table.shape[0] != b
            or not page_table.is_contiguous()):
        return None
    if not _int_vector(lens, torch.int32, b):
        return None
    store = k is not None
    n_new = 0
    if store:
        if v is None or k.dim() != nd or v.shape != k.shape or v.stride() != k.stride():
            return None
        if k.shape[0] != b or tuple(k.shape[-2:]) != (kvh, hd) or (nd == 4 and k.shape[1] < 1):
            return None
        n_new = k.shape[1] if nd == 4 else 1
        if k.dtype != q.dtype or v.dtype != q.dtype or not _rows_ok(k, hd) or (slots is not None and n_new != 1):
            return None
    elif v is not None:
        return None
    if slots is not None and not (store and _int_vector(slots, torch.int64, b)):
        return None
    if not _lse_ok(lse, (b, heads), dev):
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
        rc = lib.ca_decode_ex(
            q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0],
            k.data_ptr() if store else None, v.data_ptr() if store else None, k.stride(0) if store else 0,
            k.stride(1) if store and nd == 4 else 0, n_new, slots.data_ptr() if slots is not None else None,
            lens.data_ptr(), page_table.data_ptr(), page_table.shape[1], out.data_ptr(),
            lse.data_ptr() if lse is not None else None, b, heads, kvh, hd, page, dt, _scale(scale), ws.data_ptr(),
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
    fast = K.fastpath()
    if fast is not None and _plain_tensors(key, value, k_cache, v_cache, slots):
        # the same checks and call in C++ (cpu_attention/_fastpath)
        done = fast.store(key, value, k_cache, v_cache, slots)
        if done is not None and K.CHECK:
            K.raise_status(key.device, K.current_stream(key.device))
        return done
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


def flash(rt, q, k, v, scale, causal, lse=None, cu_q=None, cu_k=None, max_q=None, max_k=None):
    """flash_attn_func over q ``[batch, seq, heads, dim]`` and k/v ``[batch,
    seq_k, kv_heads, dim]`` (``heads % kv_heads == 0``; dims contiguous), or,
    with ``cu_q``/``cu_k`` (int32 ``[batch + 1]`` token offsets) and the
    largest lengths ``max_q``/``max_k``, over packed q ``[total_q, heads,
    dim]`` and k/v ``[total_k, kv_heads, dim]``. Each row's log-sum-exp goes to
    ``lse`` (float32 ``[batch, heads, seq]``, or ``[heads, total_q]`` packed)
    when given. Returns the output, or None (`_C.mojo:232-316`)."""
    del rt
    var = cu_q is not None or cu_k is not None
    fast = K.fastpath()
    if (not var and lse is None and fast is not None and _plain_tensors(q, k, v)
            and (causal is True or causal is False)):
        # the same checks and call in C++ (cpu_attention/_fastpath)
        out = fast.flash(q, k, v, None if scale is None else float(scale), causal)
        if out is not None and K.CHECK:
            K.raise_status(out.device, K.current_stream(out.device))
        return out
    dev = _cuda(q, k, v, lse, cu_q, cu_k)
    if dev is None or causal is not True and causal is not False:
        return None
    nd = 3 if var else 4
    if q.dim() != nd or k.dim() != nd or v.shape != k.shape:
        return None
    heads, hd, kvh = q.shape[-2], q.shape[-1], k.shape[-2]
    dt = K.DTYPES.get(q.dtype)
    if dt is None or hd not in K.HEAD_DIMS or k.shape[-1] != hd or kvh < 1 or heads % kvh:
        return None
    if k.dtype != q.dtype or v.dtype != q.dtype or q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        return None
    if var:
        if cu_q is None or cu_k is None or max_q is None or max_k is None:
            return None
        b = cu_q.shape[0] - 1
        if b < 0 or not (_int_vector(cu_q, torch.int32, b + 1) and _int_vector(cu_k, torch.int32, b + 1)):
            return None
        sq, sk, tq, tk = int(max_q), int(max_k), q.shape[0], k.shape[0]
        if sq < 1 or sk < 1:
            return None
        strides = [(0,) + tuple(x.stride()[:2]) for x in (q, k, v)]
        lse_shape = (heads, tq)
    else:
        b, sq = q.shape[0], q.shape[1]
        sk, tq, tk = k.shape[1], 0, 0
        if sq < 1 or sk < 1 or k.shape[0] != b:
            return None
        strides = [tuple(x.stride()[:3]) for x in (q, k, v)]
        lse_shape = (b, heads, sq)
    if not _lse_ok(lse, lse_shape, dev):
        return None
    out = torch.empty(q.shape, dtype=q.dtype, device=dev)
    if b == 0 or q.numel() == 0:
        return out
    stream = K.current_stream(dev)
    arr = [K.i64x3(x) for x in strides]
    ws = K.workspace(dev, stream)
    with K.on_device(dev):
        rc = K.library().ca_flash_ex(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr() if lse is not None else None,
            b, sq, sk, heads, kvh, hd, *arr, cu_q.data_ptr() if var else None, cu_k.data_ptr() if var else None,
            tq, tk, _scale(scale), int(causal), dt, ws.data_ptr(), stream)
    if not _check_rc(rc):
        return None
    if K.CHECK:
        K.raise_status(dev, stream)
    return out
