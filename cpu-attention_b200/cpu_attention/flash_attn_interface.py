"""flash-attn's interface over the B200 kernels.

Same names, arguments, defaults and error behaviour as the reference's
`cpu_attention/flash_attn_interface.py:1-227`: what the kernel cannot do raises
``NotImplementedError`` instead of being silently ignored, each call goes
straight to the native entry (`_native`), and only when that declines does
Python look again -- to raise the precise error, or to copy a layout (or move an
index tensor to the device) the kernel cannot read in place, and call again.

Tensors are CUDA tensors: q, the caches and new k/v live on one B200, and so
does the output. Index tensors (cache_seqlens, page_table, cache_batch_idx) may
be given on the CPU; they are then validated on the host, as the reference
does, and copied to the device.
"""

import torch

from . import _kernel as K
from . import _native
from .cache import reshape_and_cache

_MHA_ONLY = "cpu_attention supports MHA only (nheads == nheads_k); GQA/MQA are not supported yet"


def _plain(x):
    """A tensor subclass as a plain tensor."""
    plain = type(x) in (torch.Tensor, torch.nn.Parameter) or not isinstance(x, torch.Tensor)
    return x if plain else x.as_subclass(torch.Tensor)


def _rows(x):
    """``x`` with heads and dims contiguous (any token stride is read in place)."""
    return x if x.stride(-1) == 1 and x.stride(-2) == x.shape[-1] else x.contiguous()


def _on(x, device):
    return x if x is None or x.device == device else x.to(device, non_blocking=True)


def flash_attn_with_kvcache(
    q,
    k_cache,
    v_cache,
    k=None,
    v=None,
    qv=None,
    rotary_cos=None,
    rotary_sin=None,
    cache_seqlens=None,
    cache_batch_idx=None,
    cache_leftpad=None,
    page_table=None,
    cu_seqlens_q=None,
    cu_seqlens_k_new=None,
    max_seqlen_q=None,
    rotary_seqlens=None,
    q_descale=None,
    k_descale=None,
    v_descale=None,
    softmax_scale=None,
    causal=False,
    window_size=(-1, -1),
    attention_chunk=0,
    softcap=0.0,
    rotary_interleaved=True,
    scheduler_metadata=None,
    num_splits=0,
    pack_gqa=None,
    sm_margin=0,
    return_softmax_lse=False,
    block_table=None,
    alibi_slopes=None,
):
    """Paged decode: one query token per sequence against its cached K/V.

    flash-attn's arguments (`flash_attn_interface.py:37-127` of the reference);
    ``qv``, ``rotary_*``, ``cache_leftpad``, ``cu_seqlens_*``, ``max_seqlen_q``,
    ``*_descale``, ``window_size``, ``softcap``, ``attention_chunk``, ``alibi_slopes``
    and ``return_softmax_lse`` raise ``NotImplementedError``; the tuning hints are
    ignored. Differences from flash-attn:

    * ``q`` is ``[batch, 1, nheads, headdim]``, MHA (``nheads_k == nheads``).
    * The cache is head-major ``[num_blocks, nheads, page_block_size, headdim]``
      (K stored transposed inside the page), contiguous, and written only by
      this library: ``reshape_and_cache``, or ``k``/``v`` here -- any number of
      new tokens, appended at ``cache_seqlens`` (the length before the write).
    * ``causal`` has no effect: the query sits at the last cached position.
    * ``block_table`` (flash-attn 2's name for ``page_table``) is accepted.
    """
    if (qv is not None or rotary_cos is not None or rotary_sin is not None
            or cache_leftpad is not None or cu_seqlens_q is not None
            or cu_seqlens_k_new is not None or max_seqlen_q is not None
            or rotary_seqlens is not None or q_descale is not None
            or k_descale is not None or v_descale is not None
            or window_size != (-1, -1) or softcap or attention_chunk or return_softmax_lse
            or alibi_slopes is not None):
        raise NotImplementedError(
            "cpu_attention: qv, rotary, cache_leftpad, varlen, descale, sliding "
            "windows, softcap, attention_chunk, alibi and return_softmax_lse are not supported")
    if block_table is not None:
        if page_table is not None:
            raise ValueError("cpu_attention: pass `page_table` or `block_table`, not both")
        page_table = block_table
    if page_table is None:
        raise ValueError("cpu_attention: pass `page_table`")
    if cache_batch_idx is not None:
        page_table = page_table.index_select(0, cache_batch_idx.to(page_table.device).long())
    if not isinstance(cache_seqlens, torch.Tensor):
        if cache_seqlens is None:
            raise ValueError("cpu_attention: `cache_seqlens` is required")
        cache_seqlens = torch.full((q.shape[0],), cache_seqlens, dtype=torch.int32, device=q.device)
    if k is not None and k.shape[1] != 1:
        # Several new tokens (a prompt): appended at cache_seqlens + j by the
        # decode launch itself; when that is declined, the reference's two
        # steps (`flash_attn_interface.py:109-117`): store them at
        # cache_seqlens + j, then decode over the grown cache.
        if cache_seqlens.device == k_cache.device and page_table.device == k_cache.device:
            out = _native.decode(0, q, k_cache, v_cache, k, v, None, cache_seqlens, page_table, softmax_scale, None)
            if out is not None:
                return out
        n, page = k.shape[1], k_cache.shape[2]
        dev = k_cache.device
        lens = cache_seqlens.to(dev)
        pos = lens.long()[:, None] + torch.arange(n, device=dev)[None]
        slots = page_table.to(dev).long().gather(1, pos // page) * page + pos % page
        reshape_and_cache(k.reshape(-1, *k.shape[2:]), v.reshape(-1, *v.shape[2:]),
                          k_cache, v_cache, slots.flatten())
        cache_seqlens, k, v = lens + n, None, None
    out = _native.decode(0, q, k_cache, v_cache, k, v, None, cache_seqlens, page_table, softmax_scale, None)
    if out is None:
        q, k_cache, v_cache, k, v, page_table, cache_seqlens = _check_kvcache(
            q, k_cache, v_cache, k, v, page_table, cache_seqlens)
        out = _native.decode(0, q, k_cache, v_cache, k, v, None, cache_seqlens, page_table, softmax_scale, None)
        if out is None:
            raise RuntimeError("cpu_attention: the kernel declined arguments that passed validation")
    return out


def _check_kvcache(q, k_cache, v_cache, k, v, page_table, lens):
    """Raise the precise error for a call the kernel declined, or return its
    tensors with layouts (and devices) it reads in place
    (`flash_attn_interface.py:162-197` of the reference)."""
    q, k_cache, v_cache, k, v, page_table, lens = map(_plain, (q, k_cache, v_cache, k, v, page_table, lens))
    if q.dim() != 4:
        raise ValueError("cpu_attention: q must be [batch, 1, nheads, headdim]")
    if q.shape[1] != 1:
        raise NotImplementedError("cpu_attention decodes one query token per sequence")
    batch, _, heads, hd = q.shape
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("cpu_attention: k_cache/v_cache must be "
                         "[num_blocks, nheads, page_block_size, headdim] and match")
    if k_cache.shape[3] != hd or heads % k_cache.shape[1]:
        raise ValueError("cpu_attention: q and the caches disagree on heads or head_dim")
    if k_cache.shape[1] != heads:
        raise NotImplementedError(_MHA_ONLY)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("cpu_attention: the paged caches must be contiguous")
    if q.dtype not in K.DTYPES or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise ValueError("cpu_attention: q and the caches must share a dtype (fp32 or bf16)")
    if hd not in K.HEAD_DIMS or k_cache.shape[2] % 16:
        raise ValueError(f"cpu_attention: head_dim must be 32/64/128 (got {hd}) and the "
                         f"page a multiple of 16 (got {k_cache.shape[2]})")
    if page_table.dtype != torch.int32 or page_table.dim() != 2 or page_table.shape[0] != batch:
        raise ValueError("cpu_attention: page_table must be int32 [batch, max_blocks]")
    if lens.dtype != torch.int32 or lens.shape != (batch,):
        raise ValueError("cpu_attention: cache_seqlens must be an int or an int32 [batch] tensor")
    if (k is None) != (v is None) or k is not None and (
            k.shape != (batch, 1, heads, hd) or v.shape != k.shape
            or k.dtype != q.dtype or v.dtype != q.dtype):
        raise ValueError("cpu_attention: k/v must both be [batch, seqlen_new, nheads, headdim]")
    if batch and int(lens.max()) + (k is not None) > page_table.shape[1] * k_cache.shape[2]:
        raise ValueError("cpu_attention: cache_seqlens exceed the page table's capacity")
    dev = q.device
    if dev.type != "cuda" or any(t.device != dev for t in (k_cache, v_cache) + ((k, v) if k is not None else ())):
        raise ValueError("cpu_attention: q, the caches and k/v must be CUDA tensors on one device "
                         f"(q is on {dev})")
    if k is not None:
        k, v = (k, v) if _rows(k) is k and v.stride() == k.stride() else (k.contiguous(), v.contiguous())
    return (_rows(q), k_cache, v_cache, k, v, _on(page_table.contiguous(), dev), _on(lens.contiguous(), dev))


def flash_attn_func(q, k, v, softmax_scale=None, causal=False):
    """Dense attention over whole sequences, flash-attn's ``flash_attn_func``.

    q/k/v are ``[batch, seqlen, nheads, headdim]`` CUDA tensors (MHA; GQA/MQA
    raise ``NotImplementedError``). ``causal`` is bottom-right aligned (query
    ``i`` sees keys ``j <= i + seqlen_k - seqlen_q``); a row that sees no key is
    zero. ``softmax_scale`` defaults to ``1 / sqrt(headdim)``. Inference only
    (`flash_attn_interface.py:200-215` of the reference).
    """
    out = _native.flash(0, q, k, v, softmax_scale, causal)
    if out is None:
        q, k, v = _check_flash(q, k, v)
        out = _native.flash(0, q, k, v, softmax_scale, bool(causal))
        if out is None:
            raise RuntimeError("cpu_attention: the kernel declined arguments that passed validation")
    return out


def _check_flash(q, k, v):
    """Raise the precise error for a call the kernel declined, or return q/k/v
    with the head dim contiguous (`flash_attn_interface.py:228-244` of the
    reference)."""
    q, k, v = map(_plain, (q, k, v))
    if q.dim() != 4 or k.dim() != 4 or v.shape != k.shape:
        raise ValueError("cpu_attention: q/k/v must be [batch, seqlen, nheads, headdim]")
    batch, seq_q, heads, hd = q.shape
    if (k.shape[0] != batch or k.shape[3] != hd or heads % k.shape[2]
            or seq_q < 1 or k.shape[1] < 1):
        raise ValueError("cpu_attention: k/v must be [batch, seqlen_k, nheads, headdim] matching q")
    if k.shape[2] != heads:
        raise NotImplementedError(_MHA_ONLY)
    if q.dtype not in K.DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("cpu_attention: q/k/v must share a dtype (fp32 or bf16)")
    if hd not in K.HEAD_DIMS:
        raise ValueError(f"cpu_attention: head_dim must be 32, 64 or 128 (got {hd})")
    dev = q.device
    if dev.type != "cuda" or k.device != dev or v.device != dev:
        raise ValueError(f"cpu_attention: q/k/v must be CUDA tensors on one device (q is on {dev})")
    return tuple(x if x.stride(3) == 1 else x.contiguous() for x in (q, k, v))


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                           max_seqlen_k, softmax_scale=None, causal=False):
    """Not ported: use padded q/k/v with ``flash_attn_func``, or the paged cache."""
    raise NotImplementedError("cpu_attention: variable-length attention is not ported")


def flash_attn_qkvpacked_func(qkv, *args, **kwargs):
    """Not ported (pass q/k/v views of the packed tensor to ``flash_attn_func``)."""
    raise NotImplementedError("cpu_attention: packed attention is not ported")


flash_attn_kvpacked_func = flash_attn_varlen_qkvpacked_func = \
    flash_attn_varlen_kvpacked_func = flash_attn_qkvpacked_func
