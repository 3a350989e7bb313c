"""flash-attn's entry points on the B200 kernels.

Names, parameters, defaults and exception texts are the reference's
(`cpu_attention/flash_attn_interface.py`), so code written for it runs
unchanged. Beyond the reference, this build attends grouped heads (GQA/MQA:
``nheads_k`` divides ``nheads``), returns the softmax log-sum-exp
(``return_softmax_lse`` here, ``return_attn_probs`` for prefill) and runs
``flash_attn_varlen_func``.

A call goes to the native entry (``_native``) with its arguments as given. The
native entry answers None when it cannot use them; only then does this module
look at them: a real mistake raises the reference's exception, anything else
is brought into a form the kernels read in place (rows made contiguous, index
tensors moved to the device) and sent once more. Data tensors are CUDA
tensors; index tensors may also be given on the host.
"""

import torch

from . import _kernel as K
from . import _native
from .cache import reshape_and_cache

# flash_attn_with_kvcache options no kernel here implements; setting one raises
_NOT_SUPPORTED = ("cpu_attention: qv, rotary, cache_leftpad, varlen, descale, sliding windows, softcap, "
                  "attention_chunk and alibi are not supported")


def _as_tensor(x):
    """A tensor subclass (e.g. a Parameter wrapper) viewed as a plain tensor."""
    if isinstance(x, torch.Tensor) and type(x) not in (torch.Tensor, torch.nn.Parameter):
        return x.as_subclass(torch.Tensor)
    return x


def _readable_rows(x):
    """``x``, or a copy of it, with heads and dims packed (the token stride is free)."""
    return x if x.stride(-1) == 1 and x.stride(-2) == x.shape[-1] else x.contiguous()


def _to(x, device):
    return x if x is None or x.device == device else x.to(device, non_blocking=True)


def _options_set(opts):
    """Names of the options given a value other than their inert default."""
    named = []
    for name, value in opts.items():
        if name == "window_size":
            active = tuple(value) != (-1, -1)
        elif isinstance(value, (int, float)):
            active = value != 0
        else:
            active = value is not None
        if active:
            named.append(name)
    return named


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
    """One query token per sequence attending its paged K/V cache.

    ``q`` is ``[batch, 1, nheads, headdim]``; the caches are
    ``[num_blocks, nheads_k, page_block_size, headdim]`` (contiguous, K stored
    transposed inside each page, so only this library writes them:
    ``reshape_and_cache``, or ``k``/``v`` here), with ``nheads_k`` dividing
    ``nheads``. ``k``/``v`` (``[batch, seqlen_new, nheads_k, headdim]``) are
    appended at ``cache_seqlens`` -- the lengths before the call -- and
    attended with the rest. ``page_table`` (or flash-attn 2's
    ``block_table``) maps each sequence's pages to blocks; ``cache_batch_idx``
    picks its rows. ``return_softmax_lse`` adds the float32
    ``[batch, nheads, 1]`` log-sum-exp of each row to the result. The query
    sits at the last cached position, so ``causal`` changes nothing; the
    scheduling hints (``num_splits``, ``pack_gqa``, ...) are not needed. The
    other flash-attn options raise ``NotImplementedError``.
    """
    # (every option at its default: the common case, decided without building
    # the option table -- an engine calls this once per layer and token)
    if not (qv is None and rotary_cos is None and rotary_sin is None and cache_leftpad is None
            and cu_seqlens_q is None and cu_seqlens_k_new is None and max_seqlen_q is None
            and rotary_seqlens is None and q_descale is None and k_descale is None and v_descale is None
            and alibi_slopes is None and not attention_chunk and not softcap and window_size == (-1, -1)) \
            and _options_set(dict(qv=qv, rotary_cos=rotary_cos, rotary_sin=rotary_sin, cache_leftpad=cache_leftpad,
                                  cu_seqlens_q=cu_seqlens_q, cu_seqlens_k_new=cu_seqlens_k_new,
                                  max_seqlen_q=max_seqlen_q, rotary_seqlens=rotary_seqlens, q_descale=q_descale,
                                  k_descale=k_descale, v_descale=v_descale, window_size=window_size,
                                  softcap=softcap, attention_chunk=attention_chunk, alibi_slopes=alibi_slopes)):
        raise NotImplementedError(_NOT_SUPPORTED)
    if block_table is not None and page_table is not None:
        raise ValueError("cpu_attention: pass `page_table` or `block_table`, not both")
    table = page_table if block_table is None else block_table
    if table is None:
        raise ValueError("cpu_attention: pass `page_table`")
    if cache_batch_idx is not None:
        table = table.index_select(0, cache_batch_idx.to(table.device).long())
    lens = cache_seqlens
    if not isinstance(lens, torch.Tensor):
        if lens is None:
            raise ValueError("cpu_attention: `cache_seqlens` is required")
        lens = torch.full((q.shape[0],), int(lens), dtype=torch.int32, device=q.device)
    lse = None
    if return_softmax_lse and q.dim() == 4:
        lse = torch.empty((q.shape[0], q.shape[2]), dtype=torch.float32, device=q.device)

    def finish(out):
        return (out, lse.unsqueeze(-1)) if return_softmax_lse else out

    if k is not None and k.shape[1] > 1:
        # a prompt of several new tokens: the decode launch appends them itself
        # when it can read everything in place
        on_dev = lens.device == k_cache.device and table.device == k_cache.device
        out = _native.decode(0, q, k_cache, v_cache, k, v, None, lens, table, softmax_scale, None, lse) \
            if on_dev else None
        if out is not None:
            return finish(out)
        # else: the tokens go in first (`reshape_and_cache` at cache_seqlens + j,
        # the reference's own route), then one decode over the grown cache
        dev = k_cache.device
        count, page = k.shape[1], k_cache.shape[2]
        before = lens.to(dev).long()
        pos = before[:, None] + torch.arange(count, device=dev)[None]
        slot = table.to(dev).long().gather(1, pos // page) * page + pos % page
        reshape_and_cache(k.flatten(0, 1), v.flatten(0, 1), k_cache, v_cache, slot.flatten())
        lens, k, v = (before + count).to(torch.int32), None, None
    out = _native.decode(0, q, k_cache, v_cache, k, v, None, lens, table, softmax_scale, None, lse)
    if out is None:
        q, k_cache, v_cache, k, v, table, lens = _explain_decode(q, k_cache, v_cache, k, v, table, lens)
        out = _native.decode(0, q, k_cache, v_cache, k, v, None, lens, table, softmax_scale, None, lse)
        if out is None:
            raise RuntimeError("cpu_attention: the kernel declined arguments that passed validation")
    return finish(out)


def _explain_decode(q, k_cache, v_cache, k, v, table, lens):
    """Called when the decode entry declined: raise the reference's error for a
    bad argument, else return the tensors in layouts (and on the device) the
    kernel reads."""
    q, k_cache, v_cache, k, v, table, lens = (_as_tensor(x) for x in (q, k_cache, v_cache, k, v, table, lens))
    if q.dim() != 4:
        raise ValueError("cpu_attention: q must be [batch, 1, nheads, headdim]")
    if q.shape[1] != 1:
        raise NotImplementedError("cpu_attention decodes one query token per sequence")
    batch, _, heads, hd = q.shape
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("cpu_attention: k_cache/v_cache must be "
                         "[num_blocks, nheads, page_block_size, headdim] and match")
    kv_heads = k_cache.shape[1]
    if k_cache.shape[3] != hd or kv_heads < 1 or heads % kv_heads:
        raise ValueError("cpu_attention: q and the caches disagree on heads or head_dim")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("cpu_attention: the paged caches must be contiguous")
    if q.dtype not in K.DTYPES or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise ValueError("cpu_attention: q and the caches must share a dtype (fp32 or bf16)")
    if hd not in K.HEAD_DIMS or k_cache.shape[2] % 16:
        raise ValueError(f"cpu_attention: head_dim must be 32/64/128 (got {hd}) and the "
                         f"page a multiple of 16 (got {k_cache.shape[2]})")
    if table.dtype != torch.int32 or table.dim() != 2 or table.shape[0] != batch:
        raise ValueError("cpu_attention: page_table must be int32 [batch, max_blocks]")
    if lens.dtype != torch.int32 or tuple(lens.shape) != (batch,):
        raise ValueError("cpu_attention: cache_seqlens must be an int or an int32 [batch] tensor")
    new = k is not None
    if new != (v is not None) or new and (tuple(k.shape) != (batch, 1, kv_heads, hd) or v.shape != k.shape
                                          or k.dtype != q.dtype or v.dtype != q.dtype):
        raise ValueError("cpu_attention: k/v must both be [batch, seqlen_new, nheads, headdim]")
    if batch and int(lens.max()) + int(new) > table.shape[1] * k_cache.shape[2]:
        raise ValueError("cpu_attention: cache_seqlens exceed the page table's capacity")
    dev = q.device
    if dev.type != "cuda" or any(t.device != dev for t in (k_cache, v_cache) + ((k, v) if new else ())):
        raise ValueError("cpu_attention: q, the caches and k/v must be CUDA tensors on one device "
                         f"(q is on {dev})")
    if new and not (_readable_rows(k) is k and v.stride() == k.stride()):
        k, v = k.contiguous(), v.contiguous()
    return (_readable_rows(q), k_cache, v_cache, k, v, _to(table.contiguous(), dev), _to(lens.contiguous(), dev))


def flash_attn_func(q, k, v, softmax_scale=None, causal=False, *, return_attn_probs=False):
    """Attention over whole sequences (prefill), flash-attn's ``flash_attn_func``.

    q ``[batch, seqlen_q, nheads, headdim]``, k/v ``[batch, seqlen_k, nheads_k,
    headdim]`` with ``nheads_k`` dividing ``nheads``; any batch, token and head
    strides (chunks of a fused projection are read in place). ``causal`` aligns
    the mask bottom-right: query ``i`` sees keys ``j <= i + seqlen_k -
    seqlen_q``, and a row that sees no key is zero. ``softmax_scale`` defaults
    to ``headdim ** -0.5``. ``return_attn_probs`` (flash-attn 3's name) also
    returns the float32 ``[batch, nheads, seqlen_q]`` softmax log-sum-exp.
    Inference only: no dropout, window, softcap or alibi.
    """
    lse = None
    if return_attn_probs and q.dim() == 4:
        lse = torch.empty((q.shape[0], q.shape[2], q.shape[1]), dtype=torch.float32, device=q.device)
    out = _native.flash(0, q, k, v, softmax_scale, causal, lse)
    if out is None:
        q, k, v = _explain_flash(q, k, v)
        out = _native.flash(0, q, k, v, softmax_scale, bool(causal), lse)
        if out is None:
            raise RuntimeError("cpu_attention: the kernel declined arguments that passed validation")
    return (out, lse) if return_attn_probs else out


def _explain_flash(q, k, v):
    """Called when the prefill entry declined: raise the reference's error for
    a bad argument, else return q/k/v with the head dim packed."""
    q, k, v = (_as_tensor(x) for x in (q, k, v))
    if q.dim() != 4 or k.dim() != 4 or v.shape != k.shape:
        raise ValueError("cpu_attention: q/k/v must be [batch, seqlen, nheads, headdim]")
    batch, seq_q, heads, hd = q.shape
    if (k.shape[0] != batch or k.shape[3] != hd or k.shape[2] < 1 or heads % k.shape[2]
            or seq_q < 1 or k.shape[1] < 1):
        raise ValueError("cpu_attention: k/v must be [batch, seqlen_k, nheads, headdim] matching q")
    _check_dtypes_and_device(q, k, v, hd)
    return tuple(x if x.stride(-1) == 1 else x.contiguous() for x in (q, k, v))


def _check_dtypes_and_device(q, k, v, hd):
    if q.dtype not in K.DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("cpu_attention: q/k/v must share a dtype (fp32 or bf16)")
    if hd not in K.HEAD_DIMS:
        raise ValueError(f"cpu_attention: head_dim must be 32, 64 or 128 (got {hd})")
    dev = q.device
    if dev.type != "cuda" or k.device != dev or v.device != dev:
        raise ValueError(f"cpu_attention: q/k/v must be CUDA tensors on one device (q is on {dev})")


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, softmax_scale=None,
                           causal=False, *, return_attn_probs=False):
    """``flash_attn_func`` over sequences of different lengths packed end to end.

    q is ``[total_q, nheads, headdim]`` and k/v ``[total_k, nheads_k, headdim]``;
    sequence ``b`` owns query tokens ``cu_seqlens_q[b]:cu_seqlens_q[b + 1]`` and
    key tokens ``cu_seqlens_k[b]:cu_seqlens_k[b + 1]`` (int32 ``[batch + 1]``,
    starting at 0). ``max_seqlen_q``/``max_seqlen_k`` bound the lengths. The
    causal mask is bottom-right within each sequence. Returns ``[total_q,
    nheads, headdim]``, and with ``return_attn_probs`` also the float32
    ``[nheads, total_q]`` log-sum-exp.
    """
    lse = None
    if return_attn_probs and q.dim() == 3:
        lse = torch.empty((q.shape[1], q.shape[0]), dtype=torch.float32, device=q.device)
    out = _native.flash(0, q, k, v, softmax_scale, causal, lse, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                        max_seqlen_k)
    if out is None:
        q, k, v, cu_seqlens_q, cu_seqlens_k = _explain_varlen(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                                              max_seqlen_k)
        out = _native.flash(0, q, k, v, softmax_scale, bool(causal), lse, cu_seqlens_q, cu_seqlens_k,
                            int(max_seqlen_q), int(max_seqlen_k))
        if out is None:
            raise RuntimeError("cpu_attention: the kernel declined arguments that passed validation")
    return (out, lse) if return_attn_probs else out


def _explain_varlen(q, k, v, cu_q, cu_k, max_q, max_k):
    """Called when the varlen prefill entry declined: raise for a bad argument,
    else return the tensors packed and the offsets on q's device. Offsets given
    on the host are checked in full (monotone, within the token counts and the
    stated maxima); on the device only their shape and dtype are."""
    q, k, v = (_as_tensor(x) for x in (q, k, v))
    if q.dim() != 3 or k.dim() != 3 or v.shape != k.shape:
        raise ValueError("cpu_attention: varlen q/k/v must be [total_tokens, nheads, headdim]")
    heads, hd = q.shape[1], q.shape[2]
    if k.shape[2] != hd or k.shape[1] < 1 or heads % k.shape[1]:
        raise ValueError("cpu_attention: k/v must be [total_k, nheads_k, headdim] with nheads_k dividing nheads")
    _check_dtypes_and_device(q, k, v, hd)
    offsets = []
    for name, cu, total, most in (("cu_seqlens_q", cu_q, q.shape[0], max_q), ("cu_seqlens_k", cu_k, k.shape[0],
                                                                              max_k)):
        if not isinstance(cu, torch.Tensor) or cu.dtype != torch.int32 or cu.dim() != 1 or cu.shape[0] < 1:
            raise ValueError(f"cpu_attention: {name} must be an int32 [batch + 1] tensor")
        if most is None or int(most) < 1:
            raise ValueError("cpu_attention: max_seqlen_q/max_seqlen_k must be positive")
        if cu.device.type == "cpu":
            lengths = cu[1:] - cu[:-1]
            if int(cu[0]) != 0 or bool((lengths < 0).any()) or int(cu[-1]) > total or \
                    (lengths.numel() and int(lengths.max()) > int(most)):
                raise ValueError(f"cpu_attention: {name} must rise from 0 to at most the token count, "
                                 "no sequence longer than its max_seqlen")
        offsets.append(_to(cu.contiguous(), q.device))
    if offsets[0].shape != offsets[1].shape:
        raise ValueError("cpu_attention: cu_seqlens_q and cu_seqlens_k must have the same length")
    q, k, v = (x if x.stride(-1) == 1 else x.contiguous() for x in (q, k, v))
    return q, k, v, offsets[0], offsets[1]


def flash_attn_qkvpacked_func(qkv, *args, **kwargs):
    """Not ported (pass q/k/v views of the packed tensor to ``flash_attn_func``)."""
    raise NotImplementedError("cpu_attention: packed attention is not ported")


flash_attn_kvpacked_func = flash_attn_varlen_qkvpacked_func = \
    flash_attn_varlen_kvpacked_func = flash_attn_qkvpacked_func
