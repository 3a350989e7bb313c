"""Writing tokens into the paged KV cache: ``reshape_and_cache``.

The cache layout belongs to this library (head-major pages with K stored
transposed inside each page, the reference's x86 layout), so tokens reach it
only through this function (vLLM's signature, the reference's
`cpu_attention/cache.py`) or through ``flash_attn_with_kvcache(k=..., v=...)``.
"""

import torch

from . import _kernel as K
from . import _native


def reshape_and_cache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """Writes the K/V rows of ``num_tokens`` tokens into their cache slots.

    ``key`` and ``value`` are ``[num_tokens, nheads_k, headdim]`` with heads and
    dims packed; the token stride is free (a chunk of a fused projection needs
    no copy). The caches are ``[num_blocks, nheads_k, page_block_size,
    headdim]``. ``slot_mapping`` (int64 ``[num_tokens]``) gives each token's
    slot, ``block * page_block_size + position``; a negative slot leaves the
    token out (padding). The write is bit-exact: the cache holds the given
    values in its own layout.
    """
    if _native.store(0, key, value, k_cache, v_cache, slot_mapping) is not None:
        return
    key, value, slot_mapping = _explain_store(key, value, k_cache, v_cache, slot_mapping)
    if _native.store(0, key, value, k_cache, v_cache, slot_mapping) is None:
        raise RuntimeError("cpu_attention: the kernel declined arguments that passed validation")


def _explain_store(key, value, k_cache, v_cache, slots):
    """Called when the store entry declined: raise the reference's error for a
    bad argument, else return key/value with packed rows and the slots
    contiguous on the cache's device."""
    key, value, slots = (x.as_subclass(torch.Tensor) if isinstance(x, torch.Tensor)
                         and type(x) not in (torch.Tensor, torch.nn.Parameter) else x for x in (key, value, slots))
    if key.dim() != 3 or value.shape != key.shape:
        raise ValueError("cpu_attention: key/value must both be [num_tokens, nheads, headdim]")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("cpu_attention: k_cache/v_cache must be "
                         "[num_blocks, nheads, page_block_size, headdim] and match")
    tokens, heads, hd = key.shape
    blocks, cache_heads, page, cache_hd = k_cache.shape
    if (heads, hd) != (cache_heads, cache_hd):
        raise ValueError("cpu_attention: key/value heads or head_dim do not match the cache")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("cpu_attention: the paged caches must be contiguous")
    if key.dtype not in K.DTYPES or any(t.dtype != key.dtype for t in (value, k_cache, v_cache)):
        raise ValueError("cpu_attention: key/value and the caches must share a dtype (fp32 or bf16)")
    if hd not in K.HEAD_DIMS or page % 16:
        raise ValueError("cpu_attention: head_dim must be 32/64/128 and the page a multiple of 16")
    if slots.dtype != torch.int64 or tuple(slots.shape) != (tokens,):
        raise ValueError("cpu_attention: slot_mapping must be int64 [num_tokens]")
    if tokens and int(slots.max()) >= blocks * page:
        raise ValueError("cpu_attention: slot_mapping points past the end of the cache")
    dev = k_cache.device
    if dev.type != "cuda" or any(t.device != dev for t in (key, value, v_cache)):
        raise ValueError("cpu_attention: key/value and the caches must be CUDA tensors on one device "
                         f"(the cache is on {dev})")
    if key.stride(-1) != 1 or key.stride(-2) != hd or value.stride() != key.stride():
        key, value = key.contiguous(), value.contiguous()
    slots = slots.contiguous()
    return key, value, slots if slots.device == dev else slots.to(dev, non_blocking=True)
