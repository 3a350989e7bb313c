"""TEST INFRASTRUCTURE ONLY. The reference's paged KV-cache layout, restated in
numpy for bit-exact checks of the B200 store kernel.

Follows ``PageLayout`` (``cpu_attention/_mojo/src/paged_attn.mojo:58-131``, the
x86 layout) and ``_store_kv`` (``:151-176``) of ducviet00/cpu-attention. The
cache is ``[num_blocks, heads, page, head_dim]``; the (block, head) page starts at
element ``(block*heads + h)*page*head_dim`` and inside it

* K bf16: token t, dim d at ``((d >> 1)*page + t)*2 + (d & 1)`` (``:76-82``)
* K fp32: token t, dim d at ``d*page + t`` (``:90-94``)
* V:      token t, dim d at ``t*head_dim + d`` (``:110-113``)

Arrays are raw element bits: ``uint16`` for bf16, ``float32`` (or its ``uint32``
view) for fp32, so comparisons are byte-for-byte.
"""

import numpy as np


def k_offset(t, d, page, bf16):
    """Element offset of K (token t, dim d) inside its (block, head) page."""
    if bf16:
        return ((d >> 1) * page + t) * 2 + (d & 1)
    return d * page + t


def k_perm(page, head_dim, bf16):
    """idx[t, d] = k_offset(t, d): a [page, head_dim] gather/scatter map."""
    t = np.arange(page)[:, None]
    d = np.arange(head_dim)[None, :]
    return k_offset(t, d, page, bf16)


def store(k_cache, v_cache, key, value, slots):
    """reshape_and_cache into flat numpy caches (in place).

    k_cache/v_cache: [num_blocks, heads, page, head_dim] arrays of element bits;
    key/value: [tokens, heads, head_dim] of the same element type; slots: int64
    [tokens], token i -> page slots[i] // page at position slots[i] % page; a
    negative slot skips the token (`paged_attn.mojo:155-158`).
    """
    nb, heads, page, hd = k_cache.shape
    bf16 = k_cache.dtype == np.uint16
    perm = k_perm(page, hd, bf16)
    kflat = k_cache.reshape(nb, heads, page * hd)
    for i, s in enumerate(np.asarray(slots, dtype=np.int64)):
        if s < 0:
            continue
        blk, off = divmod(int(s), page)
        for h in range(heads):
            kflat[blk, h, perm[off]] = key[i, h]
            v_cache[blk, h, off] = value[i, h]


def slots_for_append(lens, page_table, page):
    """Slots of an append at position lens[i] through the page table
    (`paged_attn.mojo:162-168`); -1 where lens[i] < 0."""
    lens = np.asarray(lens, dtype=np.int64)
    out = np.full(lens.shape, -1, dtype=np.int64)
    for i, n in enumerate(lens):
        if n >= 0:
            out[i] = int(page_table[i, n // page]) * page + n % page
    return out


def gather(k_cache, v_cache, page_table_row, length, h):
    """The first ``length`` tokens of one sequence's head ``h``, read back through
    the layout: (K [length, head_dim], V [length, head_dim])."""
    nb, heads, page, hd = k_cache.shape
    bf16 = k_cache.dtype == np.uint16
    perm = k_perm(page, hd, bf16)
    kflat = k_cache.reshape(nb, heads, page * hd)
    ks, vs = [], []
    for pos in range(length):
        blk = int(page_table_row[pos // page])
        off = pos % page
        ks.append(kflat[blk, h, perm[off]])
        vs.append(v_cache[blk, h, off])
    if not ks:
        return np.zeros((0, hd), k_cache.dtype), np.zeros((0, hd), v_cache.dtype)
    return np.stack(ks), np.stack(vs)
