"""Seeded inputs of the parity cases, shared by the tests, the golden-fixture
script (tests/golden/make_golden.py) and the bench.

Every generator draws from a seeded CPU ``torch.Generator`` in the order the
reference's own tests draw (``tests/test_flash.py:56-60``,
``tests/test_kvcache.py:118-141`` of ducviet00/cpu-attention), so the committed
golden outputs (made by the reference's float64 oracle) belong to exactly these
inputs; ``digest()`` fingerprints the bytes to prove it.
"""

import hashlib

import torch

DTYPES = [torch.float32, torch.bfloat16]
# (seq_q, seq_k): tile edges, single rows, unequal lengths both ways (test_flash.py:53)
LENGTHS = [(1, 1), (17, 17), (64, 64), (129, 129), (1, 300), (100, 37), (37, 100), (257, 513)]


def digest(*tensors):
    """sha256 of the tensors' raw bytes (CPU)."""
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().to("cpu").contiguous()
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16
                 else t.view(torch.int16).numpy().tobytes())
    return h.hexdigest()[:16]


def flash_inputs(b, sq, sk, h, d, dtype, seed):
    """q [b, sq, h, d], k/v [b, sk, h, d] as the reference's test_flash.run draws them."""
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(b, n, h, d, generator=g).to(dtype) for n in (sq, sk, sk))


def flash_cases():
    """(name, b, sq, sk, h, d, dtype, causal, seed, scale) of the golden flash set."""
    out = []
    for dtype in DTYPES:
        dn = "bf16" if dtype == torch.bfloat16 else "fp32"
        for causal in (True, False):
            for sq, sk in LENGTHS:
                out.append((f"f_{dn}_d64_{sq}x{sk}_c{int(causal)}", 1, sq, sk, 1, 64, dtype, causal,
                            sq * 1000 + sk, None))
            for d in (32, 128):
                for sq, sk in ((17, 17), (100, 37), (37, 100), (1, 300)):
                    out.append((f"f_{dn}_d{d}_{sq}x{sk}_c{int(causal)}", 1, sq, sk, 2, d, dtype, causal,
                                sq * 1000 + sk, None))
        out.append((f"f_{dn}_batch_scale", 2, 30, 50, 3, 64, dtype, True, 1, 0.07))
    return out


def stage_inputs(lens, h, d, page, dtype, seed):
    """The reference's test_kvcache.stage draws (test_kvcache.py:118-141): the
    block order, the page table (padding points at a poisoned page), q, and each
    sequence's K/V tokens. Returns (q [B,1,h,d], bt int32, total_blocks, ks, vs)
    with ks[i]/vs[i] of shape [1, n_i, h, d]."""
    g = torch.Generator().manual_seed(seed)
    npages = [-(-n // page) for n in lens]
    total = sum(npages) + 1
    order = torch.randperm(total, generator=g).to(torch.int32)
    bt = torch.full((len(lens), max(npages) + 1), int(order[-1]), dtype=torch.int32)
    q = torch.randn(len(lens), 1, h, d, generator=g).to(dtype)
    ks, vs, start = [], [], 0
    for i, n in enumerate(lens):
        bt[i, :npages[i]] = order[start:start + npages[i]]
        start += npages[i]
        k, v = (torch.randn(1, n, h, d, generator=g).to(dtype) for _ in range(2))
        ks.append(k)
        vs.append(v)
    return q, bt, total, ks, vs


def decode_cases():
    """(name, lens, h, d, page, dtype, seed, scale) of the golden decode set:
    test_decode's lengths for every page/head_dim/dtype (test_kvcache.py:59-66),
    the threads test's lopsided batches (:86-97) and the fuzz seeds (:112-120)."""
    out = []
    for dtype in DTYPES:
        dn = "bf16" if dtype == torch.bfloat16 else "fp32"
        for page in (16, 32, 48, 64):
            for d in (32, 64, 128):
                for h in (1, 8):
                    out.append((f"d_{dn}_p{page}_d{d}_h{h}", [0, 1, page - 1, page, page + 1, 255, 257], h, d,
                                page, dtype, page + d, None))
    for i, lens in enumerate(([0, 2047, 1, 17, 64], [2047, 16], [5, 3, 1024])):
        out.append((f"d_threads_{i}", lens, 8, 64, 16, torch.float32, i + 1, None))
    import random
    for seed in range(30):
        r = random.Random(seed)
        lens = [r.randint(0, 1100) for _ in range(r.randint(1, 6))]
        d = r.choice([32, 64, 128])
        h = r.choice([1, 4, 12])
        page = r.choice([16, 32, 48, 64])
        dtype = r.choice(DTYPES)
        scale = r.choice([1.0, 0.5]) * d ** -0.5
        out.append((f"d_fuzz_{seed}", lens, h, d, page, dtype, seed, scale))
    return out


# ---- grouped heads (GQA/MQA) and packed sequences (varlen) -----------------
# The reference declines both; its float64 oracle is MHA over padded batches,
# so their golden outputs come from it with K/V heads repeated to the query
# heads (query head h reads KV head h // (h_q // h_kv)) and from one call per
# sequence (tests/golden/make_golden.py).
GQA_HEADS = [(4, 2), (6, 2), (8, 2), (10, 2), (16, 2), (8, 1)]  # groups 2, 3, 4, 5, 8 and MQA
GQA_MQA32 = (32, 1)  # a group of 32: four items of eight rows per KV head


def expand_kv(x, heads):
    """[..., h_kv, d] -> [..., heads, d]: each KV head repeated for its group."""
    return x.repeat_interleave(heads // x.shape[-2], dim=-2)


def gqa_flash_inputs(b, sq, sk, h, hk, d, dtype, seed):
    """q [b, sq, h, d], k/v [b, sk, hk, d], drawn in that order."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(b, sq, h, d, generator=g).to(dtype),
            torch.randn(b, sk, hk, d, generator=g).to(dtype),
            torch.randn(b, sk, hk, d, generator=g).to(dtype))


def gqa_flash_cases():
    """(name, b, sq, sk, h, hk, d, dtype, causal, seed) of the golden GQA prefill set."""
    out = []
    for dtype in DTYPES:
        dn = "bf16" if dtype == torch.bfloat16 else "fp32"
        for n, (h, hk) in enumerate(GQA_HEADS[:4] + [GQA_HEADS[5]]):
            d = (64, 128, 32, 32, 64)[n]
            for causal in (True, False):
                for sq, sk in ((17, 17), (40, 150)):
                    out.append((f"g_{dn}_h{h}k{hk}_d{d}_{sq}x{sk}_c{int(causal)}", 1, sq, sk, h, hk, d, dtype,
                                causal, 7 * n + sq))
    return out


def gqa_stage_inputs(lens, h, hk, d, page, dtype, seed):
    """stage_inputs with q of h heads and K/V of hk heads."""
    g = torch.Generator().manual_seed(seed)
    npages = [-(-n // page) for n in lens]
    total = sum(npages) + 1
    order = torch.randperm(total, generator=g).to(torch.int32)
    bt = torch.full((len(lens), max(npages) + 1), int(order[-1]), dtype=torch.int32)
    q = torch.randn(len(lens), 1, h, d, generator=g).to(dtype)
    ks, vs, start = [], [], 0
    for i, n in enumerate(lens):
        bt[i, :npages[i]] = order[start:start + npages[i]]
        start += npages[i]
        k, v = (torch.randn(1, n, hk, d, generator=g).to(dtype) for _ in range(2))
        ks.append(k)
        vs.append(v)
    return q, bt, total, ks, vs


def gqa_decode_cases():
    """(name, lens, h, hk, d, page, dtype, seed, scale) of the golden GQA decode set."""
    out = []
    for dtype in DTYPES:
        dn = "bf16" if dtype == torch.bfloat16 else "fp32"
        for n, (h, hk) in enumerate(GQA_HEADS + [GQA_MQA32]):
            for page in (16, 32):
                d = (128, 64, 32)[(n + page // 16) % 3] if h <= 10 else 32
                out.append((f"gd_{dn}_h{h}k{hk}_d{d}_p{page}", [0, 1, page, page + 1, 300, 2047], h, hk, d, page,
                            dtype, 100 * n + page, None))
    return out


def varlen_inputs(lq, lk, h, hk, d, dtype, seed):
    """Packed q [sum(lq), h, d], k/v [sum(lk), hk, d] and int32 offsets."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(sum(lq), h, d, generator=g).to(dtype)
    k = torch.randn(sum(lk), hk, d, generator=g).to(dtype)
    v = torch.randn(sum(lk), hk, d, generator=g).to(dtype)
    cq = torch.tensor([0] + list(torch.tensor(lq).cumsum(0)), dtype=torch.int32)
    ck = torch.tensor([0] + list(torch.tensor(lk).cumsum(0)), dtype=torch.int32)
    return q, k, v, cq, ck


def varlen_cases():
    """(name, lq, lk, h, hk, d, dtype, causal, seed): ragged batches with empty,
    single-token, tile-edge and unequal q/k lengths."""
    shapes = [([5, 1, 130, 64], [5, 7, 130, 200]), ([100, 0, 17], [100, 33, 17]), ([128, 129], [128, 260]),
              ([1, 260], [300, 260])]
    out = []
    for dtype in DTYPES:
        dn = "bf16" if dtype == torch.bfloat16 else "fp32"
        for n, (lq, lk) in enumerate(shapes):
            h, hk = ((2, 2), (4, 2), (3, 3), (2, 1))[n]
            d = (64, 128, 32, 32)[n]
            for causal in (True, False):
                out.append((f"v_{dn}_{n}_c{int(causal)}", lq, lk, h, hk, d, dtype, causal, 11 * n + 1))
    return out
