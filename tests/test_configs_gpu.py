"""Every BASELINE config at its full size on the B200, through the public API,
against the C restatement of the reference's CPU kernel (the north-star
tolerance: bf16 max-abs <= 2e-2, fp32 <= 1e-4 relative) and, on a sample of
(batch, head) pairs where the float64 oracle is affordable, against the
reference's own gates (`tests/reference.py:24-40`).

* cfg1  flash_attn_func bf16 N=1 L=S=128 H=16 E=64 causal, q/k/v drawn from
        torch.manual_seed(0) (the exact inputs the config names).
* cfg3  cross-attention decode, fp32, B=64 H=8 E=64 (and E=32) page 32, 1500
        pre-staged tokens per sequence in a shuffled block order, no append.
* cfg4  flash_attn_func bf16 N=4 L=S=2048 H=32 E=128 causal, q/k/v strided
        views of one fused [N, L, 3, H, E] tensor; cfg4nc: L=512 S=2048.
* cfg5  the engine route (`examples/ops.py:19-31`) at H=32 E=128 page 16 with
        lengths up to 8191 (several >= 6000), ~5% slot_mapping entries -1,
        reshape_and_cache then decode into a preallocated out; B=64 of the
        config's 256 sequences so that the host oracle stays in seconds.

cfg2 at full size is `test_decode_gpu.py::test_cfg2_scale_against_cpu_restatement`.
Caches are NaN-poisoned outside the written tokens (`test_kvcache.py:16-40`).
"""

import numpy as np
import pytest
import torch

from helpers import north_star_ok
from oracle import attention_f64 as F64
from oracle import cpu as ORACLE

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _api():
    import cpu_attention
    return cpu_attention


def _cpu_flash(q, k, v, causal):
    out = torch.empty(q.shape, dtype=q.dtype)
    ORACLE.flash(q.cpu(), k.cpu(), v.cpu(), out, causal=causal)
    return out


def _f64_sample(out, q, k, v, causal, pairs):
    """The reference's bf16 prefill gate on a few (batch, head) pairs."""
    E = q.shape[-1]
    for b, h in pairs:
        ref = F64.attention(q[b:b + 1, :, h:h + 1], k[b:b + 1, :, h:h + 1], v[b:b + 1, :, h:h + 1], E ** -0.5,
                            causal)
        err, tol = F64.check(out[b:b + 1, :, h:h + 1], ref, True)
        assert err <= tol, (b, h, err)


def test_cfg1_exact_inputs():
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 128, 16, 64, dtype=torch.bfloat16) for _ in range(3))
    out = _api().flash_attn_func(q.to(DEV), k.to(DEV), v.to(DEV), causal=True)
    err, tol = F64.check(out, F64.attention(q, k, v, 64 ** -0.5, True), True)
    assert err <= tol, err
    err, tol = north_star_ok(out, _cpu_flash(q, k, v, True), torch.bfloat16)
    assert err <= tol, err


@pytest.mark.parametrize("causal", [True, False], ids=["cfg4", "cfg4nc"])
def test_cfg4_full_size_fused_views(causal):
    N, S, H, E = 4, 2048, 32, 128
    L = S if causal else 512
    g = torch.Generator(device=DEV).manual_seed(4)
    qkv = torch.randn(N, S, 3, H, E, generator=g, device=DEV).to(torch.bfloat16)
    q, k, v = qkv[:, S - L:, 0], qkv[:, :, 1], qkv[:, :, 2]
    assert q.stride(1) == 3 * H * E
    out = _api().flash_attn_func(q, k, v, causal=causal)
    qc, kc, vc = (x.cpu() for x in (q, k, v))
    err, tol = north_star_ok(out, _cpu_flash(qc, kc, vc, causal), torch.bfloat16)
    assert err <= tol, err
    _f64_sample(out.cpu(), qc, kc, vc, causal, [(0, 0), (1, 17), (2, 5), (3, 31)])
    # the same call again gives the same bits (no state carried between calls)
    assert torch.equal(out, _api().flash_attn_func(q, k, v, causal=causal))


def _pool(lens, page, extra, g):
    """A page table over a shared pool of sum(ceil((len + extra) / page)) blocks
    in a seeded random order; padding entries point at block 0."""
    npages = [-(-(int(n) + extra) // page) for n in lens]
    nblocks = max(1, sum(npages))
    perm = torch.randperm(nblocks, generator=g).to(torch.int32)
    bt = torch.zeros(len(lens), max(npages), dtype=torch.int32)
    s = 0
    for i, n in enumerate(npages):
        bt[i, :n] = perm[s:s + n]
        s += n
    return bt, nblocks


def _fill(kc, vc, bt, lens, page, dtype, seed):
    """Writes lens[i] N(0,1) tokens per sequence through reshape_and_cache, in
    chunks (contiguous slot_mapping per sequence)."""
    H, E = kc.shape[1], kc.shape[3]
    seq = torch.cat([torch.full((int(n),), i, dtype=torch.int64) for i, n in enumerate(lens)])
    pos = torch.cat([torch.arange(int(n)) for n in lens])
    slots = bt[seq, pos // page].long() * page + pos % page
    gd = torch.Generator(device=DEV).manual_seed(seed)
    for a in range(0, len(slots), 32768):
        sl = slots[a:a + 32768].to(DEV)
        k = torch.randn(len(sl), H, E, generator=gd, device=DEV).to(dtype)
        v = torch.randn(len(sl), H, E, generator=gd, device=DEV).to(dtype)
        _api().reshape_and_cache(k, v, kc, vc, sl)


@pytest.mark.parametrize("E", [64, 32], ids=["cfg3", "cfg3e32"])
def test_cfg3_cross_attention_full_size(E):
    B, H, page, n = 64, 8, 32, 1500
    g = torch.Generator().manual_seed(3)
    lens = torch.full((B,), n, dtype=torch.int32)
    bt, nblocks = _pool(lens, page, 0, g)
    kc = torch.full((nblocks, H, page, E), float("nan"), dtype=torch.float32, device=DEV)
    vc = kc.clone()
    _fill(kc, vc, bt, lens, page, torch.float32, seed=E)
    q = torch.randn(B, 1, H, E, generator=g).to(DEV)
    out = _api().flash_attn_with_kvcache(q, kc, vc, cache_seqlens=lens.to(DEV), page_table=bt.to(DEV))
    ref = torch.empty(B, H, E)
    ORACLE.decode(q.cpu()[:, 0].contiguous(), kc.cpu(), vc.cpu(), lens, bt, ref)
    err, tol = north_star_ok(out[:, 0], ref, torch.float32)
    assert err <= tol, err
    # the reference's own fp32 paged gate (1e-6 against float64) on a few sequences
    kcc, vcc = kc.cpu(), vc.cpu()
    for i in (0, 31, 63):
        pages = bt[i, :-(-n // page)].long()
        ks = kcc[pages]  # [pages, H, page, E] in the page layout: K is [E][page] per (block, head)
        kt = ks.view(len(pages), H, E, page).permute(0, 3, 1, 2).reshape(-1, H, E)[:n]
        vt = vcc[pages].permute(0, 2, 1, 3).reshape(-1, H, E)[:n]
        ref64 = F64.attention(q.cpu()[i:i + 1], kt[None], vt[None], E ** -0.5)
        err, tol = F64.check(out.cpu()[i:i + 1], ref64, False, paged=True)
        assert err <= tol, (i, err)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_cfg5_engine_route_long_sequences(dtype):
    from cpu_attention import _kernel as K
    B, H, E, page = 64, 32, 128, 16
    g = torch.Generator().manual_seed(5)
    lens = torch.randint(1, 8192, (B,), generator=g, dtype=torch.int32)
    lens[:5] = torch.tensor([8191, 7000, 6500, 6001, 8176], dtype=torch.int32)  # 8176: a page-aligned end
    bt, nblocks = _pool(lens, page, 1, g)  # room for each sequence's new token
    kc = torch.full((nblocks, H, page, E), float("nan"), dtype=dtype, device=DEV)
    vc = kc.clone()
    _fill(kc, vc, bt, lens, page, dtype, seed=55)
    q = torch.randn(B, H, E, generator=g).to(dtype)
    kn, vn = (torch.randn(B, H, E, generator=g).to(dtype) for _ in range(2))
    slots = torch.tensor([int(bt[i, int(lens[i]) // page]) * page + int(lens[i]) % page for i in range(B)])
    drop = torch.rand(B, generator=g) < 0.05
    drop[7] = True
    slots[drop] = -1
    after = lens + (slots >= 0).to(torch.int32)
    # the oracle stores and attends on host copies of the caches as they are now
    kcc, vcc = kc.cpu(), vc.cpu()
    ref = torch.empty(B, H, E, dtype=dtype)
    ORACLE.decode(q, kcc, vcc, after, bt, ref, k_new=kn, v_new=vn, slots=slots)
    # the engine's step: reshape_and_cache at slot_mapping, then decode into out
    out = torch.empty(B, H, E, dtype=dtype, device=DEV)
    d = lambda x: x.to(DEV)  # noqa: E731
    _api().reshape_and_cache(d(kn), d(vn), kc, vc, d(slots))
    got = K.module().decode(K.runtime(), d(q), kc, vc, None, None, None, d(after), d(bt), None, out)
    assert got is out
    err, tol = north_star_ok(out, ref, dtype)
    assert err <= tol, err
    # the store left exactly the oracle's caches (bit-exact), NaN padding included
    assert np.array_equal(kc.cpu().view(torch.int16 if dtype == torch.bfloat16 else torch.int32).numpy(),
                          kcc.view(torch.int16 if dtype == torch.bfloat16 else torch.int32).numpy())
    assert K.status(out.device, K.current_stream(out.device)) == 0
