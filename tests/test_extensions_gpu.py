"""The hot path's extensions beyond the reference, on the B200 through the C ABI:
grouped heads (GQA/MQA) in decode and prefill, the softmax log-sum-exp
(``return_softmax_lse`` / ``return_attn_probs``) and packed sequences
(``flash_attn_varlen_func``). The reference declines all three
(`cpu_attention/flash_attn_interface.py:87-96`, `:144-145`, `:215-218`).

Each output is checked against the golden outputs of the reference's float64
oracle (K/V heads repeated to the query heads; one call per packed sequence)
with the reference's gates (`tests/reference.py:24-40`), and against the C
restatement of the reference's kernel on the same repeated heads with the
north-star tolerance (bf16 max-abs 2e-2, fp32 1e-4 relative). Log-sum-exps are
checked against the float64 definition within LSE_TOL.

Also here: a decode whose device waits are made to run out (a 1 us limit)
reports CA_STATUS_TIMEOUT and returns, and after the status is reset the same
workspace serves a correct call again.
"""

import pytest
import torch

import cases
from helpers import golden, north_star_ok, stage_cache
from oracle import attention_f64 as F64
from oracle import cpu as ORACLE

pytestmark = pytest.mark.gpu
DEV = "cuda"
LSE_TOL = 1e-4  # absolute, natural-log units


def _api():
    import cpu_attention
    return cpu_attention


def _store(key, value, kc, vc, slots):
    _api().reshape_and_cache(key, value, kc, vc, slots)


def _expand_cache(c, heads):
    """[blocks, kv_heads, page, dim] -> [blocks, heads, page, dim] (whole pages repeated)."""
    return cases.expand_kv(c.transpose(1, 2), heads).transpose(1, 2).contiguous()


def _oracle_decode(q, kc, vc, bt, lens, heads, k_new=None, v_new=None, slots=None, scale=None):
    """The C restatement on host copies of the caches with KV heads repeated."""
    b, _, _, d = kc.shape
    out = torch.empty(q.shape[0], heads, q.shape[-1], dtype=q.dtype)
    qc = q.cpu().reshape(q.shape[0], heads, q.shape[-1]).contiguous()
    ex = lambda t: None if t is None else cases.expand_kv(t.cpu().reshape(q.shape[0], -1, q.shape[-1]),  # noqa
                                                          heads).contiguous()
    ORACLE.decode(qc, _expand_cache(kc.cpu(), heads), _expand_cache(vc.cpu(), heads), lens.cpu(), bt.cpu(), out,
                  k_new=ex(k_new), v_new=ex(v_new), slots=None if slots is None else slots.cpu(), scale=scale)
    return out


# ------------------------------------------------------------------ decode --
@pytest.mark.parametrize("case", cases.gqa_decode_cases(), ids=lambda c: c[0])
def test_gqa_decode_golden(case):
    name, lens, h, hk, d, page, dtype, seed, scale = case
    q, kc, vc, bt, ks, vs = stage_cache(lens, h, d, page, dtype, seed, _store, device=DEV, gqa=hk)
    L = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out, lse = _api().flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt, return_softmax_lse=True)
    assert out.shape == q.shape and lse.shape == (len(lens), h, 1) and lse.dtype == torch.float32
    err, tol = F64.check(out, golden("ext")[name], dtype == torch.bfloat16, paged=True)
    assert err <= tol, err
    err, tol = north_star_ok(out[:, 0], _oracle_decode(q, kc, vc, bt, L, h), dtype)
    assert err <= tol, err
    # the log-sum-exp of each row against the float64 definition
    ref = [F64.logsumexp(q[i:i + 1].cpu(), cases.expand_kv(ks[i], h), None, d ** -0.5)[0, :, 0]
           for i in range(len(lens))]
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.isneginf(lse[i]).all()
        else:
            assert (lse[i, :, 0].cpu().double() - torch.from_numpy(ref[i])).abs().max() <= LSE_TOL


@pytest.mark.parametrize("dtype", cases.DTYPES)
@pytest.mark.parametrize("h,hk,n_new", [(8, 2, 1), (12, 4, 1), (32, 4, 3), (8, 1, 17)])
def test_gqa_decode_appends_new_tokens(dtype, h, hk, n_new):
    """k/v of nheads_k heads appended at cache_seqlens (one token, or a prompt)
    and attended in the same launch; the cache afterwards equals the two-step
    store-then-decode route bit for bit."""
    d, page = 64, 16
    lens = [0, 15, 16, 100, 700]
    q, kc, vc, bt, ks, vs = stage_cache(lens, h, d, page, dtype, 3, _store, device=DEV, gqa=hk)
    # room for the new tokens: past each sequence's own pages, fresh NaN blocks
    # of its own (the staged table's padding shares one poisoned block)
    W = -(-(max(lens) + n_new) // page)
    fresh = kc.shape[0]
    table = torch.zeros(len(lens), W, dtype=torch.int32)
    for i, n in enumerate(lens):
        own = -(-n // page)
        table[i, :own] = bt[i, :own].cpu()
        table[i, own:] = torch.arange(fresh, fresh + W - own, dtype=torch.int32)
        fresh += W - own
    bt = table.to(DEV)
    pad = torch.full((fresh - kc.shape[0],) + kc.shape[1:], float("nan"), dtype=dtype, device=DEV)
    kc, vc = torch.cat([kc, pad]), torch.cat([vc, pad])
    g = torch.Generator().manual_seed(h * n_new)
    kn, vn = (torch.randn(len(lens), n_new, hk, d, generator=g).to(dtype) for _ in range(2))
    L = torch.tensor(lens, dtype=torch.int32)
    kc2, vc2 = kc.clone(), vc.clone()
    out = _api().flash_attn_with_kvcache(q, kc, vc, k=kn.to(DEV), v=vn.to(DEV), cache_seqlens=L.to(DEV),
                                         page_table=bt)
    for i in range(len(lens)):
        kk = torch.cat([ks[i], kn[i:i + 1]], 1)
        vv = torch.cat([vs[i], vn[i:i + 1]], 1)
        ref = F64.attention(q[i:i + 1].cpu(), cases.expand_kv(kk, h), cases.expand_kv(vv, h), d ** -0.5)
        err, tol = F64.check(out[i:i + 1], ref, dtype == torch.bfloat16, paged=True)
        assert err <= tol, (i, err)
    # the two-step route: reshape_and_cache at lens + j, then decode the grown cache
    pos = L.long()[:, None] + torch.arange(n_new)[None]
    slots = (bt.cpu().long().gather(1, pos // page) * page + pos % page).flatten().to(DEV)
    _api().reshape_and_cache(kn.flatten(0, 1).to(DEV), vn.flatten(0, 1).to(DEV), kc2, vc2, slots)
    assert torch.equal(kc.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       kc2.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))
    assert torch.equal(vc.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       vc2.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))


@pytest.mark.parametrize("dtype", cases.DTYPES)
def test_gqa_engine_route_slots(dtype):
    """The engine's direct call with grouped heads: new tokens of nheads_k heads
    stored at slot_mapping (one padded), 3-D q, preallocated out, lse."""
    from cpu_attention import _kernel as K
    h, hk, d, page = 16, 4, 128, 16
    lens = [5, 300, 31, 1024, 77]
    q, kc, vc, bt, ks, vs = stage_cache(lens, h, d, page, dtype, 9, _store, device=DEV, gqa=hk)
    g = torch.Generator().manual_seed(9)
    B = len(lens)
    kn, vn = (torch.randn(B, hk, d, generator=g).to(dtype) for _ in range(2))
    btc = bt.cpu()
    slots = torch.tensor([int(btc[i, n // page]) * page + n % page if n % page else -1 for i, n in enumerate(lens)])
    slots[2] = -1
    after = torch.tensor(lens, dtype=torch.int32) + (slots >= 0).to(torch.int32)
    ref = _oracle_decode(q[:, 0], kc, vc, bt, after, h, k_new=kn, v_new=vn, slots=slots)
    out = torch.empty(B, h, d, dtype=dtype, device=DEV)
    lse = torch.empty(B, h, dtype=torch.float32, device=DEV)
    got = K.module().decode(K.runtime(), q[:, 0], kc, vc, kn.to(DEV), vn.to(DEV), slots.to(DEV), after.to(DEV), bt,
                            None, out, lse)
    assert got is out
    err, tol = north_star_ok(out, ref, dtype)
    assert err <= tol, err
    assert torch.isfinite(lse).all()


@pytest.mark.parametrize("page", [64, 128])
@pytest.mark.parametrize("d", [64, 128])
def test_gqa_decode_large_pages(page, d):
    """Grouped bf16 rows on large pages: several 16-key blocks per page, the
    online softmax carried across them and across the pages of a run, a
    ragged last block over NaN-poisoned slots; against the C restatement."""
    dtype, h, hk = torch.bfloat16, 16, 4
    lens = [1, page - 1, page, page + 17, 3 * page + 5, 1000]
    q, kc, vc, bt, ks, vs = stage_cache(lens, h, d, page, dtype, page + d, _store, device=DEV, gqa=hk)
    L = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = _api().flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt)
    err, tol = north_star_ok(out[:, 0], _oracle_decode(q, kc, vc, bt, L, h), dtype)
    assert err <= tol, err


@pytest.mark.parametrize("dtype", cases.DTYPES)
@pytest.mark.parametrize("h,hk", [(32, 8), (64, 8), (32, 1)])
def test_gqa_decode_bitwise_reproducible(dtype, h, hk):
    """Run states are folded in run order and split tasks in task order, so
    the result does not depend on which warp or SM streamed what: repeated
    calls, with differently sized calls in between to shift the scheduling,
    return the same bits."""
    d, page, B = 128, 16, 24
    g = torch.Generator().manual_seed(7 + h + hk)
    lens = torch.randint(1, 3000, (B,), generator=g).tolist()
    q, kc, vc, bt, ks, vs = stage_cache(lens, h, d, page, dtype, h + hk, _store, device=DEV, gqa=hk)
    L = torch.tensor(lens, dtype=torch.int32, device=DEV)
    first = _api().flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt)
    for i in range(3):
        n = B // 2 + 3 * i
        _api().flash_attn_with_kvcache(q[:n], kc, vc, cache_seqlens=L[:n], page_table=bt[:n])
        assert torch.equal(first, _api().flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt)), i


@pytest.mark.parametrize("dtype", cases.DTYPES)
@pytest.mark.parametrize("h,hk", [(32, 8), (32, 32), (64, 8), (16, 1)])
def test_gqa_decode_long_sequences(dtype, h, hk):
    """Long, ragged sequences (many split tasks and merges per item) at
    head_dim 128 page 16, against the C restatement; lse checked too."""
    d, page, B = 128, 16, 12
    g = torch.Generator().manual_seed(h + hk)
    lens = torch.randint(1, 6000, (B,), generator=g).tolist()
    lens[:2] = [6000, 4097]
    q, kc, vc, bt, ks, vs = stage_cache(lens, h, d, page, dtype, h * hk, _store, device=DEV, gqa=hk)
    L = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out, lse = _api().flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt, return_softmax_lse=True)
    err, tol = north_star_ok(out[:, 0], _oracle_decode(q, kc, vc, bt, L, h), dtype)
    assert err <= tol, err
    for i in (0, 5):
        ref = F64.logsumexp(q[i:i + 1].cpu(), cases.expand_kv(ks[i], h), None, d ** -0.5)[0, :, 0]
        assert (lse[i, :, 0].cpu().double() - torch.from_numpy(ref)).abs().max() <= LSE_TOL
    # the MHA output does not depend on whether lse was asked for
    assert torch.equal(out, _api().flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt))


# ----------------------------------------------------------------- prefill --
@pytest.mark.parametrize("case", cases.gqa_flash_cases(), ids=lambda c: c[0])
def test_gqa_flash_golden(case):
    name, b, sq, sk, h, hk, d, dtype, causal, seed = case
    q, k, v = cases.gqa_flash_inputs(b, sq, sk, h, hk, d, dtype, seed)
    out, lse = _api().flash_attn_func(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal, return_attn_probs=True)
    err, tol = F64.check(out, golden("ext")[name], dtype == torch.bfloat16)
    assert err <= tol, err
    ref = torch.empty(q.shape, dtype=dtype)
    ORACLE.flash(q, cases.expand_kv(k, h).contiguous(), cases.expand_kv(v, h).contiguous(), ref, causal=causal)
    err, tol = north_star_ok(out, ref, dtype)
    assert err <= tol, err
    want = torch.from_numpy(F64.logsumexp(q, cases.expand_kv(k, h), None, d ** -0.5, causal))
    got = lse.cpu().double()
    assert got.shape == want.shape
    fin = torch.isfinite(want)
    assert torch.equal(torch.isneginf(got), ~fin)
    assert (got[fin] - want[fin]).abs().max() <= LSE_TOL


@pytest.mark.parametrize("dtype", cases.DTYPES)
@pytest.mark.parametrize("causal", [True, False])
def test_flash_lse_mha_long(dtype, causal):
    """return_attn_probs on an MHA prefill long enough for many key tiles and
    rescales (bf16: the tensor-core kernel's slack-8 running max)."""
    b, s, h, d = 1, 700, 2, 128
    q, k, v = cases.flash_inputs(b, s, s, h, d, dtype, 5)
    out, lse = _api().flash_attn_func(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal, return_attn_probs=True)
    assert torch.equal(out, _api().flash_attn_func(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal))
    want = torch.from_numpy(F64.logsumexp(q, k, None, d ** -0.5, causal))
    assert (lse.cpu().double() - want).abs().max() <= LSE_TOL


@pytest.mark.parametrize("case", cases.varlen_cases(), ids=lambda c: c[0])
def test_varlen_golden(case):
    name, lq, lk, h, hk, d, dtype, causal, seed = case
    q, k, v, cq, ck = cases.varlen_inputs(lq, lk, h, hk, d, dtype, seed)
    C = _api()
    out, lse = C.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cq.to(DEV), ck.to(DEV), max(lq), max(lk),
                                        causal=causal, return_attn_probs=True)
    assert out.shape == q.shape and lse.shape == (h, q.shape[0])
    err, tol = F64.check(out, golden("ext")[name], dtype == torch.bfloat16)
    assert err <= tol, err
    # each sequence equals a dense call on it alone, bit for bit; host offsets too
    out_host = C.flash_attn_varlen_func(q.to(DEV), k.to(DEV), v.to(DEV), cq, ck, max(lq), max(lk), causal=causal)
    assert torch.equal(out, out_host)
    for i in range(len(lq)):
        a, z, ka, kz = int(cq[i]), int(cq[i + 1]), int(ck[i]), int(ck[i + 1])
        if z == a:
            continue
        if kz == ka:
            assert (out[a:z] == 0).all()
            assert torch.isneginf(lse[:, a:z]).all()
            continue
        dense, dl = C.flash_attn_func(q[a:z][None].to(DEV), k[ka:kz][None].to(DEV), v[ka:kz][None].to(DEV),
                                      causal=causal, return_attn_probs=True)
        assert torch.equal(out[a:z], dense[0]), i
        assert torch.equal(lse[:, a:z], dl[0]), i


def test_varlen_fused_projection_views():
    """Packed q/k/v as strided views of one [total, 3, heads, dim] projection."""
    lq = [33, 200, 1]
    qkv = torch.randn(sum(lq), 3, 4, 64, generator=torch.Generator().manual_seed(8)).bfloat16().to(DEV)
    cu = torch.tensor([0, 33, 233, 234], dtype=torch.int32, device=DEV)
    out = _api().flash_attn_varlen_func(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu, cu, 200, 200, causal=True)
    for i in range(3):
        a, z = int(cu[i]), int(cu[i + 1])
        ref = F64.attention(qkv[a:z, 0][None], qkv[a:z, 1][None], qkv[a:z, 2][None], 64 ** -0.5, True)
        err, tol = F64.check(out[a:z][None], ref, True)
        assert err <= tol, err


# ------------------------------------------------------- bounded device waits --
def test_decode_timeout_is_reported_and_the_workspace_recovers():
    """With every device wait limited to 1 us the decode gives up: the kernel
    returns, CA_STATUS_TIMEOUT is set, and resetting the status also clears the
    counter and tickets the abandoned tasks left, so the next call on the same
    workspace is right again (no fault, no hang: every wait is bounded)."""
    from cpu_attention import _kernel as K
    C = _api()
    lib = K.library()
    dtype, h, d, page = torch.bfloat16, 16, 128, 16
    g = torch.Generator().manual_seed(21)
    lens = torch.randint(500, 2000, (32,), generator=g).tolist()
    q, kc, vc, bt, ks, vs = stage_cache(lens, h, d, page, dtype, 21, _store, device=DEV)
    L = torch.tensor(lens, dtype=torch.int32, device=DEV)
    ref = C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt)
    stream = K.current_stream(q.device)
    assert K.status(q.device, stream) == 0
    lib.ca_set_wait_limit_ns(1000)
    try:
        for _ in range(3):
            C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt)
        torch.cuda.synchronize()
    finally:
        lib.ca_set_wait_limit_ns(0)
    assert K.status(q.device, stream, reset=True) & K.STATUS_TIMEOUT
    for _ in range(2):
        out = C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=L, page_table=bt)
        assert torch.equal(out, ref)
    assert K.status(q.device, stream) == 0
