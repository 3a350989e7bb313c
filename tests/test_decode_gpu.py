"""flash_attn_with_kvcache (paged decode) and reshape_and_cache on the B200,
through the C ABI, against the golden outputs of the reference's float64 oracle
(the reference's gates, `tests/reference.py:24-40`) and against the C
restatement of the reference's CPU kernel (bf16
max-abs <= 2e-2, fp32 <= 1e-4 relative). Mirrors `tests/test_kvcache.py` of the
reference case for case."""

import random
import threading

import numpy as np
import pytest
import torch

import cases
from helpers import bits, golden, north_star_ok
from oracle import attention_f64 as F64
from oracle import cpu as ORACLE

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _api():
    import cpu_attention
    return cpu_attention


def stage(lens, h, d, page, dtype, seed):
    """The reference's stage (test_kvcache.py:118-141) on the GPU: NaN-poisoned
    caches filled through the API in two appends per sequence."""
    C = _api()
    q, bt, total, ks, vs = cases.stage_inputs(lens, h, d, page, dtype, seed)
    q, bt = q.to(DEV), bt.to(DEV)
    kc = torch.full((total, h, page, d), float("nan"), dtype=dtype, device=DEV)
    vc = kc.clone()
    for i, n in enumerate(lens):
        k, v = ks[i].to(DEV), vs[i].to(DEV)
        for a, z in ((0, n // 2), (n // 2, n)):
            if z > a:
                C.flash_attn_with_kvcache(q[i:i + 1], kc, vc, k=k[:, a:z], v=v[:, a:z], cache_seqlens=a,
                                          page_table=bt[i:i + 1])
    return q, kc, vc, bt, ks, vs


def cpu_reference(q, kc, vc, bt, lens, scale=None, k_new=None, v_new=None, slots=None):
    """The C restatement of the reference kernel on copies of the same caches."""
    kcc, vcc = kc.cpu(), vc.cpu()
    out = torch.empty(q.shape[0], q.shape[-2], q.shape[-1], dtype=q.dtype)
    qc = q.cpu().reshape(q.shape[0], q.shape[-2], q.shape[-1])
    ORACLE.decode(qc, kcc, vcc, lens.cpu(), bt.cpu(), out,
                  k_new=None if k_new is None else k_new.cpu().reshape(qc.shape).contiguous(),
                  v_new=None if v_new is None else v_new.cpu().reshape(qc.shape).contiguous(),
                  slots=None if slots is None else slots.cpu(), scale=scale)
    return out


@pytest.mark.parametrize("case", cases.decode_cases(), ids=lambda c: c[0])
def test_decode_golden(case):
    name, lens, h, d, page, dtype, seed, scale = case
    C = _api()
    q, kc, vc, bt, ks, vs = stage(lens, h, d, page, dtype, seed)
    seqlens = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seqlens, page_table=bt, softmax_scale=scale)
    assert out.shape == q.shape and out.dtype == dtype and out.device.type == "cuda"
    err, tol = F64.check(out, golden("decode")[name], dtype == torch.bfloat16, paged=True)
    assert err <= tol, (name, err)
    ref = cpu_reference(q, kc, vc, bt, seqlens, scale)
    err, tol = north_star_ok(out[:, 0], ref, dtype)
    assert err <= tol, (name, err)
    for i, n in enumerate(lens):
        if n == 0:
            assert torch.all(out[i] == 0)


@pytest.mark.parametrize("dtype", cases.DTYPES)
def test_append_one_token(dtype):
    """k/v of one new token are written at cache_seqlens and attended in the same
    call; block_table is accepted (test_kvcache.py:69-84)."""
    C = _api()
    lens, h, d = [5, 31, 64, 300], 8, 64
    q, kc, vc, bt, ks, vs = stage(lens, h, d, 16, dtype, seed=3)
    g = torch.Generator().manual_seed(11)
    kn, vn = (torch.randn(len(lens), 1, h, d, generator=g).to(dtype) for _ in range(2))
    seqlens = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = C.flash_attn_with_kvcache(q, kc, vc, k=kn.to(DEV), v=vn.to(DEV), cache_seqlens=seqlens, page_table=bt)
    ref = np.concatenate([F64.attention(q[i:i + 1], torch.cat([ks[i], kn[i:i + 1]], 1),
                                        torch.cat([vs[i], vn[i:i + 1]], 1), d ** -0.5) for i in range(len(lens))])
    err, tol = F64.check(out, ref, dtype == torch.bfloat16, paged=True)
    assert err <= tol
    again = C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seqlens + 1, block_table=bt)
    err, tol = F64.check(again, ref, dtype == torch.bfloat16, paged=True)
    assert err <= tol


def _prompt_case(lens, n, h, d, page, dtype, seed):
    """Caches (NaN elsewhere) holding lens[i] tokens per sequence, with distinct
    blocks for each sequence's pages up to lens[i] + n, and n new tokens."""
    g = torch.Generator().manual_seed(seed)
    npages = [-(-(ln + n) // page) for ln in lens]
    order = torch.randperm(sum(npages), generator=g).to(torch.int32)
    bt = torch.zeros(len(lens), max(npages), dtype=torch.int32)
    start = 0
    for i, npg in enumerate(npages):
        bt[i, :npg] = order[start:start + npg]
        start += npg
    kc = torch.full((sum(npages), h, page, d), float("nan"), dtype=dtype, device=DEV)
    vc = kc.clone()
    C = _api()
    ks, vs = [], []
    for i, ln in enumerate(lens):
        k, v = (torch.randn(ln, h, d, generator=g).to(dtype) for _ in range(2))
        ks.append(k)
        vs.append(v)
        if ln:
            pos = torch.arange(ln)
            C.reshape_and_cache(k.to(DEV), v.to(DEV), kc, vc, (bt[i, pos // page].long() * page + pos % page).to(DEV))
    q = torch.randn(len(lens), 1, h, d, generator=g).to(dtype)
    # the new tokens as a strided view of a fused [B, n, 2, h, d] projection
    kv = torch.randn(len(lens), n, 2, h, d, generator=g).to(dtype)
    return q.to(DEV), kc, vc, bt.to(DEV), ks, vs, kv


@pytest.mark.parametrize("dtype", cases.DTYPES)
@pytest.mark.parametrize("page,n", [(16, 2), (16, 17), (32, 40), (16, 1)])
def test_append_prompt_in_one_launch(dtype, page, n):
    """Several new tokens per sequence (a prompt) are written at cache_seqlens + j
    and attended by the decode launch itself (the reference stores them first,
    `flash_attn_interface.py:109-117`): the output matches the float64 oracle
    over the grown sequences, and the caches match, bit for bit, the ones the
    reference's two steps (reshape_and_cache, then decode) leave."""
    C = _api()
    lens, h, d = [0, 5, 31, 64, 300], 4, 64
    q, kc, vc, bt, ks, vs, kv = _prompt_case(lens, n, h, d, page, dtype, seed=7 + n)
    kn, vn = kv[:, :, 0], kv[:, :, 1]
    kc2, vc2 = kc.clone(), vc.clone()
    seqlens = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = C.flash_attn_with_kvcache(q, kc, vc, k=kn.to(DEV), v=vn.to(DEV), cache_seqlens=seqlens, page_table=bt)
    ref = np.concatenate([F64.attention(q[i:i + 1], torch.cat([ks[i], kn[i]], 0)[None],
                                        torch.cat([vs[i], vn[i]], 0)[None], d ** -0.5) for i in range(len(lens))])
    err, tol = F64.check(out, ref, dtype == torch.bfloat16, paged=True)
    assert err <= tol, err
    pos = torch.tensor(lens)[:, None] + torch.arange(n)[None]
    slots = bt.cpu().long().gather(1, pos // page) * page + pos % page
    C.reshape_and_cache(kn.reshape(-1, h, d).to(DEV), vn.reshape(-1, h, d).to(DEV), kc2, vc2, slots.flatten().to(DEV))
    assert np.array_equal(bits(kc), bits(kc2)) and np.array_equal(bits(vc), bits(vc2))


@pytest.mark.parametrize("dtype", cases.DTYPES)
def test_fused_projection_strides(dtype):
    """q and the new k/v as chunks of one fused [b, 1, 3 h d] projection
    (test_kvcache.py:99-110)."""
    C = _api()
    lens, h, d = [40, 200], 8, 64
    q, kc, vc, bt, ks, vs = stage(lens, h, d, 32, dtype, seed=4)
    qkv = torch.randn(len(lens), 1, 3 * h * d, generator=torch.Generator().manual_seed(4)).to(dtype)
    qn, kn, vn = (qkv[..., i * h * d:(i + 1) * h * d].view(len(lens), 1, h, d) for i in range(3))
    out = C.flash_attn_with_kvcache(qn.to(DEV), kc, vc, k=kn.to(DEV), v=vn.to(DEV), page_table=bt,
                                    cache_seqlens=torch.tensor(lens, dtype=torch.int32, device=DEV))
    ref = np.concatenate([F64.attention(qn[i:i + 1], torch.cat([ks[i], kn[i:i + 1]], 1),
                                        torch.cat([vs[i], vn[i:i + 1]], 1), d ** -0.5) for i in range(len(lens))])
    err, tol = F64.check(out, ref, dtype == torch.bfloat16, paged=True)
    assert err <= tol


def test_concurrent_callers():
    """Python threads calling at once each get their own correct result
    (test_kvcache.py:122-140)."""
    C = _api()
    staged = [stage([100 + 50 * i, 33], 8, 64, 16, torch.float32, seed=i) for i in range(4)]
    refs = [np.concatenate([F64.attention(q[j:j + 1], ks[j], vs[j], 0.125) for j in range(2)])
            for q, _, _, _, ks, vs in staged]
    errors = []

    def worker(i):
        q, kc, vc, bt, _, _ = staged[i]
        seqlens = torch.tensor([100 + 50 * i, 33], dtype=torch.int32, device=DEV)
        for _ in range(20):
            out = C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seqlens, page_table=bt)
            errors.append(F64.check(out, refs[i], False, paged=True))

    pool = [threading.Thread(target=worker, args=(i,)) for i in range(4)]
    for t in pool:
        t.start()
    for t in pool:
        t.join()
    assert len(errors) == 80 and all(err <= tol for err, tol in errors)


@pytest.mark.parametrize("dtype", cases.DTYPES)
@pytest.mark.parametrize("page", [16, 32])
def test_reshape_and_cache(dtype, page):
    """reshape_and_cache writes the same cache an append does; negative slots
    skip; k/v may be chunks of a fused projection (test_kvcache.py:143-161).
    Bytes are compared exactly with the layout restatement."""
    C = _api()
    lens, h, d = [70, 5], 8, 64
    q, kc, vc, bt, ks, vs = stage(lens, h, d, page, dtype, seed=6)
    kc2, vc2 = torch.full_like(kc, float("nan")), torch.full_like(vc, float("nan"))
    kv = torch.cat([torch.cat([k[0], v[0]], -1) for k, v in zip(ks, vs)])  # [tokens, h, 2d]
    pos = torch.cat([torch.arange(n) for n in lens])
    seq = torch.cat([torch.full((n,), i) for i, n in enumerate(lens)])
    btc = bt.cpu()
    slots = btc[seq, pos // page].long() * page + pos % page
    kv = torch.cat([kv, torch.randn(3, h, 2 * d).to(dtype)]).to(DEV)  # 3 padding tokens, slot -1
    all_slots = torch.cat([slots, torch.full((3,), -1, dtype=torch.int64)]).to(DEV)
    C.reshape_and_cache(kv[..., :d], kv[..., d:], kc2, vc2, all_slots)
    assert np.array_equal(bits(kc2), bits(kc)) and np.array_equal(bits(vc2), bits(vc))
    seqlens = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = C.flash_attn_with_kvcache(q, kc2, vc2, cache_seqlens=seqlens, page_table=bt)
    ref = np.concatenate([F64.attention(q[i:i + 1], ks[i], vs[i], d ** -0.5) for i in range(len(lens))])
    err, tol = F64.check(out, ref, dtype == torch.bfloat16, paged=True)
    assert err <= tol


@pytest.mark.parametrize("dtype", cases.DTYPES)
@pytest.mark.parametrize("d", [32, 64, 128])
def test_store_bit_exact_against_layout(dtype, d):
    """The store kernel's bytes equal the numpy restatement of PageLayout
    (paged_attn.mojo:58-131), aligned (16-byte vectors) and unaligned rows."""
    from oracle import paged
    C = _api()
    g = torch.Generator().manual_seed(d)
    nb, h, page, n = 9, 4, 32, 100
    for offset in (0, 1):  # offset 1: rows not 16-byte aligned -> element path
        src = torch.randn(n, h * d * 2 + offset, generator=g).to(dtype)
        key = src[:, offset:offset + h * d].view(n, h, d)
        val = src[:, offset + h * d:offset + 2 * h * d].view(n, h, d)
        slots = torch.randperm(nb * page, generator=g)[:n].long()
        slots[::7] = -1
        kc = torch.zeros(nb, h, page, d, dtype=dtype, device=DEV)
        vc = torch.zeros_like(kc)
        C.reshape_and_cache(key.to(DEV), val.to(DEV), kc, vc, slots.to(DEV))
        kn = np.zeros((nb, h, page, d), np.uint16 if dtype == torch.bfloat16 else np.float32)
        vn = np.zeros_like(kn)
        kb, vb = bits(key), bits(val)
        paged.store(kn, vn, kb.view(kn.dtype), vb.view(vn.dtype), slots.numpy())
        assert np.array_equal(bits(kc), kn.view(bits(kc).dtype))
        assert np.array_equal(bits(vc), vn.view(bits(vc).dtype))


@pytest.mark.parametrize("seed", range(30))
def test_fuzz(seed):
    """30 seeds (test_kvcache.py:112-120): covered by the golden set as d_fuzz_*;
    here the same shapes against the C restatement with fresh random caches."""
    r = random.Random(1000 + seed)
    lens = [r.randint(0, 1100) for _ in range(r.randint(1, 6))]
    d = r.choice([32, 64, 128])
    h, page, dtype = r.choice([1, 4, 12]), r.choice([16, 32, 48, 64]), r.choice(cases.DTYPES)
    scale = r.choice([1.0, 0.5]) * d ** -0.5
    C = _api()
    q, kc, vc, bt, ks, vs = stage(lens, h, d, page, dtype, seed)
    seqlens = torch.tensor(lens, dtype=torch.int32, device=DEV)
    out = C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seqlens, page_table=bt, softmax_scale=scale)
    ref = np.concatenate([F64.attention(q[i:i + 1], ks[i], vs[i], scale) for i in range(len(lens))])
    err, tol = F64.check(out, ref, dtype == torch.bfloat16, paged=True)
    assert err <= tol


def _engine_case(dtype, B=32, H=16, E=128, page=16, maxlen=2047, seed=0, lo=17):
    """A cfg2-shaped cache filled through reshape_and_cache."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, maxlen + 1, (B,), generator=g, dtype=torch.int32)
    W = -(-(maxlen + 1) // page)
    nblocks = B * W
    perm = torch.randperm(nblocks, generator=g).to(torch.int32)
    bt = perm.view(B, W).contiguous()
    kc = torch.full((nblocks, H, page, E), float("nan"), dtype=dtype, device=DEV)
    vc = kc.clone()
    C = _api()
    for i in range(B):
        n = int(lens[i])
        pos = torch.arange(n)
        slots = (bt[i, pos // page].long() * page + pos % page).to(DEV)
        k = torch.randn(n, H, E, generator=g).to(dtype).to(DEV)
        v = torch.randn(n, H, E, generator=g).to(dtype).to(DEV)
        C.reshape_and_cache(k, v, kc, vc, slots)
    q = torch.randn(B, 1, H, E, generator=g).to(dtype).to(DEV)
    return q, kc, vc, bt.to(DEV), lens.to(DEV)


@pytest.mark.parametrize("dtype", cases.DTYPES)
def test_cfg2_scale_against_cpu_restatement(dtype):
    """BASELINE config 2 at full size (B=32 H=16 E=128 page 16, lengths 17..2047,
    one appended token) against the C restatement: exercises split pieces and
    their merge on many sequences."""
    C = _api()
    q, kc, vc, bt, lens = _engine_case(dtype)
    g = torch.Generator().manual_seed(99)
    kn, vn = (torch.randn(32, 1, 16, 128, generator=g).to(dtype).to(DEV) for _ in range(2))
    ref = cpu_reference(q, kc, vc, bt, lens, k_new=kn, v_new=vn)
    out = C.flash_attn_with_kvcache(q, kc, vc, k=kn, v=vn, cache_seqlens=lens, page_table=bt)
    err, tol = north_star_ok(out[:, 0], ref, dtype)
    assert err <= tol, err
    # idempotent: the same call again (the append rewrites the same slot)
    out2 = C.flash_attn_with_kvcache(q, kc, vc, k=kn, v=vn, cache_seqlens=lens, page_table=bt)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("dtype", cases.DTYPES)
def test_engine_route_slots_and_out(dtype):
    """The engine's direct call (examples/ops.py:19-31): store at slot_mapping
    (some -1), lens after the store, preallocated out, 3-D q."""
    from cpu_attention import _kernel as K
    q, kc, vc, bt, lens = _engine_case(dtype, B=8, H=4, E=64, page=16, maxlen=600, seed=5)
    g = torch.Generator().manual_seed(5)
    B, H, E, page = 8, 4, 64, 16
    kn, vn = (torch.randn(B, H, E, generator=g).to(dtype).to(DEV) for _ in range(2))
    btc, lc = bt.cpu(), lens.cpu()
    slots = torch.tensor([int(btc[i, int(lc[i]) // page]) * page + int(lc[i]) % page for i in range(B)])
    slots[2] = -1  # padding: nothing stored, and lens[2] stays
    after = lc.clone()
    after[[i for i in range(B) if i != 2]] += 1
    out = torch.empty(B, H, E, dtype=dtype, device=DEV)
    ref = cpu_reference(q[:, 0], kc, vc, bt, after, k_new=kn, v_new=vn, slots=slots)
    got = K.module().decode(K.runtime(), q[:, 0], kc, vc, kn, vn, slots.to(DEV), after.to(DEV), bt, None, out)
    assert got is out
    err, tol = north_star_ok(out, ref, dtype)
    assert err <= tol
    # cross-attention: no store, pre-staged cache
    out2 = K.module().decode(K.runtime(), q[:, 0], kc, vc, None, None, None, after.to(DEV), bt, 0.1, None)
    ref2 = cpu_reference(q[:, 0], kc, vc, bt, after, scale=0.1)
    err, tol = north_star_ok(out2, ref2, dtype)
    assert err <= tol


@pytest.mark.parametrize("dtype", cases.DTYPES)
def test_engine_step_replayed_from_a_cuda_graph(dtype):
    """The engine's per-layer step (reshape_and_cache, then decode into a
    preallocated out; examples/ops.py:19-31) captured once in a CUDA graph and
    replayed with fresh inputs copied into the captured tensors: every replay's
    output and caches equal those of the same calls made eagerly, bit for bit
    (neither call synchronises with the host, so the step can be captured)."""
    from cpu_attention import _kernel as K
    C = _api()
    B, H, E, page = 8, 4, 128, 16
    q, kc, vc, bt, lens = _engine_case(dtype, B=B, H=H, E=E, page=page, maxlen=900, seed=11)
    btc, lc = bt.cpu(), lens.cpu()
    slots = torch.tensor([int(btc[i, int(lc[i]) // page]) * page + int(lc[i]) % page for i in range(B)]).to(DEV)
    after = (lc + 1).to(DEV)
    kn = torch.empty(B, H, E, dtype=dtype, device=DEV)
    vn, q3 = torch.empty_like(kn), torch.empty_like(kn)
    out = torch.empty(B, H, E, dtype=dtype, device=DEV)
    kc_ref, vc_ref = kc.clone(), vc.clone()

    def step(kcache, vcache, dst):
        C.reshape_and_cache(kn, vn, kcache, vcache, slots)
        return K.module().decode(K.runtime(), q3, kcache, vcache, None, None, None, after, bt, None, dst)

    g = torch.Generator().manual_seed(12)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up on the capture stream (its workspace)
        for t in (kn, vn, q3):
            t.copy_(torch.randn(B, H, E, generator=g).to(dtype))
        step(kc.clone(), vc.clone(), torch.empty_like(out))
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step(kc, vc, out)
    for _ in range(3):
        for t in (kn, vn, q3):
            t.copy_(torch.randn(B, H, E, generator=g).to(dtype))
        graph.replay()
        ref = step(kc_ref, vc_ref, None)
        torch.cuda.synchronize()
        assert np.array_equal(bits(out), bits(ref))
        assert np.array_equal(bits(kc), bits(kc_ref)) and np.array_equal(bits(vc), bits(vc_ref))
    err, tol = north_star_ok(out, cpu_reference(q3, kc, vc, bt, after), dtype)
    assert err <= tol
    del graph


def test_device_value_errors_are_flagged_not_faulted():
    """Lengths past the page table and table entries past the cache are caught on
    the device (no out-of-bounds access) and raised by raise_status()."""
    from cpu_attention import _kernel as K
    C = _api()
    q = torch.randn(2, 1, 4, 64, device=DEV)
    kc = torch.zeros(4, 4, 16, 64, device=DEV)
    bt = torch.arange(4, dtype=torch.int32, device=DEV).view(2, 2)
    K.status()  # clear
    C.flash_attn_with_kvcache(q, kc, kc.clone(), cache_seqlens=torch.tensor([5, 40], dtype=torch.int32,
                                                                             device=DEV), page_table=bt)
    with pytest.raises(ValueError, match="capacity"):
        K.raise_status()
    bad = bt.clone()
    bad[1, 0] = 99
    C.flash_attn_with_kvcache(q, kc, kc.clone(), cache_seqlens=torch.tensor([5, 9], dtype=torch.int32,
                                                                            device=DEV), page_table=bad)
    with pytest.raises(ValueError, match="page_table"):
        K.raise_status()
    assert K.status() == 0
