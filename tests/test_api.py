"""What the kernel cannot do is rejected, never silently ignored (the reference's
`tests/test_api.py`, on CPU tensors: every rejection is decided on the host
before any device work, so these run without a GPU). Plus the C ABI itself:
the library loads and exports every symbol the header declares, and its
argument checks decline bad calls without touching a device."""

import ctypes
import os
import re

import pytest
import torch

import cpu_attention as C
from cpu_attention import _kernel as K

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def paged():
    q = torch.randn(2, 1, 4, 64)
    kc = torch.zeros(4, 4, 16, 64)
    return q, kc, kc.clone(), torch.arange(4, dtype=torch.int32).view(2, 2)


@pytest.mark.parametrize("kwargs", [
    dict(window_size=(8, 0)), dict(softcap=30.0), dict(attention_chunk=64), dict(rotary_cos=torch.ones(1)),
    dict(qv=torch.ones(1)), dict(alibi_slopes=torch.ones(4)), dict(window_size=[4, 4]),
    dict(cu_seqlens_q=torch.ones(1)), dict(k_descale=torch.ones(1)),
])
def test_kvcache_unsupported_options(kwargs):
    """The reference's list (`tests/test_api.py:15-24`) minus return_softmax_lse,
    which this build computes."""
    q, kc, vc, bt = paged()
    with pytest.raises(NotImplementedError):
        C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=4, page_table=bt, **kwargs)


@pytest.mark.parametrize("kwargs", [
    dict(window_size=[-1, -1]), dict(softcap=0), dict(attention_chunk=0), dict(num_splits=4), dict(pack_gqa=True),
    dict(scheduler_metadata=torch.ones(1)), dict(sm_margin=8), dict(causal=True), dict(rotary_interleaved=False),
])
def test_kvcache_inert_options_pass(kwargs):
    """Options at an inert value, or scheduling hints, are accepted: the call
    goes on to the device check (CPU tensors here)."""
    q, kc, vc, bt = paged()
    with pytest.raises(ValueError, match="CUDA"):
        C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=4, page_table=bt, **kwargs)


def test_kvcache_one_query_token_only():
    q, kc, vc, bt = paged()
    with pytest.raises(NotImplementedError):
        C.flash_attn_with_kvcache(q.expand(2, 3, 4, 64), kc, vc, cache_seqlens=4, page_table=bt)


@pytest.mark.parametrize("bad", ["dtype", "head_dim", "page", "heads", "no_table", "both_tables", "capacity"])
def test_kvcache_bad_arguments(bad):
    q, kc, vc, bt = paged()
    lens = 4
    if bad == "dtype":
        q = q.half()
    elif bad == "head_dim":
        q, kc, vc = q[..., :48], kc[..., :48].contiguous(), vc[..., :48].contiguous()
    elif bad == "page":
        kc, vc = kc[:, :, :8].contiguous(), vc[:, :, :8].contiguous()
    elif bad == "heads":
        q = q[:, :, :3]
    elif bad == "no_table":
        bt = None
    elif bad == "capacity":
        lens = torch.tensor([3, 33], dtype=torch.int32)  # 2 pages of 16 hold 32
    extra = dict(block_table=bt) if bad == "both_tables" else {}
    with pytest.raises(ValueError):
        C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=lens, page_table=bt, **extra)


def test_kvcache_cpu_tensors_are_refused():
    """A valid call on CPU tensors: this build computes only on CUDA tensors
    (no CPU fallback), and says so."""
    q, kc, vc, bt = paged()
    with pytest.raises(ValueError, match="CUDA"):
        C.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=4, page_table=bt)


@pytest.mark.parametrize("kv_heads", [2, 1])
def test_gqa_mqa_accepted(kv_heads):
    """Grouped heads are no longer refused (the reference raises
    NotImplementedError, `tests/test_api.py:52-59`): a call with nheads_k
    dividing nheads gets as far as the device check, and one whose nheads_k
    does not divide nheads is a ValueError."""
    q, kc, vc, bt = paged()
    kc = torch.zeros(4, kv_heads, 16, 64)
    with pytest.raises(ValueError, match="CUDA"):
        C.flash_attn_with_kvcache(q, kc, kc.clone(), cache_seqlens=4, page_table=bt)
    k = torch.randn(2, 8, kv_heads, 64)
    with pytest.raises(ValueError, match="CUDA"):
        C.flash_attn_func(torch.randn(2, 8, 4, 64), k, k)
    with pytest.raises(ValueError):
        C.flash_attn_func(torch.randn(2, 8, 3, 64), k, k)
    with pytest.raises(ValueError):
        C.flash_attn_with_kvcache(q[:, :, :3], kc, kc.clone(), cache_seqlens=4, page_table=bt)
    kn = torch.randn(2, 1, 4, 64)  # new tokens must carry nheads_k heads
    with pytest.raises(ValueError, match="k/v"):
        C.flash_attn_with_kvcache(q, kc, kc.clone(), k=kn, v=kn, cache_seqlens=4, page_table=bt)


@pytest.mark.parametrize("bad", ["dtype", "heads", "slots_dtype", "slots_len", "past_end"])
def test_reshape_and_cache_bad_arguments(bad):
    k = torch.randn(5, 2, 64)
    kc = torch.zeros(2, 2, 16, 64)
    slots = torch.arange(5)
    if bad == "dtype":
        k = k.bfloat16()
    elif bad == "heads":
        k = torch.randn(5, 3, 64)
    elif bad == "slots_dtype":
        slots = slots.int()
    elif bad == "slots_len":
        slots = slots[:4]
    elif bad == "past_end":
        slots = slots + 30
    with pytest.raises(ValueError):
        C.reshape_and_cache(k, k, kc, kc.clone(), slots)


@pytest.mark.parametrize("bad", ["dtype", "head_dim", "heads", "batch"])
def test_flash_bad_arguments(bad):
    q, k = torch.randn(2, 8, 4, 64), torch.randn(2, 8, 4, 64)
    if bad == "dtype":
        q, k = q.half(), k.half()
    elif bad == "head_dim":
        q, k = q[..., :48], k[..., :48]
    elif bad == "heads":
        q = q[:, :, :3]
    elif bad == "batch":
        k = k[:1]
    with pytest.raises(ValueError):
        C.flash_attn_func(q, k, k)


@pytest.mark.parametrize("bad", ["dims", "heads", "cu_dtype", "cu_len", "cu_order", "cu_past_end", "max"])
def test_varlen_bad_arguments(bad):
    q, k = torch.randn(10, 4, 64), torch.randn(12, 2, 64)
    cq, ck = torch.tensor([0, 4, 10], dtype=torch.int32), torch.tensor([0, 5, 12], dtype=torch.int32)
    mq, mk = 6, 7
    if bad == "dims":
        q = q[None]
    elif bad == "heads":
        k = torch.randn(12, 3, 64)
    elif bad == "cu_dtype":
        cq = cq.long()
    elif bad == "cu_len":
        ck = ck[:2]
    elif bad == "cu_order":
        cq = torch.tensor([0, 6, 4], dtype=torch.int32)
    elif bad == "cu_past_end":
        ck = torch.tensor([0, 5, 13], dtype=torch.int32)
    elif bad == "max":
        mq = 5  # the second sequence has 6 queries
    with pytest.raises(ValueError):
        C.flash_attn_varlen_func(q, k, k, cq, ck, mq, mk)


def test_varlen_valid_call_on_cpu_is_refused():
    q, k = torch.randn(10, 4, 64), torch.randn(12, 2, 64)
    cq, ck = torch.tensor([0, 4, 10], dtype=torch.int32), torch.tensor([0, 5, 12], dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        C.flash_attn_varlen_func(q, k, k, cq, ck, 6, 7, causal=True)


@pytest.mark.parametrize("fn", [C.flash_attn_qkvpacked_func, C.flash_attn_kvpacked_func,
                                C.flash_attn_varlen_qkvpacked_func,
                                C.flash_attn_varlen_kvpacked_func])
def test_not_ported(fn):
    with pytest.raises(NotImplementedError):
        fn(*[torch.zeros(1)] * 7)


def test_public_names_match_reference():
    assert set(C.__all__) == {"__version__", "flash_attn_func", "flash_attn_kvpacked_func",
                              "flash_attn_qkvpacked_func", "flash_attn_varlen_func",
                              "flash_attn_varlen_kvpacked_func", "flash_attn_varlen_qkvpacked_func",
                              "flash_attn_with_kvcache", "reshape_and_cache"}


# ---------------------------------------------------------------- the C ABI --
def header_symbols():
    text = open(os.path.join(ROOT, "include", "cpu_attention_b200.h")).read()
    return re.findall(r"CA_API\s+[\w\s\*]+?\b(ca_\w+)\s*\(", text)


def test_library_exports_every_header_symbol():
    lib = K.library()
    names = header_symbols()
    assert len(names) >= 7
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) <= set(K.SIGNATURES)
    assert lib.ca_build_info().decode().startswith("sm_100a")


def test_decode_fast_path_is_built_and_declines_cpu_tensors():
    """The C++ host path (decode, prefill, store) is built beside the kernel
    library, and it declines (None) what the Python path declines -- here, CPU tensors -- so
    the reference's checks still raise the precise errors."""
    if os.environ.get("CPU_ATTENTION_SO"):
        pytest.skip("another kernel library is selected")
    fast = K.fastpath()
    assert fast is not None
    q = torch.zeros(2, 1, 4, 64)
    lens, pt = torch.zeros(2, dtype=torch.int32), torch.zeros(2, 2, dtype=torch.int32)
    assert fast.decode(q, q, q, None, None, None, lens, pt, None, None) is None
    assert fast.flash(q, q, q, None, True) is None
    kv, cache = torch.zeros(3, 4, 64), torch.zeros(2, 4, 16, 64)
    assert fast.store(kv, kv, cache, cache, torch.zeros(3, dtype=torch.int64)) is None


def test_abi_declines_bad_arguments_without_a_device():
    """Argument checks run before any CUDA call."""
    lib = K.library()
    p = ctypes.c_void_p(16)
    args = dict(q=p, q_stride=256, kc=p, vc=p, nb=4, kn=None, vn=None, kvs=0, slots=None, lens=p, pt=p, w=2,
                out=p, b=2, h=4, e=64, page=16, dtype=0, scale=float("nan"), ws=p, wsb=1 << 20, stream=None)

    def dec(**kw):
        a = dict(args, **kw)
        return lib.ca_decode(a["q"], a["q_stride"], a["kc"], a["vc"], a["nb"], a["kn"], a["vn"], a["kvs"],
                             a["slots"], a["lens"], a["pt"], a["w"], a["out"], a["b"], a["h"], a["e"], a["page"],
                             a["dtype"], a["scale"], a["ws"], a["wsb"], a["stream"])

    assert dec(dtype=7) == K.EDTYPE
    assert dec(e=48) == K.EHEADDIM
    assert dec(page=8) == K.EPAGE
    assert dec(page=0) == K.EPAGE
    assert dec(kn=p) == K.ESHAPE  # k without v
    assert dec(slots=p) == K.ESHAPE  # slots without k/v (`_C.mojo:140-143`)
    assert dec(q=None) == K.ENULL
    assert dec(q_stride=100) == K.ELAYOUT
    assert dec(b=0) == K.OK  # nothing to do
    # the fused prompt append: n tokens per sequence at token stride ts,
    # sequence stride ss (`flash_attn_interface.py:109-117` in one launch)

    def app(n=3, ts=256, ss=768, kn=p, vn=p, **kw):
        a = dict(args, **kw)
        return lib.ca_decode_append(a["q"], a["q_stride"], a["kc"], a["vc"], a["nb"], kn, vn, ss, ts, n,
                                    a["lens"], a["pt"], a["w"], a["out"], a["b"], a["h"], a["e"], a["page"],
                                    a["dtype"], a["scale"], a["ws"], a["wsb"], a["stream"])

    assert app(n=0) == K.ESHAPE
    assert app(kn=None) == K.ESHAPE
    assert app(vn=None) == K.ESHAPE
    assert app(ts=100) == K.ELAYOUT  # tokens overlap (token stride < heads * dim)
    assert app(ss=512) == K.ELAYOUT  # sequences overlap (sequence stride < n * token stride)
    assert app(n=(1 << 20) + 1, ss=1 << 40) == K.ESHAPE
    assert app(dtype=7) == K.EDTYPE
    assert app(b=0) == K.OK
    st = (ctypes.c_int64 * 3)(0, 0, 0)
    assert lib.ca_flash(p, p, p, p, 1, 4, 4, 2, 48, st, st, st, 1.0, 1, 0, None, None) == K.EHEADDIM
    assert lib.ca_flash(p, p, p, p, 1, 0, 4, 2, 64, st, st, st, 1.0, 1, 0, None, None) == K.ESHAPE
    assert lib.ca_flash(p, p, p, p, 1, 4, 4, 2, 64, st, st, st, 1.0, 1, 3, None, None) == K.EDTYPE
    assert lib.ca_store(p, p, 128, p, p, 4, p, 3, 2, 64, 12, 0, None, None) == K.EPAGE
    assert lib.ca_store(p, p, 100, p, p, 4, p, 3, 2, 64, 16, 0, None, None) == K.ELAYOUT
    assert lib.ca_store(p, p, 128, p, p, 4, p, 0, 2, 64, 16, 0, None, None) == K.OK
