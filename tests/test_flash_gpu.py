"""flash_attn_func (dense prefill) on the B200, through the C ABI, against the
golden outputs of the reference's float64 oracle (the reference's gates:
fp32 2e-4, bf16 3e-2, `tests/reference.py:24-40`) and the C restatement of the
reference's CPU kernel (bf16 max-abs <= 2e-2, fp32 <= 1e-4 relative). Mirrors
`tests/test_flash.py` of the reference."""

import random

import pytest
import torch

import cases
from helpers import golden, north_star_ok
from oracle import attention_f64 as F64
from oracle import cpu as ORACLE

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _flash(q, k, v, **kw):
    import cpu_attention
    return cpu_attention.flash_attn_func(q, k, v, **kw)


def cpu_flash(q, k, v, scale=None, causal=False):
    out = torch.empty(q.shape, dtype=q.dtype)
    ORACLE.flash(q.cpu(), k.cpu(), v.cpu(), out, scale=scale, causal=causal)
    return out


def run(b, sq, sk, h, d, dtype, causal, seed, scale=None, ref=None):
    q, k, v = cases.flash_inputs(b, sq, sk, h, d, dtype, seed)
    out = _flash(q.to(DEV), k.to(DEV), v.to(DEV), softmax_scale=scale, causal=causal)
    assert out.shape == q.shape and out.dtype == dtype and out.is_contiguous()
    if ref is None:
        ref = F64.attention(q, k, v, scale or d ** -0.5, causal)
    err, tol = F64.check(out, ref, dtype == torch.bfloat16)
    assert err <= tol, err
    err, tol = north_star_ok(out, cpu_flash(q, k, v, scale, causal), dtype)
    assert err <= tol, err
    return out


@pytest.mark.parametrize("case", cases.flash_cases(), ids=lambda c: c[0])
def test_flash_golden(case):
    name, b, sq, sk, h, d, dtype, causal, seed, scale = case
    run(b, sq, sk, h, d, dtype, causal, seed, scale, ref=golden("flash")[name])


@pytest.mark.parametrize("dtype", cases.DTYPES)
@pytest.mark.parametrize("d", [32, 64, 128])
@pytest.mark.parametrize("sq,sk", cases.LENGTHS)
@pytest.mark.parametrize("h", [1, 8])
@pytest.mark.parametrize("causal", [True, False])
def test_shapes(dtype, d, sq, sk, h, causal):
    """test_flash.py:63-70, every shape."""
    run(1, sq, sk, h, d, dtype, causal, seed=sq * 1000 + sk)


@pytest.mark.parametrize("dtype", cases.DTYPES)
def test_batch_and_scale(dtype):
    run(3, 70, 150, 8, 64, dtype, True, seed=1, scale=0.07)


@pytest.mark.parametrize("dtype", cases.DTYPES)
def test_fused_qkv_strides(dtype):
    """q/k/v as chunks of one [b, s, 3*h*d] projection (no copy is needed)."""
    b, s, h, d = 2, 200, 4, 64
    qkv = torch.randn(b, s, 3 * h * d, generator=torch.Generator().manual_seed(2)).to(dtype).to(DEV)
    q, k, v = (qkv[..., i * h * d:(i + 1) * h * d].view(b, s, h, d) for i in range(3))
    out = _flash(q, k, v, causal=True)
    err, tol = F64.check(out, F64.attention(q, k, v, d ** -0.5, True), dtype == torch.bfloat16)
    assert err <= tol


@pytest.mark.parametrize("seed", range(40))
def test_fuzz(seed):
    r = random.Random(seed)
    run(r.randint(1, 3), r.randint(1, 900), r.randint(1, 900), r.choice([1, 4, 12]),
        r.choice([32, 64, 128]), r.choice(cases.DTYPES), r.random() < 0.5, seed)


def test_repeated_calls_follow_changes():
    """Repeated calls follow every change of scale, causal and shape."""
    for scale, causal, s in ((0.05, True, 64), (0.125, False, 64), (0.05, False, 65)):
        run(1, s, s, 4, 64, torch.float32, causal, seed=s, scale=scale)


@pytest.mark.parametrize("causal", [True, False])
def test_cfg4_shape_fused_views(causal):
    """BASELINE config 4's layout (q/k/v strided views into one fused
    [N, L, 3, H, E] tensor, token stride 3*H*E) at a reduced N*H, against the
    float64 oracle."""
    N, L, H, E = 1, 1024, 4, 128
    qkv = torch.randn(N, L, 3, H, E, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(DEV)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    if not causal:
        q = q[:, :256]
    out = _flash(q, k, v, causal=causal)
    err, tol = F64.check(out, F64.attention(q, k, v, E ** -0.5, causal), True)
    assert err <= tol
