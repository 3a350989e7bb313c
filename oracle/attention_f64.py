"""TEST INFRASTRUCTURE ONLY. The reference's float64 oracle, restated in numpy.

Follows ``tests/reference.py:7-21`` of ducviet00/cpu-attention (eager attention:
matmul, additive bottom-right causal mask, softmax with fully masked rows set to
0, matmul) and its gates ``check()`` (``tests/reference.py:24-40``).
"""

import numpy as np

try:  # torch tensors in, without making torch a hard dependency of the oracle
    import torch
except ImportError:  # pragma: no cover
    torch = None


def as_f64(x):
    """A torch tensor (any dtype, any device) or array as a float64 numpy array."""
    if torch is not None and isinstance(x, torch.Tensor):
        return x.detach().to("cpu", torch.float64).numpy()
    return np.asarray(x, dtype=np.float64)


def attention(q, k, v, scale, causal=False):
    """q [b, sq, h, d], k/v [b, sk, h, d] (MHA) -> float64 [b, sq, h, d].

    ``causal`` is bottom-right aligned (query i sees keys j <= i + sk - sq) and a
    row that sees no key is zero (`tests/reference.py:7-21`).
    """
    q, k, v = (as_f64(x).transpose(0, 2, 1, 3) for x in (q, k, v))  # [b, h, s, d]
    w = np.matmul(q, k.transpose(0, 1, 3, 2)) * scale
    sq, sk = q.shape[2], k.shape[2]
    if causal:
        mask = np.arange(sk)[None, :] > np.arange(sq)[:, None] + sk - sq
        w = np.where(mask, -np.inf, w)
    mx = w.max(axis=-1, keepdims=True, initial=-np.inf)
    with np.errstate(invalid="ignore"):
        e = np.exp(w - mx)
        p = e / e.sum(axis=-1, keepdims=True)
    p = np.nan_to_num(p, nan=0.0)  # a fully masked row is 0/0
    return np.ascontiguousarray(np.matmul(p, v).transpose(0, 2, 1, 3))


def logsumexp(q, k, v, scale, causal=False):
    """The softmax log-sum-exp of every row, float64 [b, h, sq]: ln of the sum
    over the keys row i sees of exp(scale * q_i . k_j), -inf for a row that sees
    none (flash-attn's softmax_lse; the reference computes no such output, so
    this follows the definition with the mask of `attention`). v is unused."""
    del v
    q, k = (as_f64(x).transpose(0, 2, 1, 3) for x in (q, k))
    w = np.matmul(q, k.transpose(0, 1, 3, 2)) * scale
    sq, sk = q.shape[2], k.shape[2]
    if causal:
        mask = np.arange(sk)[None, :] > np.arange(sq)[:, None] + sk - sq
        w = np.where(mask, -np.inf, w)
    mx = w.max(axis=-1, initial=-np.inf)
    safe = np.where(np.isfinite(mx), mx, 0.0)
    with np.errstate(divide="ignore"):
        return np.log(np.exp(w - safe[..., None]).sum(axis=-1)) + safe


def bf16_round(x):
    """float64 -> nearest bf16 (ties to even), back as float64."""
    f = np.asarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


def check(got, ref, bf16, paged=False):
    """Max error of ``got`` against the float64 ``ref``, and its limit
    (`tests/reference.py:24-40`): flash fp32 2e-4, bf16 3e-2; paged fp32 1e-6,
    bf16 1e-3 beyond the rounding of the exact result to bf16."""
    err = np.abs(as_f64(got) - ref)
    if not bf16:
        return float(err.max(initial=0.0)), (1e-6 if paged else 2e-4)
    if not paged:
        return float(err.max(initial=0.0)), 3e-2
    rounding = np.abs(ref - bf16_round(ref))
    return float((err - rounding).max(initial=0.0)), 1e-3
