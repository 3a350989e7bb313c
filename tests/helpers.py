"""Helpers shared by the tests: golden fixtures and cache staging."""

import os

import numpy as np
import torch

import cases

HERE = os.path.dirname(os.path.abspath(__file__))
_GOLDEN = {}


def golden(kind):
    """The committed golden outputs (``flash`` or ``decode``), lazily loaded."""
    if kind not in _GOLDEN:
        _GOLDEN[kind] = dict(np.load(os.path.join(HERE, "golden", f"golden_{kind}.npz")))
    return _GOLDEN[kind]


def append_slots(bt, lens_before, n, page):
    """Slots of n tokens appended at lens_before (per sequence) through bt."""
    out = []
    for i, a in enumerate(lens_before):
        pos = torch.arange(a, a + n[i]) if isinstance(n, (list, tuple)) else torch.arange(a, a + n)
        out.append(bt[i, pos // page].long() * page + pos % page)
    return out


def stage_cache(lens, h, d, page, dtype, seed, store, device="cpu", gqa=None):
    """The reference's ``stage`` (test_kvcache.py:118-141): caches holding
    ``lens[i]`` random tokens per sequence, everything else NaN (unused slots and
    pages, and the page-table padding, which points at a poisoned page). Tokens
    are written with ``store(key, value, kc, vc, slots)`` in two halves per
    sequence, as the reference stages through two appends. ``gqa``: the number
    of KV heads (``cases.gqa_stage_inputs``), else every head has its own.

    Returns (q [B,1,h,d], kc, vc, bt, ks, vs) on ``device``.
    """
    if gqa is None:
        q, bt, total, ks, vs = cases.stage_inputs(lens, h, d, page, dtype, seed)
    else:
        q, bt, total, ks, vs = cases.gqa_stage_inputs(lens, h, gqa, d, page, dtype, seed)
    kc = torch.full((total, gqa or h, page, d), float("nan"), dtype=dtype, device=device)
    vc = kc.clone()
    for i, n in enumerate(lens):
        for a, z in ((0, n // 2), (n // 2, n)):
            if z > a:
                pos = torch.arange(a, z)
                slots = (bt[i, pos // page].long() * page + pos % page).to(device)
                store(ks[i][0, a:z].to(device), vs[i][0, a:z].to(device), kc, vc, slots)
    return q.to(device), kc, vc, bt.to(device), ks, vs


def bits(t):
    """A tensor's raw element bits as a numpy array (bf16 -> int16, fp32 -> int32)."""
    t = t.detach().to("cpu").contiguous()
    return t.view(torch.int16 if t.dtype == torch.bfloat16 else torch.int32).numpy()


def north_star_ok(got, ref_cpu, dtype):
    """The north-star tolerance against the CPU restatement of the reference
    kernel: bf16 max-abs <= 2e-2; fp32 <= 1e-4 relative (to the output's max
    magnitude, floored at 1)."""
    g = got.detach().to("cpu", torch.float64)
    r = ref_cpu.detach().to("cpu", torch.float64)
    err = (g - r).abs().max().item() if g.numel() else 0.0
    if dtype == torch.bfloat16:
        return err, 2e-2
    scale = max(1.0, r.abs().max().item() if r.numel() else 1.0)
    return err / scale, 1e-4
