"""Makes the golden fixtures from the reference's own float64 oracle.

    python tests/golden/make_golden.py /path/to/cpu-attention   # the reference checkout

Imports ``tests/reference.py`` of ducviet00/cpu-attention (pure torch float64:
the oracle its own test suite gates against, `tests/reference.py:7-40`), runs it
on the seeded inputs of ``tests/cases.py`` and writes

* ``golden_flash.npz``: per flash case, the float64 output and an input digest;
* ``golden_decode.npz``: per decode case, the float64 output of every sequence
  (the reference's ``test_kvcache.reference``) and an input digest;
* ``golden_ext.npz``: the same for the grouped-head (GQA/MQA) prefill and
  decode cases and the packed-sequence (varlen) prefill cases, which the
  reference declines: its MHA oracle runs on K/V heads repeated to the query
  heads (``cases.expand_kv``), and per sequence for varlen; stored as float32
  (its rounding, <= 6e-8 here, is far inside the tightest gate, 1e-6).

The reference's Mojo kernel itself cannot be built in this container (no Mojo
toolchain), so these outputs -- the reference's own oracle on the reference's
own test inputs -- are what the restatements under ``oracle/`` are pinned to.
Only this script reads the reference; the fixtures travel, the reference does not.
"""

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import cases  # noqa: E402


def load_reference_oracle(root):
    path = os.path.join(root, "tests", "reference.py")
    spec = importlib.util.spec_from_file_location("ref_oracle", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(root):
    ref = load_reference_oracle(root)
    flash = {}
    for name, b, sq, sk, h, d, dtype, causal, seed, scale in cases.flash_cases():
        q, k, v = cases.flash_inputs(b, sq, sk, h, d, dtype, seed)
        out = ref.attention(q, k, v, scale or d ** -0.5, causal)
        flash[name] = out.numpy()
        flash[name + "__digest"] = np.array(cases.digest(q, k, v))
    np.savez_compressed(os.path.join(HERE, "golden_flash.npz"), **flash)
    dec = {}
    for name, lens, h, d, page, dtype, seed, scale in cases.decode_cases():
        q, bt, total, ks, vs = cases.stage_inputs(lens, h, d, page, dtype, seed)
        out = torch.cat([ref.attention(q[i:i + 1], k, v, scale or d ** -0.5) for i, (k, v) in
                         enumerate(zip(ks, vs))])
        dec[name] = out.numpy()
        dec[name + "__digest"] = np.array(cases.digest(q, bt, *ks, *vs))
    np.savez_compressed(os.path.join(HERE, "golden_decode.npz"), **dec)
    print(f"{len(flash) // 2} flash cases, {len(dec) // 2} decode cases")
    # grouped heads and packed sequences: the reference's MHA oracle on K/V
    # heads repeated to the query heads, and one call per sequence
    ext = {}
    for name, b, sq, sk, h, hk, d, dtype, causal, seed in cases.gqa_flash_cases():
        q, k, v = cases.gqa_flash_inputs(b, sq, sk, h, hk, d, dtype, seed)
        out = ref.attention(q, cases.expand_kv(k, h), cases.expand_kv(v, h), d ** -0.5, causal)
        ext[name] = out.float().numpy()
        ext[name + "__digest"] = np.array(cases.digest(q, k, v))
    for name, lens, h, hk, d, page, dtype, seed, scale in cases.gqa_decode_cases():
        q, bt, total, ks, vs = cases.gqa_stage_inputs(lens, h, hk, d, page, dtype, seed)
        out = torch.cat([ref.attention(q[i:i + 1], cases.expand_kv(k, h), cases.expand_kv(v, h), scale or d ** -0.5)
                         for i, (k, v) in enumerate(zip(ks, vs))])
        ext[name] = out.float().numpy()
        ext[name + "__digest"] = np.array(cases.digest(q, bt, *ks, *vs))
    for name, lq, lk, h, hk, d, dtype, causal, seed in cases.varlen_cases():
        q, k, v, cq, ck = cases.varlen_inputs(lq, lk, h, hk, d, dtype, seed)
        parts = []
        for i in range(len(lq)):
            qi = q[int(cq[i]):int(cq[i + 1])][None]
            ki, vi = (cases.expand_kv(x[int(ck[i]):int(ck[i + 1])], h)[None] for x in (k, v))
            if qi.shape[1] == 0:
                continue
            if ki.shape[1] == 0:  # no keys: every row sees nothing and is 0 (`tests/reference.py:20`)
                parts.append(torch.zeros(qi.shape[1:], dtype=torch.float64))
                continue
            parts.append(ref.attention(qi, ki, vi, d ** -0.5, causal)[0])
        ext[name] = torch.cat(parts).float().numpy()
        ext[name + "__digest"] = np.array(cases.digest(q, k, v, cq, ck))
    np.savez_compressed(os.path.join(HERE, "golden_ext.npz"), **ext)
    print(f"{len(ext) // 2} grouped-head and varlen cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/cpu-attention")
    main(sys.argv[1])
