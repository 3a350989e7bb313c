"""Benchmark of the B200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2]
                    [--also cfg4,cfg5] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N ...

Workloads (all inputs are seeded synthetic N(0,1) data
of the config's shapes; the reference uses no dataset):

* cfg2  paged self-attention decode: flash_attn_with_kvcache, bf16, B=32 H=16
        E=128 page 16, cache_seqlens uniform in [17, 2047], page_table
        [32, 128] over a seeded permutation of 4096 distinct blocks, one
        appended token. The headline line. N GPUs: each rank decodes its own
        32 sequences (sharded by sequence, weak scaling; no collective).
* cfg3  cross-attention decode (no append), fp32, B=64 H=8 E=64 page 32, 1500
        tokens per sequence in a shuffled block order (cfg3e32: head_dim 32).
* cfg5  engine decode: B=256 H=32 E=128 page 16, lens uniform in [1, 8191],
        a shared pool of sum(ceil((len + 1) / 16)) blocks (room for each new
        token) in a seeded order; per step reshape_and_cache of 256 tokens
        (~5% slot -1) then decode with a preallocated out; sequences sharded
        over ranks in contiguous ranges balanced on context + 16 (strong
        scaling), with and without the output all-gather.
* cfg1  prefill: flash_attn_func bf16 N=1 L=S=128 H=16 E=64 causal, q/k/v from
        torch.manual_seed(0).
* cfg4  prefill: bf16 N=4 L=S=2048 H=32 E=128 causal, q/k/v strided views of a
        fused [N, L, 3, H, E] tensor (cfg4nc: L=512 S=2048 non-causal).

The line is the --workload's record (default cfg2, the config the metric is
quoted on), plus ``also``: the same record for each --also workload (default
cfg4 and cfg5, so one run measures decode, prefill and the engine config).

A step is one call of the hot path over the workload's batch, inputs resident
in HBM; L2 is flushed (a 256 MiB write) before every timed step and the step
alone is timed with CUDA events on the launching stream; the max over ranks is
taken. ``e2e`` is the same metric through the public API with the step's
inputs copied from pinned host memory and the output read back inside the
timed region. ``roofline`` times the dominant kernel alone. ``cpu_baseline``
times the C restatement of the reference's CPU kernel (``oracle/``) on the
host's physical cores on a bounded sample, caches flushed (a write sweep of
twice the LLC) before each call, median. ``--impl reference`` times that CPU
path as the reference arm, staged on the host alone (rank 0 only).
"""

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "cpu-attention_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

FLUSH_BYTES = 256 << 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
CPU_BUDGET_S = 10.0  # wall time of one cpu_baseline (after its warm-up)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ host cores --
def physical_cores():
    """Physical cores visible to this process, from the sysfs topology (the
    reference's thread count, `cpu_attention/_kernel.py:92-104`)."""
    cores = set()
    try:
        for cpu in range(os.cpu_count() or 1):
            base = f"/sys/devices/system/cpu/cpu{cpu}/topology"
            with open(f"{base}/core_id") as f, open(f"{base}/physical_package_id") as g:
                cores.add((g.read().strip(), f.read().strip()))
    except OSError:
        cores = set()
    return len(cores) or (os.cpu_count() or 1)


def llc_bytes():
    """The last-level cache size from sysfs, 32 MiB if unknown
    (`cpu_attention/_kernel.py:106-117`)."""
    for idx in (3, 2, 1, 0):
        try:
            with open(f"/sys/devices/system/cpu/cpu0/cache/index{idx}/size") as f:
                text = f.read().strip()
        except OSError:
            continue
        unit = {"K": 1 << 10, "M": 1 << 20}.get(text[-1], 1)
        return int(text.rstrip("KM")) * unit
    return 32 << 20


class HostFlush:
    """A write sweep of twice the LLC before each CPU call
    (`benchmarks/bench.py:112-127`, `:234`)."""

    def __init__(self):
        torch.set_num_threads(physical_cores())
        self.buf = torch.zeros(2 * llc_bytes() // 4, dtype=torch.int32)

    def __call__(self):
        self.buf.add_(1)


def time_cpu(fn, flush, warmup, max_calls, budget_s):
    """Median seconds of fn over up to max_calls calls within budget_s, after
    `warmup` calls; caches flushed before every call."""
    for _ in range(warmup):
        flush()
        fn()
    times = []
    t_start = time.perf_counter()
    while len(times) < max_calls and (not times or time.perf_counter() - t_start < budget_s):
        flush()
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


# ------------------------------------------------------------------ workloads --
def _pool(lens, page, extra, g):
    """Page table over a shared pool of sum(ceil((len + extra) / page)) blocks
    in a seeded order; padding entries stay 0."""
    npages = [-(-(int(n) + extra) // page) for n in lens]
    nblocks = max(1, sum(npages))
    perm = torch.randperm(nblocks, generator=g).to(torch.int32)
    bt = torch.zeros(len(lens), max(npages) if npages else 1, dtype=torch.int32)
    s = 0
    for i, n in enumerate(npages):
        bt[i, :n] = perm[s:s + n]
        s += n
    return bt, nblocks


class DecodeSpec:
    """The host-side plan of a decode workload: lengths, page table, slots."""

    def __init__(self, name, label, dtype, B, H, E, page, lens_fn, append, engine=False, width=None, kv_heads=None):
        self.name, self.label, self.dtype = name, label, dtype
        self.B_all, self.H, self.E, self.page, self.append, self.engine = B, H, E, page, append, engine
        self.Hk = kv_heads or H  # the caches' heads (fewer than H: grouped query heads)
        self.lens_fn, self.width = lens_fn, width

    def plan(self, rank, world):
        g = torch.Generator().manual_seed(1234)
        lens_all = self.lens_fn(g).to(torch.int32)  # the global batch (the same on every rank)
        if self.engine:  # strong scaling: this rank's contiguous, cost-balanced share
            ranges = shard_ranges(lens_all, world)
            lo, hi = ranges[rank]
            self.counts = [b - a for a, b in ranges]
            lens = lens_all[lo:hi]
        else:  # weak scaling: every rank has the full per-GPU batch
            self.counts = [len(lens_all)] * world
            lens = lens_all
        self.global_batch = len(lens_all) * (1 if self.engine else world)
        self.lens = lens.contiguous()
        self.B = len(lens)
        gp = torch.Generator().manual_seed(4321 + rank)
        if self.width:  # a fixed-width table over distinct blocks (B * width of them)
            self.nblocks = self.B * self.width
            self.bt = torch.randperm(self.nblocks, generator=gp).to(torch.int32).view(self.B, self.width).contiguous()
        else:
            self.bt, self.nblocks = _pool(self.lens, self.page, 1 if (self.append or self.engine) else 0, gp)
        extra = 1 if self.append else 0
        if self.engine:
            # one new token per sequence at its current length, ~5% padding (-1)
            ls = [int(n) for n in self.lens]
            slots = torch.tensor([int(self.bt[i, ls[i] // self.page]) * self.page + ls[i] % self.page
                                  for i in range(self.B)], dtype=torch.int64)
            slots[torch.rand(self.B, generator=gp) < 0.05] = -1
            self.slots = slots
            self.after = (self.lens + (slots >= 0).to(torch.int32)).contiguous()  # lengths after the store
            self.attended = [int(n) for n in self.after]
        else:
            self.attended = [int(n) + extra for n in self.lens]
        self.kv_bytes = sum(self.attended) * self.Hk * self.E * self.dtype.itemsize * 2
        # token slots of the pre-filled cache (contiguous per sequence)
        seq = torch.cat([torch.full((int(n),), i, dtype=torch.int64) for i, n in enumerate(self.lens)]) \
            if self.B else torch.zeros(0, dtype=torch.int64)
        pos = torch.cat([torch.arange(int(n)) for n in self.lens]) if self.B else torch.zeros(0, dtype=torch.int64)
        self.fill_slots = self.bt[seq, pos // self.page].long() * self.page + pos % self.page
        return self

    def config(self, world):
        lens = [int(n) for n in self.lens]
        c = {"workload": self.label, "global_batch": self.global_batch, "batch_per_gpu": self.B, "heads": self.H,
             "kv_heads": self.Hk, "head_dim": self.E, "page": self.page, "mean_len": round(sum(lens) / max(1, len(lens)), 1),
             "append": self.append, "num_blocks": self.nblocks, "table_width": int(self.bt.shape[1]),
             "parallelism": f"sequence-shard x{world}", "l2": "flushed (256 MiB write) before each step"}
        if self.engine:
            c["store_tokens"] = self.B
            c["store_skipped"] = int((self.slots < 0).sum())
        return c


class Decode:
    """A decode workload staged on the GPU (the caches written through the
    product's reshape_and_cache)."""

    kind = "decode"

    def __init__(self, spec, rank, dev):
        import cpu_attention as C
        from cpu_attention import _kernel as K

        self.C, self.K, self.s, self.dev = C, K, spec, dev
        s = spec
        self.dtype, self.B, self.H, self.E, self.page = s.dtype, s.B, s.H, s.E, s.page
        self.engine = s.engine
        self.kc = torch.empty(s.nblocks, s.Hk, s.page, s.E, dtype=s.dtype, device=dev)
        self.vc = torch.empty_like(self.kc)
        self.bt = s.bt.to(dev)
        self.lens = s.lens.to(dev)
        gd = torch.Generator(device=dev).manual_seed(99 + rank)
        for a in range(0, len(s.fill_slots), 65536):
            sl = s.fill_slots[a:a + 65536].to(dev)
            k = torch.randn(len(sl), s.Hk, s.E, generator=gd, device=dev, dtype=torch.float32).to(s.dtype)
            v = torch.randn(len(sl), s.Hk, s.E, generator=gd, device=dev, dtype=torch.float32).to(s.dtype)
            C.reshape_and_cache(k, v, self.kc, self.vc, sl)
        rnd = lambda *shape: torch.randn(*shape, generator=gd, device=dev, dtype=torch.float32).to(s.dtype)  # noqa
        if s.engine:
            self.q = rnd(s.B, s.H, s.E)
            self.kn, self.vn = rnd(s.B, s.Hk, s.E), rnd(s.B, s.Hk, s.E)
            self.slots = s.slots.to(dev)
            self.after = s.after.to(dev)
            self.out = torch.empty(s.B, s.H, s.E, dtype=s.dtype, device=dev)
        else:
            self.q = rnd(s.B, 1, s.H, s.E)
            self.kn = rnd(s.B, 1, s.Hk, s.E) if s.append else None
            self.vn = rnd(s.B, 1, s.Hk, s.E) if s.append else None
        self.attend_lens = torch.tensor(s.attended, dtype=torch.int32, device=dev)
        # engine: store + decode; a one-token append is fused into the decode
        self.launches_per_step = 2 if s.engine else 1
        torch.cuda.synchronize(dev)

    # the measured step (device-resident inputs)
    def step(self):
        if self.engine:
            self.C.reshape_and_cache(self.kn, self.vn, self.kc, self.vc, self.slots)
            K = self.K
            K.module().decode(K.runtime(), self.q, self.kc, self.vc, None, None, None, self.after, self.bt, None,
                              self.out)
            return self.out
        return self.C.flash_attn_with_kvcache(self.q, self.kc, self.vc, k=self.kn, v=self.vn, cache_seqlens=self.lens,
                                              page_table=self.bt)

    # the step followed by the optional collective: every rank's outputs
    # all-gathered in sequence order (NCCL all_gather_into_tensor)
    def gather_step(self):
        from cpu_attention.shard import gather_outputs
        out = self.step()
        return gather_outputs(out.reshape(out.shape[0], -1), self.s.counts)

    # the dominant kernel alone: decode over the attended lengths, no store
    def kernel_step(self):
        K = self.K
        q = self.q if self.q.dim() == 3 else self.q[:, 0]
        K.module().decode(K.runtime(), q, self.kc, self.vc, None, None, None, self.attend_lens, self.bt, None, None)

    def units(self):
        return self.s.kv_bytes

    kernel_units = units

    # end to end through the public API from pinned host buffers: the step's
    # inputs (query rows, new K/V rows, slots, lengths, page table) staged in
    # one pinned host buffer and sent with one copy into one device buffer,
    # as an engine stages them; the API reads views of it
    def e2e_setup(self):
        if self.engine:
            srcs = [self.q, self.kn, self.vn, self.slots, self.after, self.bt]
        else:
            srcs = [t for t in (self.q, self.kn, self.vn, self.lens, self.bt) if t is not None]
        offs, total = [], 0
        for t in srcs:
            offs.append(total)
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        self.h_buf = torch.empty(total, dtype=torch.uint8).pin_memory()
        self.d_buf = torch.empty(total, dtype=torch.uint8, device=self.dev)

        def view(buf, t, off):
            n = t.numel() * t.element_size()
            return buf[off:off + n].view(t.dtype).view(t.shape)

        views = []
        for t, off in zip(srcs, offs):
            view(self.h_buf, t, off).copy_(t.cpu())
            views.append(view(self.d_buf, t, off))
        self.d = views
        self.h_out = torch.empty(self.q.shape, dtype=self.dtype).pin_memory()
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in srcs)
        self.d2h_bytes = self.h_out.numel() * self.h_out.element_size()

    def e2e_step(self):
        self.d_buf.copy_(self.h_buf, non_blocking=True)
        if self.engine:
            q, kn, vn, slots, after, bt = self.d
            self.C.reshape_and_cache(kn, vn, self.kc, self.vc, slots)
            K = self.K
            out = K.module().decode(K.runtime(), q, self.kc, self.vc, None, None, None, after, bt, None, self.out)
        else:
            it = iter(self.d)
            q = next(it)
            kn = next(it) if self.kn is not None else None
            vn = next(it) if self.vn is not None else None
            lens, bt = next(it), next(it)
            out = self.C.flash_attn_with_kvcache(q, self.kc, self.vc, k=kn, v=vn, cache_seqlens=lens, page_table=bt)
        self.h_out.copy_(out, non_blocking=True)

    # the C restatement of the reference kernel on the host cores, on the
    # first `max_seqs` sequences (their pages gathered into a compact cache)
    def cpu_setup(self, max_seqs=64):
        s = self.s
        n = min(self.B, max_seqs)
        npg = [-(-a // s.page) for a in s.attended[:n]]
        W = max(npg)
        blocks = torch.cat([s.bt[i, :npg[i]].long() for i in range(n)])
        if self.engine:  # the store goes to the sequence's page at its length
            blocks = torch.unique(torch.cat([blocks, s.bt[:n].long().flatten()]))
        else:
            blocks = torch.unique(blocks)
        remap = torch.full((s.nblocks,), 0, dtype=torch.int32)
        remap[blocks] = torch.arange(len(blocks), dtype=torch.int32)
        self.c_bt = remap[s.bt[:n, :W].long()].contiguous()
        idx = blocks.to(self.dev)
        self.c_kc, self.c_vc = self.kc[idx].cpu(), self.vc[idx].cpu()
        q = self.q if self.q.dim() == 3 else self.q[:, 0]
        self.c_q = q[:n].cpu().contiguous()
        self.c_kn = self.kn.reshape(self.B, self.H, self.E)[:n].cpu().contiguous() if self.kn is not None else None
        self.c_vn = self.vn.reshape(self.B, self.H, self.E)[:n].cpu().contiguous() if self.vn is not None else None
        self.c_out = torch.empty(self.c_q.shape, dtype=self.dtype)
        if self.engine:
            sl = s.slots[:n]
            blk = torch.where(sl >= 0, remap[(sl.clamp(min=0) // s.page)].long(), torch.full_like(sl, -1))
            self.c_slots = torch.where(sl >= 0, blk * s.page + sl % s.page, sl).contiguous()
            self.c_lens = s.after[:n].contiguous()
        else:
            self.c_slots, self.c_lens = None, s.lens[:n].contiguous()
        self.cpu_units = sum(s.attended[:n]) * self.H * self.E * self.dtype.itemsize * 2
        self.cpu_sample = f"the first {n} of {self.B} sequences" if n < self.B else "the full workload"

    def cpu_step(self, threads):
        from oracle import cpu as ORACLE
        ORACLE.decode(self.c_q, self.c_kc, self.c_vc, self.c_lens, self.c_bt, self.c_out, k_new=self.c_kn,
                      v_new=self.c_vn, slots=self.c_slots, threads=threads)

    def config(self, world):
        return self.s.config(world)


class HostDecode(Decode):
    """The reference arm's decode workload, staged on the host alone: caches
    written by the oracle's restatement of the store (no device, none of the
    product's libraries), N(0,1) data from a CPU generator."""

    def __init__(self, spec):
        from oracle import cpu as ORACLE
        s = spec
        self.s, self.dtype, self.B, self.H, self.E, self.page, self.engine = s, s.dtype, s.B, s.H, s.E, s.page, \
            s.engine
        g = torch.Generator().manual_seed(99)
        self.c_kc = torch.empty(s.nblocks, s.H, s.page, s.E, dtype=s.dtype)
        self.c_vc = torch.empty_like(self.c_kc)
        for a in range(0, len(s.fill_slots), 65536):
            sl = s.fill_slots[a:a + 65536].contiguous()
            k = torch.randn(len(sl), s.H, s.E, generator=g).to(s.dtype)
            v = torch.randn(len(sl), s.H, s.E, generator=g).to(s.dtype)
            ORACLE.store(k, v, self.c_kc, self.c_vc, sl)
        self.c_q = torch.randn(s.B, s.H, s.E, generator=g).to(s.dtype)
        new = s.append or s.engine
        self.c_kn = torch.randn(s.B, s.H, s.E, generator=g).to(s.dtype) if new else None
        self.c_vn = torch.randn(s.B, s.H, s.E, generator=g).to(s.dtype) if new else None
        self.c_bt = s.bt
        self.c_slots = s.slots if s.engine else None
        self.c_lens = s.after if s.engine else s.lens
        self.c_out = torch.empty(s.B, s.H, s.E, dtype=s.dtype)
        self.cpu_units = s.kv_bytes
        self.cpu_sample = "the full workload per step"


class Prefill:
    """Dense prefill workloads (cfg1, cfg4, cfg4nc)."""

    kind = "prefill"

    def __init__(self, name, label, rank, world, dev, N, L, S, H, E, causal, fused):
        self.name, self.label, self.dev = name, label, dev
        self.N, self.L, self.S, self.H, self.E, self.causal, self.fused = N, L, S, H, E, causal, fused
        self.dtype = torch.bfloat16
        if fused:
            gd = torch.Generator(device=dev).manual_seed(7 + rank) if dev is not None else None
            self.qkv = torch.randn(N, S, 3, H, E, generator=gd, device=dev, dtype=torch.float32).to(self.dtype)
            self.q, self.k, self.v = self.qkv[:, S - L:, 0], self.qkv[:, :, 1], self.qkv[:, :, 2]
        else:
            torch.manual_seed(0)
            q, k, v = (torch.randn(N, n, H, E, dtype=self.dtype) for n in (L, S, S))
            self.q, self.k, self.v = (x.to(dev) if dev is not None else x for x in (q, k, v))
        pairs = sum(min(S, max(0, i + S - L + 1)) for i in range(L)) if causal else L * S
        self.flops = 4 * N * H * E * pairs
        self.global_batch = N * world
        self.launches_per_step = 1

    def step(self):
        import cpu_attention as C
        return C.flash_attn_func(self.q, self.k, self.v, causal=self.causal)

    kernel_step = step

    def units(self):
        return self.flops

    kernel_units = units

    def e2e_setup(self):
        # the step's inputs in one pinned host buffer, sent with one copy: the
        # fused [N, S, 3, H, E] tensor whose strided views q/k/v are (cfg4), or
        # q, k, v back to back (cfg1)
        srcs = (self.qkv,) if self.fused else (self.q, self.k, self.v)
        sizes = [t.numel() * t.element_size() for t in srcs]
        offs = [0]
        for n in sizes[:-1]:
            offs.append(offs[-1] + (n + 255) // 256 * 256)
        total = offs[-1] + (sizes[-1] + 255) // 256 * 256
        self.h_buf = torch.empty(total, dtype=torch.uint8).pin_memory()
        self.d_buf = torch.empty(total, dtype=torch.uint8, device=self.dev)
        dev_views = []
        for t, off, n in zip(srcs, offs, sizes):
            self.h_buf[off:off + n].view(t.dtype).view(t.shape).copy_(t.cpu())
            dev_views.append(self.d_buf[off:off + n].view(t.dtype).view(t.shape))
        if self.fused:
            qkv = dev_views[0]
            self.d = (qkv[:, self.S - self.L:, 0], qkv[:, :, 1], qkv[:, :, 2])
        else:
            self.d = tuple(dev_views)
        self.h_out = torch.empty(self.q.shape, dtype=self.dtype).pin_memory()
        self.h2d_bytes = sum(sizes)
        self.d2h_bytes = self.h_out.numel() * self.h_out.element_size()

    def e2e_step(self):
        import cpu_attention as C
        self.d_buf.copy_(self.h_buf, non_blocking=True)
        out = C.flash_attn_func(*self.d, causal=self.causal)
        self.h_out.copy_(out, non_blocking=True)

    def cpu_setup(self, max_seqs=None):
        # a bounded sample: the first heads of the first batch entry, one per
        # physical core
        nh = min(self.H, physical_cores())
        self.c = [t[:1, :, :nh].cpu() for t in (self.q, self.k, self.v)]
        self.c_out = torch.empty(self.c[0].shape, dtype=self.dtype)
        self.cpu_units = self.flops * nh / (self.N * self.H)
        self.cpu_sample = f"{nh} (batch, head) pairs of the workload"

    def cpu_step(self, threads):
        from oracle import cpu as ORACLE
        ORACLE.flash(*self.c, self.c_out, causal=self.causal, threads=threads)

    def config(self, world):
        return {"workload": self.label, "global_batch": self.global_batch, "seq_q": self.L, "seq_k": self.S,
                "heads": self.H, "head_dim": self.E, "causal": self.causal,
                "inputs": ("strided views of a fused [N, S, 3, H, E] tensor" if self.fused
                           else "contiguous, torch.manual_seed(0)"),
                "parallelism": f"batch-shard x{world}", "l2": "flushed (256 MiB write) before each step"}


def shard_ranges(lens, world):
    """Contiguous sequence ranges per rank, balanced on context + 16 (the
    reference's `_share` cost model, paged_attn.mojo:788-816)."""
    from cpu_attention.shard import balanced_ranges
    return balanced_ranges([int(n) for n in lens], world)


DECODE = {
    "cfg2": lambda: DecodeSpec("cfg2", "cfg2: flash_attn_with_kvcache bf16 B=32 H=16 E=128 page16 lens~U[17,2047] "
                               "+1 append", torch.bfloat16, 32, 16, 128, 16,
                               lambda g: torch.randint(17, 2048, (32,), generator=g), append=True, width=128),
    "cfg3": lambda: DecodeSpec("cfg3", "cfg3: cross-attention decode fp32 B=64 H=8 E=64 page32 len=1500 no append",
                               torch.float32, 64, 8, 64, 32, lambda g: torch.full((64,), 1500), append=False),
    "cfg3e32": lambda: DecodeSpec("cfg3e32", "cfg3e32: cross-attention decode fp32 B=64 H=8 E=32 page32 len=1500 "
                                  "no append", torch.float32, 64, 8, 32, 32, lambda g: torch.full((64,), 1500),
                                  append=False),
    # grouped query heads (GQA/MQA; the reference declines them): the bf16
    # cfg2 shape with 4 and 8 query heads per KV head, and one KV head
    "gqa4": lambda: DecodeSpec("gqa4", "gqa4: flash_attn_with_kvcache bf16 B=32 H=32 Hk=8 E=128 page16 lens~U[17,2047] "
                               "+1 append", torch.bfloat16, 32, 32, 128, 16,
                               lambda g: torch.randint(17, 2048, (32,), generator=g), append=True, width=128,
                               kv_heads=8),
    "gqa8": lambda: DecodeSpec("gqa8", "gqa8: flash_attn_with_kvcache bf16 B=32 H=64 Hk=8 E=128 page16 lens~U[17,2047] "
                               "+1 append", torch.bfloat16, 32, 64, 128, 16,
                               lambda g: torch.randint(17, 2048, (32,), generator=g), append=True, width=128,
                               kv_heads=8),
    "mqa": lambda: DecodeSpec("mqa", "mqa: flash_attn_with_kvcache bf16 B=128 H=32 Hk=1 E=128 page16 lens~U[17,2047] "
                              "+1 append", torch.bfloat16, 128, 32, 128, 16,
                              lambda g: torch.randint(17, 2048, (128,), generator=g), append=True, width=128,
                              kv_heads=1),
    "cfg5": lambda: DecodeSpec("cfg5", "cfg5: engine decode bf16 B=256 H=32 E=128 page16 lens~U[1,8191] "
                               "store+decode out=", torch.bfloat16, 256, 32, 128, 16,
                               lambda g: torch.randint(1, 8192, (256,), generator=g), append=False, engine=True),
}
PREFILL = {
    "cfg1": ("cfg1: flash_attn_func bf16 N=1 L=S=128 H=16 E=64 causal", 1, 128, 128, 16, 64, True, False),
    "cfg4": ("cfg4: flash_attn_func bf16 N=4 L=S=2048 H=32 E=128 causal fused-QKV views", 4, 2048, 2048, 32, 128,
             True, True),
    "cfg4nc": ("cfg4nc: flash_attn_func bf16 N=4 L=512 S=2048 H=32 E=128 non-causal fused-QKV views", 4, 512, 2048,
               32, 128, False, True),
}


def make_workload(name, rank, world, dev):
    if name in DECODE:
        return Decode(DECODE[name]().plan(rank, world), rank, dev)
    if name in PREFILL:
        label, *shape = PREFILL[name]
        return Prefill(name, label, rank, world, dev, *shape)
    raise SystemExit(f"unknown workload {name}")


# --------------------------------------------------------------------- timing --
class ClockSampler:
    """SM clocks and throttle reasons sampled during the run; each workload
    reads the samples of its own time window. NVML (read-only queries) from a
    background thread every 5 ms, so that even a timed region of a few
    milliseconds holds samples; `nvidia-smi -lms 50` when NVML is missing."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpus):
        self.proc = None
        self.path = None
        self.gpus = gpus
        self.thread = None
        self.samples = []  # (wall time, sm MHz, max sm MHz, reason names)

    def _nvml_loop(self, nv, handles, bits):
        reasons_of = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        maxes = [nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM) for h in handles]
        while not self.halt.is_set():
            t = time.time()
            for h, mx in zip(handles, maxes):
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    r = reasons_of(h)
                except nv.NVMLError:
                    continue
                self.samples.append((t, float(sm), float(mx), {n for n, b in bits if r & b}))
            self.halt.wait(0.005)

    def start(self):
        """Start sampling; returns once the first sample is in (at most ~5 s)."""
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            handles = [nv.nvmlDeviceGetHandleByIndex(g) for g in self.gpus]
            pre = "nvmlClocksEventReason" if hasattr(nv, "nvmlClocksEventReasonHwSlowdown") else "nvmlClocksThrottleReason"
            bits = [(n, getattr(nv, pre + k)) for n, k in zip(
                self.NAMES, ["HwSlowdown", "HwThermalSlowdown", "SwThermalSlowdown", "SwPowerCap"])]
            self.halt = threading.Event()
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, handles, bits), daemon=True)
            self.thread.start()
            self.nv = nv
            t0 = time.time()
            while not self.samples and time.time() - t0 < 5.0:
                time.sleep(0.01)
            return
        except Exception:  # no NVML: fall back to nvidia-smi
            self.thread = None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={','.join(str(g) for g in self.gpus)}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 5.0:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)

    def window(self, t0, t1):
        """Clocks of the samples taken in [t0, t1] (wall time, seconds)."""
        sm, mx, reasons = [], 0.0, set()
        if self.thread is not None:
            for t, s, m, rs in list(self.samples):
                if t0 <= t <= t1:
                    sm.append(s)
                    mx = max(mx, m)
                    reasons |= rs
        elif self.proc is not None:
            self.fh.flush()
            a, b = datetime.datetime.fromtimestamp(t0), datetime.datetime.fromtimestamp(t1)
            with open(self.path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) < 9:
                        continue
                    try:
                        ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                        if ts < a or ts > b:
                            continue
                        sm.append(float(parts[2]))
                        mx = max(mx, float(parts[3]))
                    except ValueError:
                        continue
                    for n, v in zip(self.NAMES, parts[5:9]):
                        if v.lower().startswith("active"):
                            reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml" if self.thread is not None else "nvidia-smi"}

    def stop(self):
        if self.thread is not None:
            self.halt.set()
            self.thread.join(timeout=5)
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass
            return
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        os.unlink(self.path)


# DRAM bytes (read + write) of one launch of the roofline kernel, from one ncu
# capture of the same workload (the files under profiles/ give the commands).
TRAFFIC = {
    "cfg2": (284.4e6, "profiles/decode_kernel_cfg2.md"),
    "cfg4": (556.8e6, "profiles/flash_tc_kernel_cfg4.md"),
}

HOST_HIDE_CYCLES = 400_000  # ~0.2 ms of device spin: longer than the host needs to enqueue one step


def timed(fn, steps, warmup, flush, stream, hide_host=True):
    """Per-step CUDA-event times (ms) on `stream`, L2 flushed before each step.

    With hide_host, a device-side spin follows the flush, so the device is
    still busy when the host has enqueued the step: the events then bracket
    the step's device work, not the host's enqueue latency (the e2e timing
    runs without it: there the host's share belongs to the number)."""
    for _ in range(warmup):
        flush()
        fn()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in evs:
        flush()
        if hide_host:
            torch.cuda._sleep(HOST_HIDE_CYCLES)
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def _reduce_device():
    import torch.distributed as dist
    return "cuda" if dist.get_backend() == "nccl" else "cpu"


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=_reduce_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=_reduce_device())
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def metric_of(wl):
    if wl.kind == "prefill":
        return "prefill bf16 TFLOP/s", "TFLOP/s", 1e12
    return "paged-decode KV GB/s", "GB/s", 1e9


def cpu_baseline(wl, flush, threads):
    """The oracle's C restatement of the reference kernel on the host's
    physical cores: 3 warm-up + up to 10 timed calls within ~CPU_BUDGET_S,
    caches flushed before each, median."""
    wl.cpu_setup()
    sec, n = time_cpu(lambda: wl.cpu_step(threads), flush, 3, 10, CPU_BUDGET_S)
    return sec, wl.cpu_units, n


def measure(wl, name, args, world, rank, sampler, flush_host):
    """One workload's record: the device-timed step, the roofline kernel, e2e,
    the N > 1 gather (decode), and at N = 1 the CPU baseline."""
    dev, stream = wl.dev, torch.cuda.current_stream(wl.dev)
    flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    flush = lambda: flush_buf.fill_(1)  # noqa: E731
    metric, unit, scale = metric_of(wl)
    barrier(world)
    t_begin = time.time()
    step_ms = timed(wl.step, args.steps, args.warmup, flush, stream)
    barrier(world)
    total_ms = max_over_ranks(sum(step_ms), world)
    units = sum_over_ranks(wl.units(), world)
    ms_per_step = total_ms / args.steps
    value = units / (ms_per_step * 1e-3) / scale

    # the dominant kernel alone (roofline)
    kern_ms = timed(wl.kernel_step, args.steps, 2, flush, stream)
    kern_avg = statistics.mean(kern_ms)
    pk, pk_kind = peaks()
    if wl.kind == "prefill":
        achieved = wl.kernel_units() / (kern_avg * 1e-3) / 1e12
        peak, bound, runit = pk["bf16_tflops"], "tensor", "TFLOP/s"
    else:
        achieved = wl.kernel_units() / (kern_avg * 1e-3) / 1e9
        peak, bound, runit = pk["hbm_gbs"], "hbm", "GB/s"
    achieved = -max_over_ranks(-achieved, world)  # the slowest rank
    roofline = {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "peak_kind": pk_kind, "unit": runit,
                "frac": round(achieved / peak, 4),
                "traffic": TRAFFIC[name][0] if name in TRAFFIC else None,
                "traffic_source": TRAFFIC[name][1] if name in TRAFFIC else None,
                "kernel_ms": round(kern_avg, 4)}

    # end to end through the public API, host buffers
    wl.e2e_setup()
    e2e_ms = timed(wl.e2e_step, args.steps, 2, flush, stream, hide_host=False)
    e2e_total = max_over_ranks(sum(e2e_ms), world)
    e2e_value = units / (e2e_total / args.steps * 1e-3) / scale

    # N > 1 decode: the same step with the output all-gather after it
    with_gather = None
    if world > 1 and wl.kind == "decode":
        g_ms = timed(wl.gather_step, args.steps, 2, flush, stream)
        g_total = max_over_ranks(sum(g_ms), world)
        with_gather = {"value": round(units / (g_total / args.steps * 1e-3) / scale, 3), "unit": unit,
                       "ms_per_step": round(g_total / args.steps, 4), "collective": "all_gather_into_tensor"}
    barrier(world)
    t_end = time.time()
    rec = {"metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "us_per_call": round(ms_per_step * 1e3, 2),
           "higher_is_better": True, "scaling": "strong" if getattr(wl, "engine", False) else "weak",
           "vs_baseline": None, "dtype": str(wl.dtype).split(".")[-1], "data": "synthetic",
           "config": wl.config(world), "roofline": roofline,
           "e2e": {"value": round(e2e_value, 3), "unit": unit, "h2d_bytes_per_step": wl.h2d_bytes,
                   "d2h_bytes_per_step": wl.d2h_bytes, "ms_per_step": round(e2e_total / args.steps, 4)},
           "gpu_launches": wl.launches_per_step * args.steps,
           "clocks": sampler.window(t_begin, t_end) if sampler else None}
    if with_gather is not None:
        rec["with_gather"] = with_gather
    grouped = getattr(getattr(wl, "s", None), "Hk", None) not in (None, getattr(wl, "H", None))
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not grouped:  # the C restatement is MHA only
        threads = physical_cores()
        sec, cunits, n = cpu_baseline(wl, flush_host, threads)
        rec["cpu_baseline"] = {"value": round(cunits / sec / scale, 4), "unit": unit, "cores": threads,
                               "kind": "port", "sample": f"{wl.cpu_sample}, median of {n} calls, caches flushed",
                               "ms_per_call": round(sec * 1e3, 3)}
    return rec


def run_reference(args):
    """The reference arm: the C restatement of the reference's CPU kernel
    (`oracle/`; the reference's own Mojo kernel cannot be built here), staged
    and timed on the host alone -- none of this repository's CUDA libraries is
    loaded -- on its physical cores, caches flushed before every call, the
    median of --steps calls after --warmup. Rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    if args.workload not in DECODE:
        label, *shape = PREFILL[args.workload]
        wl = Prefill(args.workload, label, 0, 1, None, *shape)
        wl.cpu_setup()
    else:
        spec = DECODE[args.workload]()
        if spec.engine:
            raise SystemExit("the reference arm stages cfg2/cfg3 decode and the prefill configs")
        if spec.Hk != spec.H:
            print(json.dumps({"impl": "reference", "unavailable": "the reference declines grouped query heads "
                              "(its kernel needs as many KV heads as query heads)"}), flush=True)
            return 0
        wl = HostDecode(spec.plan(0, 1))
    threads = physical_cores()
    flush = HostFlush()
    metric, unit, scale = metric_of(wl)
    sec, n = time_cpu(lambda: wl.cpu_step(threads), flush, args.warmup, args.steps, 1e9)
    value = wl.cpu_units / sec / scale
    line = {"impl": "reference", "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": str(wl.dtype).split(".")[-1],
            "data": "synthetic", "config": wl.config(1),
            "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": threads, "kind": "port",
                             "sample": f"{wl.cpu_sample}, median of {n} calls, caches flushed (2x LLC)"},
            "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="cfg2")
    ap.add_argument("--also", default="cfg4,cfg5", help="comma-separated workloads recorded under 'also' ('' none)")
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    also = [w for w in args.also.split(",") if w and w not in (args.workload, "none")]
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
    flush_host = HostFlush() if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    line = None
    records = {}
    for name in [args.workload] + also:
        wl = make_workload(name, rank, world, dev)
        rec = measure(wl, name, args, world, rank, sampler, flush_host)
        if line is None:
            line = rec
        else:
            records[name] = rec
        del wl
        torch.cuda.empty_cache()
    if sampler:
        sampler.stop()
    if records:
        line["also"] = records
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
