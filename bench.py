"""Benchmark of the B200 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2]
                    [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N ...

Workloads (the default, cfg2, is the one the metric is
quoted on; all inputs are seeded synthetic N(0,1) data of the config's shapes):

* cfg2  paged self-attention decode: flash_attn_with_kvcache, bf16, B=32 H=16
        E=128 page 16, cache_seqlens uniform in [17, 2047], one appended token.
        N GPUs: each rank decodes its own 32 sequences (sharded by sequence,
        weak scaling; no collective on the data path).
* cfg3  cross-attention decode (no append), fp32, B=64 H=8 E=64 page 32, 1500
        tokens per sequence (cfg3e32: head_dim 32).
* cfg5  engine decode: B=256 H=32 E=128 page 16, lens uniform in [1, 8191];
        per step reshape_and_cache of 256 tokens (~5% slot -1) then decode with a
        preallocated out; sequences sharded over ranks in contiguous ranges
        balanced on context + 16 (strong scaling).
* cfg1  prefill: flash_attn_func bf16 N=1 L=S=128 H=16 E=64 causal.
* cfg4  prefill: bf16 N=4 L=S=2048 H=32 E=128 causal, q/k/v strided views of a
        fused [N, L, 3, H, E] tensor (cfg4nc: L=512 S=2048 non-causal).

A step is one call of the hot path over the workload's batch, inputs resident
in HBM; L2 is flushed (a 256 MiB write) before every timed step and the step
alone is timed with CUDA events on the launching stream; the max over ranks is
taken. ``e2e`` is the same metric through the public API with the step's inputs
copied from pinned host memory and the output read back inside the timed
region. ``roofline`` times the dominant kernel alone. ``cpu_baseline`` times
the C restatement of the reference's CPU kernel (``oracle/``) on the host cores
on a bounded sample. ``--impl reference`` times that CPU path as the reference
arm (rank 0 only).
"""

import argparse
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


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ workloads --
class Decode:
    """Paged decode workloads (cfg2, cfg3, cfg5)."""

    def __init__(self, name, rank, world, dev, dtype, B, H, E, page, lens_fn, append, engine=False):
        import cpu_attention as C
        from cpu_attention import _kernel as K

        self.C, self.K = C, K
        self.name, self.dev, self.dtype = name, dev, dtype
        self.H, self.E, self.page, self.append, self.engine = H, E, page, append, engine
        g = torch.Generator().manual_seed(1234 + rank)
        lens_all = lens_fn(g)  # the global batch (same on every rank)
        if engine:  # strong scaling: this rank's contiguous, cost-balanced share
            lo, hi = shard_ranges(lens_all, world)[rank]
            lens = lens_all[lo:hi]
        else:  # weak scaling: every rank has the full per-GPU batch
            lens = lens_all
        self.global_batch = len(lens_all) * (1 if engine else world)
        self.lens_host = lens.to(torch.int32)
        B = len(lens)
        self.B = B
        extra = 1 if append else 0
        npages = [-(-(int(n) + extra) // page) for n in lens]
        W = max(npages) if npages else 1
        nblocks = max(1, sum(npages))
        perm = torch.randperm(nblocks, generator=g).to(torch.int32)
        bt = torch.zeros(B, W, dtype=torch.int32)
        s = 0
        for i, n in enumerate(npages):
            bt[i, :n] = perm[s:s + n]
            s += n
        self.bt_host = bt
        self.kc = torch.empty(nblocks, H, page, E, dtype=dtype, device=dev)
        self.vc = torch.empty_like(self.kc)
        self.bt = bt.to(dev)
        self.lens = self.lens_host.to(dev)
        gd = torch.Generator(device=dev).manual_seed(99 + rank)
        # pre-fill through reshape_and_cache from N(0,1) tokens, in chunks
        tok_seq = torch.cat([torch.full((int(n),), i, dtype=torch.int64) for i, n in enumerate(lens)]) \
            if B else torch.zeros(0, dtype=torch.int64)
        tok_pos = torch.cat([torch.arange(int(n)) for n in lens]) if B else torch.zeros(0, dtype=torch.int64)
        slots = (bt[tok_seq, tok_pos // page].long() * page + tok_pos % page)
        for a in range(0, len(slots), 65536):
            sl = slots[a:a + 65536].to(dev)
            k = torch.randn(len(sl), H, E, generator=gd, device=dev, dtype=torch.float32).to(dtype)
            v = torch.randn(len(sl), H, E, generator=gd, device=dev, dtype=torch.float32).to(dtype)
            C.reshape_and_cache(k, v, self.kc, self.vc, sl)
        self.q = torch.randn(B, 1, H, E, generator=gd, device=dev, dtype=torch.float32).to(dtype)
        if append:
            self.kn = torch.randn(B, 1, H, E, generator=gd, device=dev, dtype=torch.float32).to(dtype)
            self.vn = torch.randn(B, 1, H, E, generator=gd, device=dev, dtype=torch.float32).to(dtype)
        else:
            self.kn = self.vn = None
        if engine:
            # per step: 256 (global) new tokens, ~5% padding slots; this rank's share
            self.eng_k = torch.randn(B, H, E, generator=gd, device=dev, dtype=torch.float32).to(dtype)
            self.eng_v = torch.randn(B, H, E, generator=gd, device=dev, dtype=torch.float32).to(dtype)
            ls = [int(n) for n in lens]
            es = torch.tensor([int(bt[i, ls[i] // page]) * page + ls[i] % page if ls[i] // page < W else -1
                               for i in range(B)], dtype=torch.int64)
            drop = torch.rand(B, generator=g) < 0.05
            es[drop] = -1
            self.eng_slots = es.to(dev)
            # lens after the store: +1 where a token was stored (examples/ops.py:19-25)
            eng_lens = self.lens_host + (es >= 0).to(torch.int32)
            self.eng_lens = eng_lens.to(dev)
            self.out = torch.empty(B, H, E, dtype=dtype, device=dev)
            attended = [int(n) for n in eng_lens]
        else:
            attended = [int(n) + extra for n in lens]
        self.kv_bytes = sum(attended) * H * E * dtype.itemsize * 2
        self.attend_lens = torch.tensor(attended, dtype=torch.int32, device=dev)
        # engine: store + decode; a one-token append is fused into the decode
        self.launches_per_step = 2 if engine else 1
        self.counts = [b - a for a, b in shard_ranges(lens_all, world)] if engine else [B] * world

    # the measured step (device-resident inputs)
    def step(self):
        if self.engine:
            self.C.reshape_and_cache(self.eng_k, self.eng_v, self.kc, self.vc, self.eng_slots)
            K = self.K
            K.module().decode(K.runtime(), self.q[:, 0], self.kc, self.vc, None, None, None, self.eng_lens, self.bt,
                              None, self.out)
            return self.out
        return self.C.flash_attn_with_kvcache(self.q, self.kc, self.vc, k=self.kn, v=self.vn, cache_seqlens=self.lens,
                                              page_table=self.bt)

    # the step followed by the optional collective: every rank's outputs
    # all-gathered in sequence order (NCCL all_gather_into_tensor)
    def gather_step(self):
        from cpu_attention.shard import gather_outputs
        out = self.step()
        return gather_outputs(out.reshape(out.shape[0], -1), self.counts)

    # the dominant kernel alone: decode over the attended lengths, no store
    def kernel_step(self):
        K = self.K
        K.module().decode(K.runtime(), self.q, self.kc, self.vc, None, None, None, self.attend_lens, self.bt,
                          None, None)

    def units(self):
        return self.kv_bytes

    def kernel_units(self):
        return self.kv_bytes

    # end to end through the public API from pinned host buffers
    def e2e_setup(self):
        # The step's inputs (query rows, new K/V rows, lengths, page table)
        # staged in one pinned host buffer and sent with one copy into one
        # device buffer; the API reads views of it.
        srcs = [t for t in (self.q, self.kn, self.vn, self.lens, self.bt) if t is not None]
        offs, total = [], 0
        for t in srcs:
            offs.append(total)
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        self.h_buf = torch.empty(total, dtype=torch.uint8).pin_memory()
        self.d_buf = torch.empty(total, dtype=torch.uint8, device=self.q.device)

        def view(buf, t, off):
            n = t.numel() * t.element_size()
            return buf[off:off + n].view(t.dtype).view(t.shape)

        views = []
        for t, off in zip(srcs, offs):
            view(self.h_buf, t, off).copy_(t.cpu())
            views.append(view(self.d_buf, t, off))
        it = iter(views)
        self.d_q = next(it)
        self.d_kn = next(it) if self.kn is not None else None
        self.d_vn = next(it) if self.vn is not None else None
        self.d_lens, self.d_bt = next(it), next(it)
        self.h_out = torch.empty(self.q.shape, dtype=self.dtype).pin_memory()
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in srcs)
        self.d2h_bytes = self.h_out.numel() * self.h_out.element_size()

    def e2e_step(self):
        self.d_buf.copy_(self.h_buf, non_blocking=True)
        out = self.C.flash_attn_with_kvcache(self.d_q, self.kc, self.vc, k=self.d_kn, v=self.d_vn,
                                             cache_seqlens=self.d_lens, page_table=self.d_bt)
        self.h_out.copy_(out, non_blocking=True)

    # the C restatement of the reference kernel on the host cores
    def cpu_setup(self):
        self.c_kc, self.c_vc = self.kc.cpu(), self.vc.cpu()
        self.c_q = self.q.cpu().reshape(self.B, self.H, self.E).contiguous()
        self.c_kn = self.kn.cpu().reshape(self.c_q.shape).contiguous() if self.kn is not None else None
        self.c_vn = self.vn.cpu().reshape(self.c_q.shape).contiguous() if self.vn is not None else None
        self.c_out = torch.empty(self.c_q.shape, dtype=self.dtype)

    def cpu_step(self, threads):
        from oracle import cpu as ORACLE
        ORACLE.decode(self.c_q, self.c_kc, self.c_vc, self.lens_host, self.bt_host, self.c_out, k_new=self.c_kn,
                      v_new=self.c_vn, threads=threads)

    def config(self, world):
        lens = [int(n) for n in self.lens_host]
        return {"workload": self.name, "global_batch": self.global_batch, "batch_per_gpu": self.B,
                "heads": self.H, "head_dim": self.E, "page": self.page,
                "mean_len": round(sum(lens) / max(1, len(lens)), 1), "append": self.append,
                "parallelism": f"sequence-shard x{world}", "l2": "flushed (256 MiB write) before each step"}


class Prefill:
    """Dense prefill workloads (cfg1, cfg4, cfg4nc)."""

    def __init__(self, name, rank, world, dev, N, L, S, H, E, causal, fused):
        import cpu_attention as C

        self.C, self.name, self.dev = C, name, dev
        self.N, self.L, self.S, self.H, self.E, self.causal = N, L, S, H, E, causal
        self.dtype = torch.bfloat16
        gd = torch.Generator(device=dev).manual_seed(7 + rank)
        if fused:
            qkv = torch.randn(N, S, 3, H, E, generator=gd, device=dev, dtype=torch.float32).to(self.dtype)
            self.q, self.k, self.v = qkv[:, S - L:, 0], qkv[:, :, 1], qkv[:, :, 2]
        else:
            self.q = torch.randn(N, L, H, E, generator=gd, device=dev, dtype=torch.float32).to(self.dtype)
            self.k = torch.randn(N, S, H, E, generator=gd, device=dev, dtype=torch.float32).to(self.dtype)
            self.v = torch.randn(N, S, H, E, generator=gd, device=dev, dtype=torch.float32).to(self.dtype)
        pairs = sum(min(S, max(0, i + S - L + 1)) for i in range(L)) if causal else L * S
        self.flops = 4 * N * H * E * pairs
        self.global_batch = N * world
        self.launches_per_step = 1

    def step(self):
        self.C.flash_attn_func(self.q, self.k, self.v, causal=self.causal)

    kernel_step = step

    def units(self):
        return self.flops

    kernel_units = units

    def e2e_setup(self):
        # q, k, v staged in one pinned host buffer and sent with one copy into
        # one device buffer (contiguous [N, L, H, E] views of it)
        srcs = (self.q, self.k, self.v)
        sizes = [t.numel() * t.element_size() for t in srcs]
        offs = [0]
        for n in sizes[:-1]:
            offs.append(offs[-1] + (n + 255) // 256 * 256)
        total = offs[-1] + (sizes[-1] + 255) // 256 * 256
        self.h_buf = torch.empty(total, dtype=torch.uint8).pin_memory()
        self.d_buf = torch.empty(total, dtype=torch.uint8, device=self.dev)
        self.d = []
        for t, off, n in zip(srcs, offs, sizes):
            self.h_buf[off:off + n].view(t.dtype).view(t.shape).copy_(t.cpu())
            self.d.append(self.d_buf[off:off + n].view(t.dtype).view(t.shape))
        self.h_out = torch.empty(self.q.shape, dtype=self.dtype).pin_memory()
        self.h2d_bytes = sum(sizes)
        self.d2h_bytes = self.h_out.numel() * self.h_out.element_size()

    def e2e_step(self):
        self.d_buf.copy_(self.h_buf, non_blocking=True)
        out = self.C.flash_attn_func(*self.d, causal=self.causal)
        self.h_out.copy_(out, non_blocking=True)

    def cpu_setup(self):
        # a bounded sample: the first head of the first batch entry
        self.c = [t[:1, :, :1].cpu() for t in (self.q, self.k, self.v)]
        self.c_out = torch.empty(self.c[0].shape, dtype=self.dtype)
        self.cpu_units = self.flops / (self.N * self.H)

    def cpu_step(self, threads):
        from oracle import cpu as ORACLE
        ORACLE.flash(*self.c, self.c_out, causal=self.causal, threads=threads)

    def config(self, world):
        return {"workload": self.name, "global_batch": self.global_batch, "seq_q": self.L, "seq_k": self.S,
                "heads": self.H, "head_dim": self.E, "causal": self.causal,
                "parallelism": f"batch-shard x{world}", "l2": "flushed (256 MiB write) before each step"}


def shard_ranges(lens, world):
    """Contiguous sequence ranges per rank, balanced on context + 16 (the
    reference's `_share` cost model, paged_attn.mojo:788-816)."""
    from cpu_attention.shard import balanced_ranges
    return balanced_ranges([int(n) for n in lens], world)


def make_workload(name, rank, world, dev):
    if name == "cfg2":
        return Decode("cfg2: flash_attn_with_kvcache bf16 B=32 H=16 E=128 page16 lens~U[17,2047] +1 append",
                      rank, world, dev, torch.bfloat16, 32, 16, 128, 16,
                      lambda g: torch.randint(17, 2048, (32,), generator=g), append=True)
    if name in ("cfg3", "cfg3e32"):
        E = 64 if name == "cfg3" else 32
        return Decode(f"{name}: cross-attention decode fp32 B=64 H=8 E={E} page32 len=1500 no append",
                      rank, world, dev, torch.float32, 64, 8, E, 32,
                      lambda g: torch.full((64,), 1500, dtype=torch.int64), append=False)
    if name == "cfg5":
        return Decode("cfg5: engine decode bf16 B=256 H=32 E=128 page16 lens~U[1,8191] store+decode out=",
                      rank, world, dev, torch.bfloat16, 256, 32, 128, 16,
                      lambda g: torch.randint(1, 8192, (256,), generator=g), append=False, engine=True)
    if name == "cfg1":
        return Prefill("cfg1: flash_attn_func bf16 N=1 L=S=128 H=16 E=64 causal", rank, world, dev,
                       1, 128, 128, 16, 64, True, False)
    if name == "cfg4":
        return Prefill("cfg4: flash_attn_func bf16 N=4 L=S=2048 H=32 E=128 causal fused-QKV views", rank, world,
                       dev, 4, 2048, 2048, 32, 128, True, True)
    if name == "cfg4nc":
        return Prefill("cfg4nc: flash_attn_func bf16 N=4 L=512 S=2048 H=32 E=128 non-causal fused-QKV views",
                       rank, world, dev, 4, 512, 2048, 32, 128, False, True)
    raise SystemExit(f"unknown workload {name}")


# --------------------------------------------------------------------- timing --
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.proc = None
        self.path = None
        self.gpus = gpus

    def start(self):
        """Start sampling every 50 ms; returns once the first sample is in
        (at most ~5 s), so the timed region that follows is covered."""
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

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 8:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = max(mx, float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[4:8]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# DRAM bytes (read + write) of one launch of the roofline kernel, from one ncu
# capture of the same command (the files under profiles/ give the commands).
TRAFFIC = {
    "cfg2": (284.9e6, "profiles/decode_kernel_cfg2.md"),
    "cfg4": (555.6e6, "profiles/flash_tc_kernel_cfg4.md"),
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
    if isinstance(wl, Prefill):
        return "prefill bf16 TFLOP/s", "TFLOP/s", 1e12
    return "paged-decode KV GB/s", "GB/s", 1e9


def cpu_baseline(wl, threads, budget_s=20.0):
    """The oracle's C restatement of the reference kernel on the host cores,
    3 warm-up + up to 10 timed calls within about budget_s seconds; median."""
    wl.cpu_setup()
    for _ in range(2):
        wl.cpu_step(threads)
    times = []
    t_start = time.perf_counter()
    while len(times) < 10 and (time.perf_counter() - t_start) < budget_s:
        t0 = time.perf_counter()
        wl.cpu_step(threads)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    units = getattr(wl, "cpu_units", wl.units())
    return sec, units, len(times)


def run_reference(args):
    """The reference arm: the C restatement of the reference's CPU kernel
    (`oracle/`), the reference's own Mojo kernel being unbuildable here, timed
    on all host threads, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
    wl = make_workload(args.workload, 0, 1, dev)
    metric, unit, scale = metric_of(wl)
    wl.cpu_setup()
    for _ in range(args.warmup):
        wl.cpu_step(threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        wl.cpu_step(threads)
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    units = getattr(wl, "cpu_units", wl.units())
    value = units / sec / scale
    sample = "full workload per step" if not hasattr(wl, "cpu_units") else "one (batch, head) of the workload per step"
    line = {"impl": "reference", "metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": str(wl.dtype).split(".")[-1],
            "data": "synthetic", "config": wl.config(1),
            "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="cfg2")
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
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    wl = make_workload(args.workload, rank, world, dev)
    stream = torch.cuda.current_stream(dev)
    flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    flush = lambda: flush_buf.fill_(1)  # noqa: E731
    metric, unit, scale = metric_of(wl)

    # clocks are sampled from here through the roofline and e2e phases: the
    # whole window in which this run keeps the GPUs busy
    barrier(world)
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
    barrier(world)
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
    if isinstance(wl, Prefill):
        achieved = wl.kernel_units() / (kern_avg * 1e-3) / 1e12
        peak, bound, runit = pk["bf16_tflops"], "tensor", "TFLOP/s"
    else:
        achieved = wl.kernel_units() / (kern_avg * 1e-3) / 1e9
        peak, bound, runit = pk["hbm_gbs"], "hbm", "GB/s"
    achieved = max_over_ranks(-achieved, world) * -1  # the slowest rank
    roofline = {"bound": bound, "achieved": round(achieved, 2), "peak": peak, "peak_kind": pk_kind,
                "unit": runit, "frac": round(achieved / peak, 4),
                "traffic": TRAFFIC[args.workload][0] if args.workload in TRAFFIC else None,
                "traffic_source": TRAFFIC[args.workload][1] if args.workload in TRAFFIC else None,
                "kernel_ms": round(kern_avg, 4)}

    # end to end through the public API, host buffers
    wl.e2e_setup()
    e2e_ms = timed(wl.e2e_step, args.steps, 2, flush, stream, hide_host=False)
    e2e_total = max_over_ranks(sum(e2e_ms), world)
    e2e_value = units / (e2e_total / args.steps * 1e-3) / scale

    # N > 1 decode: the same step with the output all-gather after it
    with_gather = None
    if world > 1 and hasattr(wl, "gather_step"):
        g_ms = timed(wl.gather_step, args.steps, 2, flush, stream)
        g_total = max_over_ranks(sum(g_ms), world)
        with_gather = {"value": round(units / (g_total / args.steps * 1e-3) / scale, 3), "unit": unit,
                       "ms_per_step": round(g_total / args.steps, 4), "collective": "all_gather_into_tensor"}
    barrier(world)
    clocks = sampler.stop() if sampler else None

    line = {"metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "us_per_call": round(ms_per_step * 1e3, 2),
            "higher_is_better": True, "scaling": "strong" if getattr(wl, "engine", False) else "weak",
            "vs_baseline": None, "dtype": str(wl.dtype).split(".")[-1], "data": "synthetic",
            "config": wl.config(world), "roofline": roofline,
            "e2e": {"value": round(e2e_value, 3), "unit": unit, "h2d_bytes_per_step": wl.h2d_bytes,
                    "d2h_bytes_per_step": wl.d2h_bytes, "ms_per_step": round(e2e_total / args.steps, 4)},
            "gpu_launches": wl.launches_per_step * args.steps, "clocks": clocks}
    if with_gather is not None:
        line["with_gather"] = with_gather
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        sec, cunits, n = cpu_baseline(wl, threads)
        sample = ("the full workload, median of %d calls" % n if not hasattr(wl, "cpu_units")
                  else "one (batch, head) slice of the workload, median of %d calls" % n)
        line["cpu_baseline"] = {"value": round(cunits / sec / scale, 4), "unit": unit, "cores": threads,
                                "kind": "port", "sample": sample, "ms_per_call": round(sec * 1e3, 3)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
