"""The N>1 path's host logic on CPU, as world_size-2 ``gloo`` ranks: the decode
batch split by sequence (``shard.balanced_ranges``, the reference's ``_share``
one level up: ``paged_attn.mojo:788-816``), each rank attending only its own
sequences, the optional output all-gather (``shard.gather_outputs``) and the
bench's max/sum over ranks. The attention itself is the float64 restatement,
so the sharded result must equal the unsharded one bit for bit."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from cpu_attention.shard import balanced_ranges, gather_outputs
from oracle import attention_f64 as F64

LENS = [17, 2047, 5, 0, 300, 1024, 1, 777, 64, 1500, 33]
H, D, PAGE = 2, 32, 16


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rows(lo, hi):
    q, bt, total, ks, vs = cases.stage_inputs(LENS, H, D, PAGE, torch.float32, seed=5)
    return [F64.attention(q[i:i + 1], ks[i], vs[i], D ** -0.5) for i in range(lo, hi)]


def _worker(rank, world, port, out_path):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ranges = balanced_ranges(LENS, world)
        lo, hi = ranges[rank]
        rows = _rows(lo, hi)
        local = torch.from_numpy(np.concatenate(rows)) if rows else torch.zeros((0, 1, H, D), dtype=torch.float64)
        full = gather_outputs(local, [b - a for a, b in ranges])
        import bench
        slowest = bench.max_over_ranks(float(rank + 1), world)
        units = bench.sum_over_ranks(float(hi - lo), world)
        if rank == 0:
            torch.save({"full": full, "slowest": slowest, "units": units}, out_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8, 16])
def test_balanced_ranges_cover_in_order_and_balance(parts):
    ranges = balanced_ranges(LENS, parts)
    assert len(ranges) == parts and ranges[0][0] == 0 and ranges[-1][1] == len(LENS)
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert a <= b == c <= d
    cost = [n + 16 for n in LENS]
    target = sum(cost) / parts
    for a, b in ranges:  # each part within one sequence's cost of its share
        assert abs(sum(cost[a:b]) - target) <= max(cost) + 1e-9 or b - a == 0


def test_balanced_ranges_matches_bench_shard():
    import bench
    for world in (1, 2, 4, 8):
        assert bench.shard_ranges(torch.tensor(LENS), world) == balanced_ranges(LENS, world)


def test_sharded_decode_gathers_to_the_unsharded_result(tmp_path):
    out_path = str(tmp_path / "rank0.pt")
    mp.start_processes(_worker, args=(2, _free_port(), out_path), nprocs=2, join=True, start_method="spawn")
    got = torch.load(out_path)
    ref = torch.from_numpy(np.concatenate(_rows(0, len(LENS))))
    assert got["full"].shape == ref.shape
    assert torch.equal(got["full"], ref)
    assert got["slowest"] == 2.0
    assert got["units"] == float(len(LENS))


def _even_worker(rank, world, port, out_path):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        local = torch.full((3, 2, 4), float(rank), dtype=torch.float32) + torch.arange(3.0)[:, None, None] / 10
        full = gather_outputs(local, [3] * world)
        if rank == 0:
            torch.save(full, out_path)
    finally:
        dist.destroy_process_group()


def test_even_shards_gather_without_padding(tmp_path):
    """Equal shard sizes take the direct all-gather (no pad, no cut); the
    rows still come back in rank order."""
    out_path = str(tmp_path / "even.pt")
    mp.start_processes(_even_worker, args=(2, _free_port(), out_path), nprocs=2, join=True, start_method="spawn")
    full = torch.load(out_path)
    ref = torch.cat([torch.full((3, 2, 4), float(r)) + torch.arange(3.0)[:, None, None] / 10 for r in range(2)])
    assert torch.equal(full, ref)
