"""Multi-rank host path of bench.py on CPU: world_size-2 gloo ranks, one all_gather of stats.

Requests shard across ranks with no data-path collective; the only collective is
the post-timing gather of per-rank stats, and the job's time is the slowest rank's.
"""
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path):
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from datetime import timedelta
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # rank r: elapsed 10+r ms, e2e 20+2r ms, status bit 1<<r, 35 launches
        stats = torch.tensor([10.0 + rank, 20.0 + 2 * rank, float(1 << rank), 35.0], dtype=torch.float64)
        allstats = bench.gather_stats(stats, world)
        agg = bench.aggregate_stats(allstats)
        if rank == 0:
            torch.save(dict(allstats=allstats, agg=agg), out_path)
        # every rank must see the same gathered table
        assert allstats.shape == (world, 4)
        assert allstats[:, 0].tolist() == [10.0 + r for r in range(world)]
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_gather_and_aggregate_over_two_gloo_ranks(tmp_path):
    world, port = 2, _free_port()
    out = str(tmp_path / 'agg.pt')
    mp.start_processes(_rank_main, args=(world, port, out), nprocs=world, join=True, start_method='spawn')
    res = torch.load(out)
    agg = res['agg']
    assert agg['elapsed_ms'] == 11.0          # slowest rank
    assert agg['e2e_ms'] == 22.0
    assert agg['status'] == 3                 # OR of every rank's status bits
    assert agg['launches'] == 70


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench
    stats = torch.tensor([5.0, 6.0, 0.0, 35.0], dtype=torch.float64)
    agg = bench.aggregate_stats(bench.gather_stats(stats, 1))
    assert agg == dict(elapsed_ms=5.0, e2e_ms=6.0, status=0, launches=35)


def test_weak_scaling_units_and_seeds():
    """Every rank streams the same context lengths (drawn once per config from its seed);
    only the K/V values differ by rank, so per-rank bytes are equal at every N."""
    sys.path.insert(0, ROOT)
    import bench
    assert bench.query_units() == 64 * 7 * 5 + 128 * 7 * 28
    c0 = bench.contexts(bench.VERIFY)
    assert len(c0) == 128 and c0 == bench.contexts(bench.VERIFY)
    assert all(256 <= c <= 8192 for c in c0)
    d0 = bench.contexts(bench.DRAFT)
    assert len(d0) == 64 and all(128 <= c <= 4096 for c in d0)
