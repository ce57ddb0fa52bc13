"""Batch sharding across ranks (host logic, CPU + gloo).

Images are independent, so N ranks split the batch with no collective on the
data path; the only cross-rank operation is the max over ranks of the timed
duration, outside the timed region.  Each rank here computes its shard with
the CPU oracle; the gathered shards must equal the whole-batch result.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from depthwise_conv_b200.shard import shard_range


@pytest.mark.parametrize("batch,world", [(0, 2), (1, 2), (2, 2), (7, 2), (16, 4), (5, 8), (256, 8), (3, 1)])
def test_shard_range_partitions_the_batch(batch, world):
    ranges = [shard_range(batch, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == batch
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1 and sizes == sorted(sizes, reverse=True)


def test_shard_range_rejects_bad_args():
    with pytest.raises(ValueError):
        shard_range(4, 0, 0)
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, B, out_dir):
    import torch
    import torch.distributed as dist
    from depthwise_conv_b200.shard import max_over_ranks, shard_range, sum_over_ranks
    from oracle import oracle as O
    from conftest import make_problem

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x, w = make_problem(9, B, 6, 7, 16, 5)
    lo, hi = shard_range(B, world, rank)
    y32, _ = O.dw_forward(x[lo:hi], w, nthreads=1)
    # gather the shards (test only; the engine itself never exchanges data)
    t = torch.zeros(B, 6, 7, 16, dtype=torch.float32)
    t[lo:hi] = torch.from_numpy(y32)
    dist.all_reduce(t)
    slow = max_over_ranks(float(rank + 1))
    total = sum_over_ranks(float(hi - lo))
    if rank == 0:
        np.save(os.path.join(out_dir, "gathered.npy"), t.numpy())
        np.save(os.path.join(out_dir, "stats.npy"), np.array([slow, total]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharded_run_equals_whole_batch(tmp_path, oracle_mod):
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    B, world = 5, 2
    mp.start_processes(_worker, args=(world, _free_port(), B, str(tmp_path)), nprocs=world, start_method="spawn")
    from conftest import make_problem
    x, w = make_problem(9, B, 6, 7, 16, 5)
    full, _ = oracle_mod.dw_forward(x, w)
    np.testing.assert_array_equal(np.load(tmp_path / "gathered.npy"), full)
    slow, total = np.load(tmp_path / "stats.npy")
    assert slow == world and total == B
