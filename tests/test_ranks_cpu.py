"""Multi-rank host logic (one process per GPU in the bench) on two gloo CPU ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from neuratensor_b200.inference import ranks


def test_batch_shard_covers_the_batch_once():
    for gb in (1, 7, 8, 33):
        for world in (1, 2, 3, 8):
            rows = []
            for r in range(world):
                a, b = ranks.batch_shard(gb, world, r)
                rows += list(range(a, b))
            assert rows == list(range(gb)), (gb, world)
    with pytest.raises(ValueError):
        ranks.batch_shard(8, 2, 2)


def test_single_process_is_identity():
    c = torch.tensor([3, 5], dtype=torch.int64)
    assert torch.equal(ranks.sum_counts(c), c)
    assert ranks.max_over_ranks(2.5, torch.device("cpu")) == 2.5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # each rank's per-layer counts, as forward_device returns them
        counts = torch.tensor([10 * (rank + 1), rank, 7], dtype=torch.int64)
        total = ranks.sum_counts(counts)
        slowest = ranks.max_over_ranks(1.0 + rank, torch.device("cpu"))
        q.put((rank, total.tolist(), slowest, ranks.batch_shard(9, world, rank)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_sum_counts_and_take_the_max():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    out = sorted(q.get(timeout=10) for _ in range(world))
    for rank, total, slowest, shard in out:
        assert total == [30, 1, 14]
        assert slowest == 2.0
    assert [o[3] for o in out] == [(0, 5), (5, 9)]
