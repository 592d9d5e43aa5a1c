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


def _metrics_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from neuratensor_b200 import ModelConfig, NeuraTensorModel
        model = NeuraTensorModel(ModelConfig(vocab_size=64, d_model=16, n_layers=3, d_state=4))
        # rank 0 ran 3 rows of 10 steps, rank 1 one row; d_inner 32
        rows = 3 if rank == 0 else 1
        counts = torch.tensor([100 * (rank + 1), 7 + rank, 0], dtype=torch.int64)
        tot, numel = ranks.global_counts(counts, rows * 10 * 32)
        q.put((rank, tot.tolist(), numel, model.metrics_from_counts(tot.tolist(), numel, torch.bfloat16)))
    finally:
        dist.destroy_process_group()


def test_global_metrics_over_uneven_gloo_ranks():
    """The engine's torchrun mode: per-layer spike counts and element counts are
    summed over ranks, so every rank reports the reference's metrics of the whole
    global batch (model.py:286-291), equal to one process over all rows."""
    from neuratensor_b200 import ModelConfig, NeuraTensorModel
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_metrics_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    out = sorted(q.get(timeout=10) for _ in range(world))
    one = NeuraTensorModel(ModelConfig(vocab_size=64, d_model=16, n_layers=3, d_state=4))
    expect = one.metrics_from_counts([300, 15, 0], 4 * 10 * 32, torch.bfloat16)
    for rank, tot, numel, metrics in out:
        assert tot == [300, 15, 0] and numel == 4 * 10 * 32
        assert metrics == expect
    c = torch.tensor([3, 5])
    assert ranks.global_counts(c, 11) == (c, 11)            # one process: unchanged
