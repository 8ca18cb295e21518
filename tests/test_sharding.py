"""The multi-GPU path's host logic on CPU: two gloo ranks shard the batch by
columns (no data exchange), compute their shards, and reduce their timings to
the slowest rank's; the gathered shards equal the one-process result.  A
parameter update from rank 0 reaches every rank's replica."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from ponni_b200 import sharding

NIN, PER_RANK = 5, 777


def keyed_inputs(col0: int, n: int) -> np.ndarray:
    """Inputs keyed by global column (like the device generator): any column
    range gives the same values whichever rank produces it."""
    cols = np.arange(col0, col0 + n, dtype=np.uint64)[None, :]
    feats = np.arange(NIN, dtype=np.uint64)[:, None]
    h = (cols * np.uint64(0x9E3779B97F4A7C15) + feats * np.uint64(0xBF58476D1CE4E5B9)) & np.uint64((1 << 53) - 1)
    return (h.astype(np.float64) / float(1 << 53) * 4.0 - 2.0).astype(np.float32)


def layers():
    import ponni_b200 as pb
    rng = np.random.default_rng(3)
    return [pb.Matvec(rng.normal(0, 0.5, (NIN, 6))), pb.Bias(rng.normal(0, 0.1, 6)), pb.Relu(6),
            pb.Matvec(rng.normal(0, 0.5, (6, 2))), pb.Bias(rng.normal(0, 0.1, 2))]


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    from oracle import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    col0, n = sharding.shard_range(rank, world, PER_RANK)
    y = oracle.forward(layers(), 0, keyed_inputs(col0, n), 1)
    shards = [torch.empty((2, PER_RANK), dtype=torch.float32) for _ in range(world)]
    dist.all_gather(shards, torch.from_numpy(np.ascontiguousarray(y)))
    t = sharding.job_time(0.5 + rank, world)  # rank r "took" 0.5 + r seconds
    if rank == 0:
        out.put((torch.cat(shards, dim=1).numpy(), t))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range():
    assert sharding.shard_range(0, 1, 10) == (0, 10)
    assert sharding.shard_range(3, 4, 10) == (30, 10)
    with pytest.raises(ValueError):
        sharding.shard_range(4, 4, 10)
    with pytest.raises(ValueError):
        sharding.shard_range(0, 2, 0)
    assert sharding.job_time(1.25, 1) == 1.25


def test_split_range_strong_scaling():
    # a fixed batch split into contiguous ranges that tile it exactly
    for total in (8, 67_108_864, 134_217_728 + 5, 1001):
        for world in (1, 2, 4, 8):
            parts = [sharding.split_range(r, world, total) for r in range(world)]
            assert parts[0][0] == 0
            assert all(a[0] + a[1] == b[0] for a, b in zip(parts, parts[1:]))
            assert parts[-1][0] + parts[-1][1] == total
            assert max(p[1] for p in parts) - min(p[1] for p in parts) <= 1
    with pytest.raises(ValueError):
        sharding.split_range(0, 4, 3)
    with pytest.raises(ValueError):
        sharding.split_range(4, 4, 100)


def test_two_gloo_ranks_match_one_process(oracle_lib):
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    y_sharded, t = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from oracle import oracle
    y_full = oracle.forward(layers(), 0, keyed_inputs(0, world * PER_RANK), 1)
    assert np.array_equal(y_sharded, y_full)
    assert t == 1.5  # the slowest rank's time


class _Replica:
    """Stands in for a model on CPU ranks: records the device update."""

    def __init__(self, n):
        self.n, self.got = n, None

    def get_num_trainable_parameters(self):
        return self.n

    def parameter_device(self):
        import torch
        return torch.device("cpu")

    def set_trainable_parameters_device(self, values):
        self.got = values.clone()


def _bcast_rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    m = _Replica(11)
    vals = torch.arange(11, dtype=torch.float64) * 0.5 if rank == 0 else None
    sharding.broadcast_parameters(m, vals, src=0)
    out.put((rank, m.got.dtype == torch.float64, m.got.tolist()))
    dist.barrier()
    dist.destroy_process_group()


def test_parameter_broadcast_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bcast_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    got = [out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, is_f64, vals in got:
        assert is_f64 and vals == [0.5 * i for i in range(11)], rank


def test_parameter_broadcast_single_process():
    m = _Replica(3)
    import torch
    sharding.broadcast_parameters(m, torch.ones(3), world=1)
    assert m.got.tolist() == [1.0, 1.0, 1.0]
