"""Parameter update across GPUs: rank 0's new parameters reach every rank's
replica (NCCL broadcast in device memory, then each rank's device scatter),
and every rank's forward equals a model planned from scratch with the same
values on that GPU.  Needs two GPUs; runs as two child processes."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import torch.distributed as dist

    import ponni_b200 as pb
    from ponni_b200 import configs, sharding

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device(f"cuda:{rank}"))
    try:
        layers = configs.cfg2(batch=8).layers
        m = pb.Inference(layers, dtype=pb.F32, device=rank)
        x = torch.randn(30, 999, device=f"cuda:{rank}", generator=torch.Generator(f"cuda:{rank}").manual_seed(1))
        m.forward_batch_parallel(x)
        n = m.get_num_trainable_parameters()
        vals = None
        if rank == 0:
            vals = torch.from_numpy(np.random.default_rng(4).normal(0, 0.2, n)).cuda(0)
        sharding.broadcast_parameters(m, vals, src=0)
        y = m.forward_batch_parallel(x).clone()
        fresh = pb.Inference(layers, dtype=pb.F32, device=rank)
        fresh.set_trainable_parameters(np.random.default_rng(4).normal(0, 0.2, n))
        y_ref = fresh.forward_batch_parallel(x)
        torch.cuda.synchronize()
        out.put((rank, bool(torch.equal(y.view(torch.int32), y_ref.view(torch.int32))), m.check_parameters()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_parameter_broadcast_two_gpus():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    got = [out.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same, check in got:
        assert same, f"rank {rank} differs from a fresh plan"
        assert check == (0, 0), rank
