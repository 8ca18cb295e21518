"""Column sharding of a batch across the ranks of one node (weak scaling).

Samples (batch columns) are independent, so rank r of `world` owns the
global columns [r * per_rank, (r + 1) * per_rank) and no data crosses ranks
on the forward path; the collectives are the reduction of each rank's timing
to the job's (the slowest rank's) time, outside the timed region, and the
broadcast of a parameter update to every rank's replica of the model.
"""
from __future__ import annotations


def shard_range(rank: int, world: int, per_rank: int) -> tuple[int, int]:
    """First global column and column count of `rank`'s shard."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if per_rank <= 0:
        raise ValueError("each rank needs a nonzero number of columns")
    return rank * per_rank, per_rank


def split_range(rank: int, world: int, total: int) -> tuple[int, int]:
    """First global column and column count of `rank`'s part of a fixed
    batch of `total` columns split across `world` ranks (strong scaling):
    contiguous ranges, the first total % world ranks one column longer."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if total < world:
        raise ValueError(f"a batch of {total} columns cannot give each of {world} ranks a column")
    base, rem = divmod(total, world)
    return rank * base + min(rank, rem), base + (1 if rank < rem else 0)


def bind_numa(local_rank: int):
    """Restrict this process to the CPUs of its GPU's NUMA node (best effort),
    so that pinned host buffers allocated afterwards are placed on that node
    (first touch).  Returns the node, or None when it cannot be determined."""
    import os
    import subprocess
    try:
        bus = subprocess.run(["nvidia-smi", "-i", str(local_rank), "--query-gpu=pci.bus_id",
                              "--format=csv,noheader"], capture_output=True, text=True, timeout=10).stdout.strip()
        dom, rest = bus.split(":", 1)
        path = f"/sys/bus/pci/devices/{dom[-4:].lower()}:{rest.lower()}/numa_node"
        node = int(open(path).read().strip())
        if node < 0:
            return None
        cpus = set()
        for part in open(f"/sys/devices/system/node/node{node}/cpulist").read().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
        return node
    except Exception:
        return None


def job_time(seconds: float, world: int, device=None) -> float:
    """The job's time: the maximum of every rank's `seconds` (all ranks call)."""
    if world <= 1:
        return float(seconds)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def broadcast_parameters(model, values=None, src: int = 0, world: int | None = None) -> None:
    """Replace the trainable parameters of every rank's replica with `values`
    from rank `src` (tuple order; a tensor on this rank's device, any of
    fp32 / fp64 / fp16 / bf16; ignored on the other ranks).

    One broadcast of the values in device memory (NCCL over NVLink on GPUs),
    then each rank writes them into its own planned device images
    (`set_trainable_parameters_device`: converted to the model dtype on the
    device, no re-plan).  Collective: every rank calls it.
    """
    import torch
    import torch.distributed as dist

    if world is None:
        world = dist.get_world_size() if dist.is_initialized() else 1
    n = model.get_num_trainable_parameters()
    if world > 1:
        rank = dist.get_rank()
        # Every rank needs the source dtype to size its receive buffer.
        codes = [torch.float32, torch.float64, torch.float16, torch.bfloat16]
        dev = values.device if (rank == src and values is not None) else model.parameter_device()
        hdr = torch.zeros(1, dtype=torch.int64, device=dev)
        if rank == src:
            if values is None or values.numel() != n:
                raise ValueError(f"rank {src} must pass {n} parameter values")
            hdr[0] = codes.index(values.dtype)
        dist.broadcast(hdr, src)
        dtype = codes[int(hdr.item())]
        buf = values.reshape(-1).contiguous() if rank == src else torch.empty(n, dtype=dtype, device=dev)
        dist.broadcast(buf, src)
        values = buf
    model.set_trainable_parameters_device(values)
