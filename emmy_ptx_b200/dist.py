"""Multi-GPU plumbing: one process per GPU, units sharded by rank, the sum's partials combined once.

Every benchmark configuration partitions into independent units (rows, batches, (b,h) pairs), so each
rank owns a full-size shard of a weak-scaled global problem and runs the same kernel on it with no
data-path collective.  The full-array sum is the one exchange: each rank reduces its shard to one
partial, then one ``ncclAllReduce`` (through the C ABI) adds the partials.  ``torch.distributed``
carries only control traffic: the NCCL unique id, barriers and the max-over-ranks of timings.
"""
from __future__ import annotations

import datetime
import os


def env() -> tuple[int, int, int]:
    """(world size, rank, local rank) from the torchrun environment (1, 0, 0 when absent)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(world: int, local: int, backend: str = "nccl", timeout_s: float = 180.0):
    """Initialise the process group (world > 1) and bind this process to its GPU; returns the
    ``torch.distributed`` module or None for a single process."""
    import torch
    import torch.distributed as dist
    if backend == "nccl":
        torch.cuda.set_device(local)
    if world <= 1:
        return None
    if not dist.is_initialized():
        kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kw)
    return dist


def shard(n_units: int, world: int, rank: int) -> range:
    """This rank's contiguous share of ``n_units`` (sizes differ by at most one)."""
    lo = n_units * rank // world
    hi = n_units * (rank + 1) // world
    return range(lo, hi)


def max_over_ranks(dist, value: float) -> float:
    """The largest ``value`` over all ranks (identity for a single process)."""
    if dist is None:
        return value
    import torch
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def share_unique_id(dist, rank: int, make_uid) -> bytes:
    """Rank 0 makes the 128-byte NCCL unique id (``make_uid()``); every rank receives it."""
    box = [make_uid() if rank == 0 else None]
    if dist is not None:
        dist.broadcast_object_list(box, src=0)
    uid = box[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("NCCL unique id missing or malformed")
    return bytes(uid)


class AllReducePartials:
    """The sum's exchange step: ``ncclAllReduce(sum)`` of each rank's partial through the C ABI."""

    def __init__(self, device, dist, rank: int, world: int):
        self.dev = device
        self.active = world > 1
        if self.active:
            uid = share_unique_id(dist, rank, device.nccl_unique_id)
            device.nccl_init(rank, world, uid)

    def __call__(self, tensor, dtype: str, stream: int) -> None:
        if self.active:
            self.dev.allreduce_sum(tensor.data_ptr(), tensor.numel(), dtype, stream)

    def close(self) -> None:
        if self.active:
            self.dev.nccl_destroy()
            self.active = False
