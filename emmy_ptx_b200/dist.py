"""Multi-GPU plumbing: one process per GPU, units sharded by rank, the sum's partials combined once.

Every benchmark configuration partitions into independent units (rows, batches, (b,h) pairs), so each
rank owns a shard (``shard``) and runs the same kernel on it with no data-path collective.  The
full-array sum is the one exchange: each rank reduces its shard to one partial, then either one
``ncclAllReduce`` through the C ABI (``AllReducePartials``) or the peer-exchange kernel over NVLink
(``PeerAllReduce``, :mod:`.kernels.peer_sum`) adds the partials.  ``torch.distributed`` carries only
control traffic: the NCCL unique id and IPC handles, barriers and the max-over-ranks of timings.
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


def agree(dist, ok: bool) -> bool:
    """True only if ``ok`` holds on every rank (so that all ranks take the same path)."""
    if dist is None:
        return ok
    import torch
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def exchange_handles(dist, rank: int, world: int, handle: bytes) -> list:
    """Every rank's 64-byte IPC handle, in rank order."""
    if dist is None:
        return [handle]
    out = [None] * world
    dist.all_gather_object(out, handle)
    if any(not isinstance(h, (bytes, bytearray)) or len(h) != 64 for h in out):
        raise RuntimeError("an IPC handle is missing or malformed")
    return [bytes(h) for h in out]


class PeerAllReduce:
    """The sum's exchange step as the peer-exchange kernel (:mod:`.kernels.peer_sum`).

    Set-up: each rank allocates a 2 KiB exchange buffer (``cuMemAlloc``, zeroed), exports its IPC
    handle, receives every rank's handle, maps the others' buffers into this process and writes the
    table of the ``world`` buffer addresses to the device.  Every rank must then launch the kernel the
    same number of times (each launch is one step); the kernel's bounded wait writes status code 51
    if a peer never arrives.  ``close`` unmaps the peers' buffers and frees this rank's."""

    def __init__(self, device, dist, rank: int, world: int, dtype: str):
        import torch
        from .codegen.module import module_text
        from .kernels import peer_sum
        self.dev, self.rank, self.world, self.dtype = device, rank, world, dtype
        self.opened: list[int] = []
        self.xch = 0
        self.module = None
        # each stage ends with an agreement, so a failure on any rank fails the set-up on every rank
        # (and no rank is left waiting in a collective the others skipped)
        handle, why = None, ""
        try:
            self.xch = device.mem_alloc(peer_sum.BUF_BYTES)
            device.memset_d32(self.xch, 0, peer_sum.BUF_BYTES // 4, 0)
            device.sync()
            handle = device.ipc_handle(self.xch)
        except Exception as exc:           # noqa: BLE001 - reported on every rank below
            why = f"{type(exc).__name__}: {exc}"
        if not agree(dist, handle is not None):
            self.close()
            raise RuntimeError(f"peer exchange set-up failed on some rank ({why or 'another rank'})")
        handles = exchange_handles(dist, rank, world, handle)
        ok = True
        try:
            ptrs = []
            for r, h in enumerate(handles):
                if r == rank:
                    ptrs.append(self.xch)
                else:
                    q = device.ipc_open(h)
                    self.opened.append(q)
                    ptrs.append(q)
            self.table = torch.tensor(ptrs, dtype=torch.int64, device=f"cuda:{device.index}")
            self.err = torch.zeros(4, dtype=torch.int32, device=f"cuda:{device.index}")
            rec = peer_sum.peer_sum_entry(f"peer_sum_{dtype}", rank, world, dtype)
            self.module = device.load_ptx(module_text([rec]))
            self.fn = device.function(self.module, rec["name"])
        except Exception as exc:           # noqa: BLE001
            ok, why = False, f"{type(exc).__name__}: {exc}"
        if not agree(dist, ok):
            self.close()
            raise RuntimeError(f"peer exchange mapping failed on some rank ({why or 'another rank'})")

    def __call__(self, tensor, dtype: str, stream: int) -> None:
        if dtype != self.dtype or tensor.numel() != 1:
            raise ValueError("the peer exchange adds one partial of the dtype it was built for")
        self.dev.launch_u64(self.fn, [1, 1, 1], [32, 1, 1], 0, stream,
                            [tensor.data_ptr(), self.xch, self.table.data_ptr(), self.err.data_ptr()])

    def error_code(self) -> int:
        return int(self.err[0].item())

    def close(self) -> None:
        for q in self.opened:
            try:
                self.dev.ipc_close(q)
            except Exception:
                pass
        self.opened = []
        if getattr(self, "module", None) is not None:
            self.dev.unload(self.module)
            self.module = None
        if self.xch:
            self.dev.mem_free(self.xch)
            self.xch = 0
