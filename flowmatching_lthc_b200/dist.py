"""Data-parallel plumbing for the LTHC path: one process per GPU, the batch split
into contiguous per-rank shards, no collective on the data path.  The only
cross-rank steps are the max-over-ranks reduction of device timings (benchmark)
and, in training, the gradient all-reduce that DDP performs on the LTHC weights
(their gradients are sums over the batch, so per-rank sums add up exactly to
the full-batch gradient)."""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Rank:
    rank: int
    world: int
    local_rank: int

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def from_env() -> Rank:
    """Read RANK / WORLD_SIZE / LOCAL_RANK as set by torch.distributed.run."""
    return Rank(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, r: Rank, timeout_s: float = 120.0, device: torch.device | None = None) -> None:
    """Initialise the default process group (no-op for a single rank).  `device`
    binds an NCCL group to this rank's GPU."""
    if r.world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = {"device_id": device} if device is not None else {}
        dist.init_process_group(backend, rank=r.rank, world_size=r.world, timeout=timedelta(seconds=timeout_s), **kw)


def shard(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of `total` items for `rank`; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def reduce_max(value: float, device: torch.device | str = "cpu") -> float:
    """Max of a scalar over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum_(t: torch.Tensor) -> torch.Tensor:
    """In-place sum over ranks (identity without a process group)."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t


class FlatGradients:
    """Data-parallel gradient exchange as one collective per step.

    Every trainable parameter's ``.grad`` is made a view into one contiguous fp32
    buffer, so backward accumulates straight into it; ``allreduce()`` then averages
    the whole buffer over the ranks with a single all-reduce (a no-op on one rank).
    The result equals DistributedDataParallel's (the mean of the per-rank
    gradients); the exchange is one large collective after backward instead of
    DDP's bucketed collectives interleaved with it, which on one NVSwitch node
    cost more than the transfer itself.  Call ``zero_grad()`` instead of the
    optimiser's (the views must survive; ``set_to_none`` would drop them)."""

    def __init__(self, params) -> None:
        self.params = [q for q in params if q.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        dev = self.params[0].device
        if any(q.dtype != torch.float32 or q.device != dev for q in self.params):
            raise ValueError("FlatGradients expects fp32 parameters on one device")
        self.flat = torch.zeros(sum(q.numel() for q in self.params), device=dev)
        off = 0
        for q in self.params:
            q.grad = self.flat[off:off + q.numel()].view_as(q)
            off += q.numel()

    def zero_grad(self) -> None:
        self.flat.zero_()

    def allreduce(self) -> None:
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.AVG if self.flat.is_cuda else dist.ReduceOp.SUM)
            if not self.flat.is_cuda:  # gloo has no AVG
                self.flat.div_(dist.get_world_size())


def barrier() -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def shutdown() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
