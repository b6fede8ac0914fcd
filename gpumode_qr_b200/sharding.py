"""Batch sharding across GPUs: one process per GPU, no collective on the hot path.

Each matrix factors independently, so a batch is split into contiguous shards,
one per rank; every rank generates (or receives) its own shard and factors it
locally. ``torch.distributed`` (NCCL between GPUs, gloo on CPU) is used only
around the hot path: a barrier before timing, a MAX-reduce of per-rank device
times, and the optional gather of the (H, tau) shards to one rank.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_range(batch: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, end) of ``rank``'s shard; sizes differ by at most one."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank/world {rank}/{world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class DistInfo:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    initialized: bool = False

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def init_from_env(backend: str | None = None, timeout_s: float = 120.0) -> DistInfo:
    """Join the process group described by RANK/WORLD_SIZE/LOCAL_RANK (torchrun).

    With WORLD_SIZE unset or 1 nothing is initialised. The backend defaults to
    NCCL when CUDA is available, gloo otherwise.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world <= 1:
        return DistInfo(rank, 1, local, False)
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kwargs = {}
    if backend == "nccl":
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(
        backend=backend, rank=rank, world_size=world,
        timeout=datetime.timedelta(seconds=timeout_s), **kwargs,
    )
    return DistInfo(rank, world, local, True)


def _reduce_device(info: DistInfo) -> torch.device:
    if dist.is_initialized() and dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def max_over_ranks(value: float, info: DistInfo) -> float:
    if not info.initialized:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_reduce_device(info))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, info: DistInfo) -> float:
    if not info.initialized:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_reduce_device(info))
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(info: DistInfo) -> None:
    if info.initialized:
        dist.barrier()


def gather_shards(x: torch.Tensor, total: int, info: DistInfo, dst: int = 0):
    """Gather each rank's contiguous shard ``x`` (leading dim) of a ``total`` batch.

    Returns the full tensor on ``dst`` and None elsewhere. Shards are padded to
    the largest shard so the exchange is one ``all_gather_into_tensor`` (NCCL
    over NVLink between GPUs). Not part of the timed hot path.
    """
    if not info.initialized:
        return x
    per = -(-total // info.world)
    pad = torch.zeros((per, *x.shape[1:]), dtype=x.dtype, device=x.device)
    pad[: x.shape[0]] = x
    out = torch.empty((per * info.world, *x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, pad)
    if info.rank != dst:
        return None
    parts = []
    for r in range(info.world):
        s, e = shard_range(total, r, info.world)
        parts.append(out[r * per : r * per + (e - s)])
    return torch.cat(parts, 0)


def run_sharded(fn, A_full: torch.Tensor, info: DistInfo):
    """Factor this rank's shard of ``A_full`` with ``fn`` -> (start, end, H, tau)."""
    s, e = shard_range(A_full.shape[0], info.rank, info.world)
    H, tau = fn(A_full[s:e])
    return s, e, H, tau


def destroy(info: DistInfo) -> None:
    if info.initialized and dist.is_initialized():
        dist.destroy_process_group()
