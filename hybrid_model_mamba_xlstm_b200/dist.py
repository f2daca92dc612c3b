"""Data-parallel plumbing for the hot path: one process per GPU.

The recurrent workloads shard over independent units — (batch row, channel)
for the selective scan, (batch, head) for mLSTM / SSD / sLSTM, batch rows for
the hybrid prefill — so no collective sits on the data path.  NCCL (over
NVLink / NVSwitch) is used only around the timed region: a barrier, the
max-over-ranks reduction of device times, and all-gathers of output shards
(``gather_rows``) or per-rank figures for verification after timing.  Every function works with the ``gloo``
backend on CPU tensors as well, which is how the multi-rank logic is tested.
"""
from __future__ import annotations

import datetime
import os
from typing import Tuple

import torch
import torch.distributed as dist


def env_world() -> Tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment (1, 0, 0 without it)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str = "nccl", timeout_s: float = 120.0):
    """Initialise the default process group from the environment (no-op for world 1).
    Returns (world, rank, device)."""
    world, rank, local = env_world()
    if backend == "nccl":
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
    else:
        device = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        kw = dict(timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(backend, **kw)
    return world, rank, device


def shard_range(n_units: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) share of n_units for `rank` (remainder spread over the first ranks)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, rem = divmod(n_units, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def _tensor_device():
    if dist.is_initialized() and dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def barrier(world: int):
    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    """The slowest rank's value (times are taken on each rank's device)."""
    if world == 1:
        return float(x)
    t = torch.tensor([x], dtype=torch.float64, device=_tensor_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_checksums(values, world: int):
    """All-gather a short float64 vector of per-rank output checksums -> (world, k)."""
    v = torch.as_tensor(values, dtype=torch.float64).reshape(-1).to(_tensor_device())
    if world == 1:
        return v.reshape(1, -1).cpu()
    out = [torch.empty_like(v) for _ in range(world)]
    dist.all_gather(out, v)
    return torch.stack(out).cpu()


def gather_rows(t: torch.Tensor, n_rows: int, world: int) -> torch.Tensor:
    """All-gather row shards (dim 0) cut by ``shard_range(n_rows, world, rank)``
    into the full (n_rows, ...) tensor on every rank, in rank order.  Shards
    of unequal size are padded to the largest for the collective."""
    if world == 1:
        return t
    per = max(b - a for a, b in (shard_range(n_rows, world, r) for r in range(world)))
    buf = t.new_zeros((per,) + tuple(t.shape[1:]))
    buf[:t.shape[0]] = t
    out = t.new_empty((world * per,) + tuple(t.shape[1:]))
    dist.all_gather_into_tensor(out, buf.contiguous())
    parts = [out[r * per:r * per + (b - a)] for r, (a, b) in enumerate(shard_range(n_rows, world, r) for r in range(world))]
    return torch.cat(parts, 0)


def checksum(t: torch.Tensor):
    """Order-independent checksum of a tensor: (sum, sum of squares, max |x|) in float64."""
    x = t.detach().double()
    return [float(x.sum()), float((x * x).sum()), float(x.abs().max()) if x.numel() else 0.0]


def finalize(world: int):
    if world > 1 and dist.is_initialized():
        dist.destroy_process_group()
