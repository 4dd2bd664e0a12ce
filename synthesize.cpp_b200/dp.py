"""Data-parallel plumbing for the replica-only multi-GPU path.

Nothing on the Q8_0 path shards: every GPU holds all weights and serves its
own synthesis streams.  This module only splits the streams over ranks,
times with a barrier and takes the max over ranks -- the one collective
(all_reduce MAX of a scalar) the path needs, for measurement.  It works with
any torch.distributed backend (NCCL on the GPU box, gloo in the CPU tests).
"""
from __future__ import annotations

from datetime import timedelta

import torch
import torch.distributed as dist

from .shapes import partition_streams  # noqa: F401  (re-exported: the stream split lives with the workload geometry)


def init(backend: str, timeout_s: float = 300.0, device: torch.device | None = None) -> tuple[int, int]:
    """Initialises the default process group from the torchrun environment; returns (rank, world)."""
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist.get_rank(), dist.get_world_size()


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """The largest `value` over all ranks (the step time every rank reports)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device or torch.device("cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(device: torch.device | None = None) -> None:
    if dist.is_initialized() and dist.get_world_size() > 1:
        if device is not None and device.type == "cuda":
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()
