"""Distributed context — the reference's ``moe_bench/context.py`` contract (NCCL path only).

``DistContext(rank, world_size, local_rank, device, group, nvshmem_initialized)``
(``context.py:9-20``); ``init_context`` reads ``RANK``/``WORLD_SIZE``/``LOCAL_RANK``,
initialises NCCL when world_size > 1, pins the device and barriers (``:64-88``).
``backend`` and ``timeout_s`` exist so CPU tests can use gloo ranks and so a rank
that dies ends its peers' next collective with an error instead of a hang.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Any


@dataclass(frozen=True)
class DistContext:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    device: Any = "cpu"
    group: Any | None = None
    nvshmem_initialized: bool = False

    @property
    def is_rank0(self) -> bool:
        return self.rank == 0


def init_context(backend: str = "nccl", timeout_s: float = 120.0, device: Any | None = None) -> DistContext:
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world_size > 1 and not dist.is_initialized():
        kwargs = {"backend": backend, "timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local_rank)
        dist.init_process_group(**kwargs)
    if backend == "nccl":
        resolved = torch.device("cuda", local_rank) if device is None else torch.device(device)
        torch.cuda.set_device(resolved)
    else:
        resolved = torch.device("cpu") if device is None else torch.device(device)
    if dist.is_initialized():
        dist.barrier()
    return DistContext(rank=rank, world_size=world_size, local_rank=local_rank, device=resolved)


def finalize_context(ctx: DistContext | None = None) -> None:
    import torch.distributed as dist

    if dist.is_initialized():
        dist.destroy_process_group()
