"""Tensor-parallel process-group state.

One process per GPU; ``torch.distributed`` (NCCL on GPUs, gloo on CPU) is the
bootstrap and the baseline collective path.  Layers query the TP rank and size
from here instead of from the default group, so a TP group can live inside a
larger job (for example several data-parallel replicas under one launcher).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta

import torch
import torch.distributed as dist


@dataclass
class TPState:
    rank: int = 0
    size: int = 1
    group: object | None = None
    backend: str | None = None


_STATE = TPState()


def tp_state() -> TPState:
    return _STATE


def tp_rank() -> int:
    return _STATE.rank


def tp_size() -> int:
    return _STATE.size


def tp_group():
    return _STATE.group


def set_tp_state(rank: int, size: int, group=None, backend: str | None = None) -> None:
    global _STATE
    _STATE = TPState(int(rank), int(size), group, backend)


def init_tp(world_size: int, rank: int, *, backend: str, init_method: str | None = None,
            timeout_minutes: float | None = None) -> None:
    """Join (or create) the default process group and record the TP layout."""
    if timeout_minutes is None:
        timeout_minutes = float(os.environ.get("TORCH_DISTRIBUTED_TIMEOUT_MINUTES", "3"))
    if world_size > 1 and not dist.is_initialized():
        dist.init_process_group(
            backend,
            init_method=init_method,
            world_size=world_size,
            rank=rank,
            timeout=timedelta(minutes=timeout_minutes),
        )
    group = dist.group.WORLD if world_size > 1 else None
    set_tp_state(rank, world_size, group, backend if world_size > 1 else None)


def all_reduce(x: torch.Tensor) -> torch.Tensor:
    if _STATE.size > 1:
        dist.all_reduce(x, group=_STATE.group)
    return x


def broadcast(x: torch.Tensor, src: int = 0) -> torch.Tensor:
    if _STATE.size > 1:
        dist.broadcast(x, src=src, group=_STATE.group)
    return x


def all_gather_last_dim(x: torch.Tensor) -> torch.Tensor:
    if _STATE.size == 1:
        return x
    parts = [torch.empty_like(x) for _ in range(_STATE.size)]
    dist.all_gather(parts, x.contiguous(), group=_STATE.group)
    return torch.cat(parts, dim=-1)


def divide(numerator: int, denominator: int) -> int:
    if numerator % denominator:
        raise ValueError(f"{numerator} is not divisible by {denominator}")
    return numerator // denominator
