"""Tensor-parallel reductions over ``torch.distributed`` (NCCL on GPUs).

Mirrors src/taomate_hd/distributed/collectives.py:9-78 (all-reduce with and
without a clone, all-gather-concat, the ``tp_*`` helpers bound to the current
``ParallelContext``) and adds the row-split reduce-scatter used by the
row-parallel fc2 of the BASELINE configuration.  NCCL is the measured
baseline for the row-parallel reduction; :mod:`taomate_hd_b200.peer_reduce`
holds the fused peer-memory path.
"""
from __future__ import annotations

import os
from contextlib import contextmanager, nullcontext
from typing import Any, Iterator

import torch

from .parallel import ParallelContext, current_parallel_context

_NVTX = os.environ.get("H3_PROFILE_NVTX", "0") == "1"


@contextmanager
def _nvtx(name: str) -> Iterator[None]:
    """NVTX range gated by ``H3_PROFILE_NVTX=1`` (inference/profiling.py:7-22)."""
    if not _NVTX or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def _require_distributed(world_size: int, group: Any | None, name: str) -> Any:
    if world_size == 1:
        return None
    if not torch.distributed.is_available() or not torch.distributed.is_initialized():
        raise RuntimeError(f"{name} collective requires initialized torch.distributed")
    if group is None:
        raise RuntimeError(f"{name} process group is absent")
    return group


def all_reduce_sum(value: torch.Tensor, *, group: Any, world_size: int) -> torch.Tensor:
    """Sum over the group into a fresh tensor (collectives.py:19-30)."""
    _require_distributed(world_size, group, "all-reduce")
    if world_size == 1:
        return value
    if torch.is_grad_enabled() and value.requires_grad:
        from torch.distributed.nn.functional import all_reduce

        return all_reduce(value, group=group)
    with _nvtx(f"collective.all_reduce.world{world_size}"):
        output = value.clone()
        torch.distributed.all_reduce(output, group=group)
    return output


def all_reduce_sum_inplace_(value: torch.Tensor, *, group: Any, world_size: int) -> torch.Tensor:
    """Sum over the group in place (collectives.py:33-40)."""
    _require_distributed(world_size, group, "all-reduce")
    if world_size == 1:
        return value
    with _nvtx(f"collective.all_reduce_inplace.world{world_size}"):
        torch.distributed.all_reduce(value, group=group)
    return value


def all_gather_concat(value: torch.Tensor, *, dim: int, group: Any, world_size: int) -> torch.Tensor:
    """Gather every rank's tensor and concatenate along ``dim`` (collectives.py:43-57)."""
    _require_distributed(world_size, group, "all-gather")
    if world_size == 1:
        return value
    if torch.is_grad_enabled() and value.requires_grad:
        from torch.distributed.nn.functional import all_gather

        gathered = all_gather(value, group=group)
    else:
        with _nvtx(f"collective.all_gather.world{world_size}"):
            gathered = [torch.empty_like(value) for _ in range(world_size)]
            torch.distributed.all_gather(gathered, value.contiguous(), group=group)
    return torch.cat(tuple(gathered), dim=dim)


def reduce_scatter_rows(
    value: torch.Tensor, *, group: Any, world_size: int, out: torch.Tensor | None = None
) -> torch.Tensor:
    """Sum ``value [M, ...]`` over the group; rank r keeps rows [r*M/t, (r+1)*M/t).

    Requires ``M % world_size == 0``.  No reference counterpart: the
    reference only all-reduces (collectives.py:19-40); the BASELINE fc2 is
    row-parallel with a reduce-scatter.
    """
    _require_distributed(world_size, group, "reduce-scatter")
    if world_size == 1:
        return value if out is None else out.copy_(value)
    rows = value.shape[0]
    if rows % world_size:
        raise ValueError(f"reduce-scatter rows {rows} not divisible by {world_size}")
    if out is None:
        out = torch.empty((rows // world_size, *value.shape[1:]), dtype=value.dtype,
                          device=value.device)
    with _nvtx(f"collective.reduce_scatter.world{world_size}"):
        torch.distributed.reduce_scatter_tensor(out, value.contiguous(), group=group)
    return out


def tp_all_reduce(value: torch.Tensor, context: ParallelContext | None = None) -> torch.Tensor:
    context = context or current_parallel_context()
    return all_reduce_sum(value, group=context.tp_group, world_size=context.tp_world_size)


def tp_all_reduce_inplace_(
    value: torch.Tensor, context: ParallelContext | None = None
) -> torch.Tensor:
    context = context or current_parallel_context()
    return all_reduce_sum_inplace_(value, group=context.tp_group, world_size=context.tp_world_size)


def tp_all_gather(
    value: torch.Tensor, *, dim: int = -1, context: ParallelContext | None = None
) -> torch.Tensor:
    context = context or current_parallel_context()
    return all_gather_concat(value, dim=dim, group=context.tp_group,
                             world_size=context.tp_world_size)


def tp_reduce_scatter_rows(
    value: torch.Tensor, context: ParallelContext | None = None, out: torch.Tensor | None = None
) -> torch.Tensor:
    context = context or current_parallel_context()
    return reduce_scatter_rows(value, group=context.tp_group, world_size=context.tp_world_size,
                               out=out)


def nvtx_range(name: str):
    """Public NVTX helper (no-op unless ``H3_PROFILE_NVTX=1``)."""
    return _nvtx(name) if _NVTX else nullcontext()
