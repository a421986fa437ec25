"""Rank topology for tensor-parallel execution.

Mirrors ``ParallelContext`` / ``current_parallel_context`` /
``use_parallel_context`` of src/taomate_hd/distributed/parallel.py:9-53: an
explicit, immutable view of this worker's TP (and Ulysses / ring) coordinates
and process groups, installed per worker through a context variable.  Groups
are never inferred here; the runtime that builds them installs the view.
"""
from __future__ import annotations

from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass
from typing import Any, Iterator


@dataclass(frozen=True)
class ParallelContext:
    """This worker's tensor-parallel coordinates (parallel.py:9-35)."""

    tp_world_size: int = 1
    tp_rank: int = 0
    ulysses_world_size: int = 1
    ulysses_rank: int = 0
    ring_world_size: int = 1
    ring_rank: int = 0
    tp_group: Any | None = None
    ulysses_group: Any | None = None

    def __post_init__(self) -> None:
        for axis in ("tp", "ulysses", "ring"):
            size = getattr(self, f"{axis}_world_size")
            rank = getattr(self, f"{axis}_rank")
            if size <= 0 or not 0 <= rank < size:
                raise ValueError(f"invalid {axis} topology: world_size={size}, rank={rank}")
        if self.tp_world_size > 1 and self.tp_group is None:
            raise ValueError("tp_group is required when TP world size exceeds one")
        if self.ulysses_world_size > 1 and self.ulysses_group is None:
            raise ValueError("ulysses_group is required when Ulysses world size exceeds one")


_CURRENT: ContextVar[ParallelContext] = ContextVar(
    "taomate_hd_b200_parallel_context", default=ParallelContext()
)


def current_parallel_context() -> ParallelContext:
    return _CURRENT.get()


@contextmanager
def use_parallel_context(context: ParallelContext) -> Iterator[ParallelContext]:
    if not isinstance(context, ParallelContext):
        raise TypeError("context must be ParallelContext")
    token = _CURRENT.set(context)
    try:
        yield context
    finally:
        _CURRENT.reset(token)
