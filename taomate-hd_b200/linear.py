"""Tensor-parallel linears with the W8A8 dispatch.

Mirrors src/taomate_hd/distributed/linear.py:

* ``linear_dispatch`` (``_linear``, linear.py:43-68): a module carrying
  ``_cutlass_w8a8_weight_scale`` runs the W8A8 path on the sm_100a kernels;
  otherwise ``F.linear`` (BF16).  The reference's FP8 alternative
  (linear.py:69-110, unused by its CLI) is not provided and raises.
* ``ColumnParallelLinear`` (linear.py:113-173): local N = N / t, no collective
  unless ``gather_output``.
* ``MergedColumnParallelLinear`` (linear.py:176-225): each logical projection
  (Q, K, V / gate, up) is sharded separately; the local weight is the
  concatenation of the per-projection shards.
* ``RowParallelLinear`` (linear.py:228-296): local K = K / t; the partial
  output is summed over the TP group (all-reduce, optionally in place), then
  the bias is added.  For W8A8 the per-token activation scale covers the
  local K slice only (the activation is quantised after slicing), so int8
  results depend on the TP degree exactly as in the reference.
"""
from __future__ import annotations

from typing import Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .collectives import tp_all_gather, tp_all_reduce, tp_all_reduce_inplace_
from .parallel import ParallelContext, current_parallel_context


def linear_dispatch(
    inputs: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    fp8_weight_scale: torch.Tensor | None = None,
    cutlass_w8a8_weight_scale: torch.Tensor | None = None,
    cutlass_w8a8_workspace: object | None = None,
    cutlass_w8a8_weight_t: torch.Tensor | None = None,
    cutlass_w8a8_weight_scale_t: torch.Tensor | None = None,
) -> torch.Tensor:
    if cutlass_w8a8_weight_scale is not None:
        if fp8_weight_scale is not None:
            raise RuntimeError("a linear cannot combine CUTLASS W8A8 with another quantizer")
        from .w8a8 import cutlass_w8a8_linear

        return cutlass_w8a8_linear(
            torch, inputs, weight, cutlass_w8a8_weight_scale, bias=bias,
            workspace=cutlass_w8a8_workspace, weight_t=cutlass_w8a8_weight_t,
            weight_scale_t=cutlass_w8a8_weight_scale_t,
        )
    if fp8_weight_scale is not None:
        raise NotImplementedError("the FP8 linear path is outside this package's scope")
    return F.linear(inputs, weight, bias)


_linear = linear_dispatch


def _w8a8_args(module: nn.Module) -> tuple:
    return (
        getattr(module, "_fp8_weight_scale", None),
        getattr(module, "_cutlass_w8a8_weight_scale", None),
        getattr(module, "_cutlass_w8a8_workspace", None),
        getattr(module, "_cutlass_w8a8_weight_t", None),
        getattr(module, "_cutlass_w8a8_weight_scale_t", None),
    )


class ColumnParallelLinear(nn.Module):
    """Output-column sharded linear (linear.py:113-173)."""

    def __init__(
        self,
        input_size: int,
        output_size: int,
        *,
        bias: bool,
        gather_output: bool,
        dtype: torch.dtype,
        weight_requires_grad: bool = True,
        context: ParallelContext | None = None,
        device: torch.device | str | None = None,
    ) -> None:
        super().__init__()
        self.parallel_context = context or current_parallel_context()
        self.input_size = int(input_size)
        self.output_size = int(output_size)
        self.tp_size = self.parallel_context.tp_world_size
        self.tp_rank = self.parallel_context.tp_rank
        self.gather_output = bool(gather_output)
        if self.output_size % self.tp_size:
            raise ValueError(f"column output {self.output_size} is not divisible by TP={self.tp_size}")
        self.local_output_size = self.output_size // self.tp_size
        self.weight = nn.Parameter(
            torch.empty(self.local_output_size, self.input_size, dtype=dtype, device=device),
            requires_grad=weight_requires_grad,
        )
        self.bias = (
            nn.Parameter(torch.empty(self.local_output_size, dtype=dtype, device=device))
            if bias else None
        )

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        output = linear_dispatch(inputs, self.weight, self.bias, *_w8a8_args(self))
        if self.gather_output:
            output = tp_all_gather(output, context=self.parallel_context)
        return output

    def full_weight_slice(self, value: torch.Tensor) -> torch.Tensor:
        if tuple(value.shape) != (self.output_size, self.input_size):
            raise ValueError("full column-parallel weight shape differs")
        return value.narrow(0, self.tp_rank * self.local_output_size,
                            self.local_output_size).contiguous()

    def full_bias_slice(self, value: torch.Tensor) -> torch.Tensor:
        if tuple(value.shape) != (self.output_size,):
            raise ValueError("full column-parallel bias shape differs")
        return value.narrow(0, self.tp_rank * self.local_output_size,
                            self.local_output_size).contiguous()


class MergedColumnParallelLinear(ColumnParallelLinear):
    """Column sharding applied to each fused logical projection (linear.py:176-225)."""

    def __init__(
        self,
        input_size: int,
        output_sizes: Sequence[int],
        *,
        bias: bool,
        gather_output: bool,
        dtype: torch.dtype,
        weight_requires_grad: bool = True,
        context: ParallelContext | None = None,
        device: torch.device | str | None = None,
    ) -> None:
        self.output_sizes = tuple(int(v) for v in output_sizes)
        if not self.output_sizes or any(v <= 0 for v in self.output_sizes):
            raise ValueError("merged column output sizes must be positive")
        ctx = context or current_parallel_context()
        if any(v % ctx.tp_world_size for v in self.output_sizes):
            raise ValueError("every merged output must be divisible by TP")
        super().__init__(input_size, sum(self.output_sizes), bias=bias,
                         gather_output=gather_output, dtype=dtype,
                         weight_requires_grad=weight_requires_grad, context=ctx, device=device)
        self.local_output_sizes = tuple(v // self.tp_size for v in self.output_sizes)

    def _merged_slice(self, value: torch.Tensor) -> torch.Tensor:
        pieces, offset = [], 0
        for size, local in zip(self.output_sizes, self.local_output_sizes):
            pieces.append(value.narrow(0, offset + self.tp_rank * local, local))
            offset += size
        return torch.cat(pieces, dim=0).contiguous()

    def full_weight_slice(self, value: torch.Tensor) -> torch.Tensor:
        if tuple(value.shape) != (self.output_size, self.input_size):
            raise ValueError("full merged-column weight shape differs")
        return self._merged_slice(value)

    def full_bias_slice(self, value: torch.Tensor) -> torch.Tensor:
        if tuple(value.shape) != (self.output_size,):
            raise ValueError("full merged-column bias shape differs")
        return self._merged_slice(value)


class RowParallelLinear(nn.Module):
    """Input-row sharded linear with summed TP partial outputs (linear.py:228-296)."""

    def __init__(
        self,
        input_size: int,
        output_size: int,
        *,
        bias: bool,
        input_is_parallel: bool,
        dtype: torch.dtype,
        weight_requires_grad: bool = True,
        context: ParallelContext | None = None,
        device: torch.device | str | None = None,
    ) -> None:
        super().__init__()
        self.parallel_context = context or current_parallel_context()
        self.input_size = int(input_size)
        self.output_size = int(output_size)
        self.tp_size = self.parallel_context.tp_world_size
        self.tp_rank = self.parallel_context.tp_rank
        self.input_is_parallel = bool(input_is_parallel)
        self.inference_inplace_reduce_enabled = False
        if self.input_size % self.tp_size:
            raise ValueError(f"row input {self.input_size} is not divisible by TP={self.tp_size}")
        self.local_input_size = self.input_size // self.tp_size
        self.weight = nn.Parameter(
            torch.empty(self.output_size, self.local_input_size, dtype=dtype, device=device),
            requires_grad=weight_requires_grad,
        )
        self.bias = (
            nn.Parameter(torch.empty(self.output_size, dtype=dtype, device=device)) if bias else None
        )

    def forward_local(self, inputs: torch.Tensor) -> torch.Tensor:
        """This rank's partial output, before the reduction and the bias."""
        local = inputs if self.input_is_parallel else inputs.narrow(
            -1, self.tp_rank * self.local_input_size, self.local_input_size)
        return linear_dispatch(local, self.weight, None, *_w8a8_args(self))

    def reduce_local_output(self, output: torch.Tensor) -> torch.Tensor:
        if self.inference_inplace_reduce_enabled and not torch.is_grad_enabled():
            return tp_all_reduce_inplace_(output, context=self.parallel_context)
        return tp_all_reduce(output, context=self.parallel_context)

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        output = self.reduce_local_output(self.forward_local(inputs))
        if self.bias is not None:
            output = output + self.bias
        return output

    def full_weight_slice(self, value: torch.Tensor) -> torch.Tensor:
        if tuple(value.shape) != (self.output_size, self.input_size):
            raise ValueError("full row-parallel weight shape differs")
        return value.narrow(1, self.tp_rank * self.local_input_size,
                            self.local_input_size).contiguous()
