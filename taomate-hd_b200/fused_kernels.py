"""The reference's adaLN producers with the W8A8 activation quant fused in.

The reference's block forward (src/taomate_hd/model/layers.py:728-766) builds
the attention input with ``fused_rms_norm_modulate`` and the MLP input with
``fused_residual_gate_rms_norm_modulate`` (inference/fused_kernels.py:
723-797); the interior QKV and fc1 linears that consume them are W8A8, so
each producer is followed by ``scaled_int8_quant`` inside
``cutlass_w8a8_linear`` (inference/w8a8.py:117-145).  The functions here take
the reference's arguments in the reference's order, raise its errors, and
return the quantised activation (:class:`QuantizedActivation`) in place of
the bf16 hidden state; :func:`w8a8_linear_prequantized` is the W8A8 linear
that takes it, so the bf16 hidden state never makes a round trip through
HBM between the producer and the GEMM.
"""
from __future__ import annotations

from typing import NamedTuple

import torch

from . import ops


class QuantizedActivation(NamedTuple):
    """Per-token int8 rows of a ``[..., K]`` activation, as ``scaled_int8_quant``
    returns them: ``q`` int8 ``[rows, K]``, ``scale`` fp32 ``[rows, 1]``;
    ``shape`` is the activation's shape; ``hidden`` the bf16 activation
    itself when it was asked for, else None."""

    q: torch.Tensor
    scale: torch.Tensor
    shape: torch.Size
    hidden: torch.Tensor | None = None


def _tables(*tables: torch.Tensor) -> tuple[torch.Tensor, ...]:
    # the reference makes every table contiguous when any last-dimension
    # stride is not 1 (fused_kernels.py:743-745, 773-774)
    if any(t.stride(-1) != 1 for t in tables):
        return tuple(t.contiguous() for t in tables)
    return tables


def fused_rms_norm_modulate_quant(
    value: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    indices: torch.Tensor,
    eps: float,
    *,
    return_hidden: bool = False,
) -> QuantizedActivation:
    """``fused_rms_norm_modulate`` (fused_kernels.py:723-754) followed by the
    dynamic per-token quant, in one pass."""
    shape = value.shape
    flat = value.reshape(-1, shape[-1]).contiguous()
    index = indices.reshape(-1).contiguous()
    if int(index.numel()) != int(flat.shape[0]):
        raise ValueError("SOL RMSNorm/AdaLN indices do not cover every row")
    scale, shift = _tables(scale, shift)
    q, s, hidden = ops.rms_norm_modulate_int8_quant(
        flat, weight.contiguous(), eps, shift, scale, index, return_hidden=return_hidden)
    return QuantizedActivation(q, s, shape, None if hidden is None else hidden.reshape(shape))


def fused_residual_gate_rms_norm_modulate_quant(
    residual: torch.Tensor,
    branch: torch.Tensor,
    gate: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    shift: torch.Tensor,
    indices: torch.Tensor,
    eps: float,
    *,
    return_hidden: bool = False,
) -> tuple[torch.Tensor, QuantizedActivation]:
    """``fused_residual_gate_rms_norm_modulate`` (fused_kernels.py:757-797)
    followed by the dynamic per-token quant, in one pass: returns the updated
    residual stream (the reference's first output) and the quantised
    modulated activation (its second output, quantised)."""
    shape = residual.shape
    columns = shape[-1]
    residual_flat = residual.reshape(-1, columns).contiguous()
    branch_flat = branch.reshape(-1, columns).contiguous()
    index = indices.reshape(-1).contiguous()
    if int(index.numel()) != int(residual_flat.shape[0]):
        raise ValueError("SOL residual/AdaLN indices do not cover every row")
    gate, scale, shift = _tables(gate, scale, shift)
    q, s, value, hidden = ops.residual_gate_rms_norm_modulate_int8_quant(
        residual_flat, branch_flat, gate, weight.contiguous(), eps, shift, scale, index,
        return_hidden=return_hidden)
    return value.reshape(shape), QuantizedActivation(
        q, s, shape, None if hidden is None else hidden.reshape(shape))


def w8a8_linear_prequantized(
    activation: QuantizedActivation,
    weight: torch.Tensor,
    weight_scale: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    gelu_tanh: bool = False,
    swiglu: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """The scaled GEMM of ``cutlass_w8a8_linear`` (w8a8.py:141-144) on an
    activation a producer above already quantised: ``weight`` int8 ``[N, K]``,
    ``weight_scale`` fp32 ``[N, 1]``; returns bf16 ``[..., N]`` (``[..., N/2]``
    with ``swiglu``, whose weight rows are interleaved by
    ``ops.interleave_gate_up``)."""
    if int(activation.q.shape[-1]) != int(weight.shape[-1]):
        raise ValueError("activation width differs from the weight's input width")
    n_out = int(weight.shape[0]) // (2 if swiglu else 1)
    y = ops.scaled_mm(activation.q, weight.t(), activation.scale, weight_scale.reshape(1, -1),
                      torch.bfloat16, bias, gelu_tanh=gelu_tanh, swiglu=swiglu, out=out)
    return y.reshape(*activation.shape[:-1], n_out)
