"""Tensor-parallel LoRA over the (W8A8) parallel linears.

Mirrors the inference LoRA bank of src/taomate_hd/inference/lora_checkpoint.py:

* ``canonical_h3_lora_targets`` (lora_checkpoint.py:10-17)
* ``column_local_b`` / ``row_local_a`` (lora_checkpoint.py:73-97): LoRA-B of a
  merged column linear is sharded per logical projection; LoRA-A of a row
  linear is sliced along K.
* ``ParallelLinearLoRA`` (``H3InferenceParallelLinearLoRA``,
  lora_checkpoint.py:115-154): ``y = base(x) + bf16(bf16(x A^T) B^T) * scale``;
  for row-parallel bases with ``fused_row_reduce_enabled`` the update is added
  to the partial before the single TP reduction.
* ``apply_lora_state`` (``apply_h3_lora_checkpoint``, lora_checkpoint.py:100-204)
  from an in-memory state mapping (checkpoint file loading is out of scope).
* ``materialize_lora_bf16_buffers_`` / ``enable_fused_lora_row_reduce_``
  (lora_checkpoint.py:207-247).
"""
from __future__ import annotations

from typing import Any, Mapping

import torch

from . import collectives
from .linear import MergedColumnParallelLinear, RowParallelLinear

LORA_TARGET_SUFFIXES = ("attn.qkv_proj", "attn.out_proj", "mlp.fc1", "mlp.fc2")


class LoRAError(RuntimeError):
    pass


def canonical_h3_lora_targets(refiner_blocks: int = 2, blocks: int = 50) -> tuple[str, ...]:
    names = [f"token_refiner.blocks.{i}" for i in range(refiner_blocks)]
    names += [f"blocks.{i}" for i in range(blocks)]
    return tuple(f"{block}.{suffix}" for block in names for suffix in LORA_TARGET_SUFFIXES)


def _tp_coordinates(module: Any) -> tuple[int, int]:
    size, rank = int(module.tp_size), int(module.tp_rank)
    if size <= 0 or rank < 0 or rank >= size:
        raise LoRAError("LoRA TP coordinates are invalid")
    return size, rank


def column_local_b(full_b: torch.Tensor, module: Any) -> torch.Tensor:
    """Per-projection shard of LoRA-B for a merged column linear."""
    size, rank = _tp_coordinates(module)
    pieces, offset = [], 0
    for raw in module.output_sizes:
        width = int(raw)
        if width % size:
            raise LoRAError("merged-column LoRA output is not TP-divisible")
        shard = width // size
        pieces.append(full_b.narrow(0, offset + rank * shard, shard))
        offset += width
    if offset != int(full_b.shape[0]):
        raise LoRAError("merged-column LoRA output inventory differs")
    return torch.cat(pieces, dim=0).contiguous()


def row_local_a(full_a: torch.Tensor, module: Any) -> torch.Tensor:
    """K-slice of LoRA-A for a row-parallel linear."""
    size, rank = _tp_coordinates(module)
    width = int(full_a.shape[1])
    if width % size:
        raise LoRAError("row LoRA input is not TP-divisible")
    shard = width // size
    return full_a.narrow(1, rank * shard, shard).contiguous()


class ParallelLinearLoRA(torch.nn.Module):
    """LoRA adapter around a TP linear (lora_checkpoint.py:115-154)."""

    def __init__(self, base: Any, *, kind: str, a: torch.Tensor, b: torch.Tensor, scale: float):
        super().__init__()
        if kind not in ("column", "row"):
            raise LoRAError("kind must be 'column' or 'row'")
        self.base = base
        self.kind = kind
        self.scale = float(scale)
        self.fused_row_reduce_enabled = False
        self._taomate_hd_inference_lora = True
        self.register_buffer("lora_a", a, persistent=False)
        self.register_buffer("lora_b", b, persistent=False)

    def _update(self, inputs: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        return torch.nn.functional.linear(
            torch.nn.functional.linear(inputs.to(dtype), self.lora_a.to(dtype)),
            self.lora_b.to(dtype))

    def forward(self, inputs: torch.Tensor) -> torch.Tensor:
        if self.kind == "row" and self.fused_row_reduce_enabled and int(self.base.tp_size) > 1:
            partial = self.base.forward_local(inputs)
            update = self._update(inputs, partial.dtype)
            output = self.base.reduce_local_output(partial + update * self.scale)
            if self.base.bias is not None:
                output = output + self.base.bias
            return output
        output = self.base(inputs)
        update = self._update(inputs, output.dtype)
        if self.kind == "row" and int(self.base.tp_size) > 1:
            update = collectives.tp_all_reduce(update, context=self.base.parallel_context)
        if tuple(update.shape) != tuple(output.shape):
            raise LoRAError("LoRA output shape differs")
        return output + update * self.scale


def apply_lora_state(
    transformer: torch.nn.Module,
    state: Mapping[str, torch.Tensor],
    *,
    rank: int,
    alpha: float,
    targets: tuple[str, ...] | None = None,
) -> dict[str, Any]:
    """Wrap every target linear with a TP-sharded ``ParallelLinearLoRA``."""
    targets = canonical_h3_lora_targets() if targets is None else targets
    modules = dict(transformer.named_modules())
    scale = float(alpha) / int(rank)
    plans = []
    local_numel = 0
    for target in targets:
        module = modules.get(target)
        if type(module) is MergedColumnParallelLinear:
            if bool(getattr(module, "gather_output", False)):
                raise LoRAError("gathered column output is not qualified")
            kind = "column"
        elif type(module) is RowParallelLinear:
            kind = "row"
        else:
            raise LoRAError(f"LoRA target type differs: {target}")
        full_a, full_b = state[f"{target}.lora_a"], state[f"{target}.lora_b"]
        if int(full_a.shape[1]) != int(module.input_size) or int(full_b.shape[0]) != int(module.output_size):
            raise LoRAError(f"LoRA full shape differs: {target}")
        device = module.weight.device
        if kind == "column":
            a = full_a.to(device=device, dtype=torch.float32)
            b = column_local_b(full_b, module).to(device=device, dtype=torch.float32)
        else:
            a = row_local_a(full_a, module).to(device=device, dtype=torch.float32)
            b = full_b.to(device=device, dtype=torch.float32)
        if int(a.shape[1]) != int(module.weight.shape[1]) or int(b.shape[0]) != int(module.weight.shape[0]):
            raise LoRAError(f"LoRA local shape differs: {target}")
        plans.append((target, module, ParallelLinearLoRA(module, kind=kind, a=a, b=b, scale=scale).eval()))
        local_numel += int(a.numel() + b.numel())
    for target, expected, replacement in plans:
        parent = transformer
        parts = target.split(".")
        for part in parts[:-1]:
            parent = getattr(parent, part)
        if getattr(parent, parts[-1]) is not expected:
            raise LoRAError(f"LoRA target changed: {target}")
        setattr(parent, parts[-1], replacement)
    return {
        "rank": int(rank),
        "alpha": float(alpha),
        "scale": scale,
        "target_count": len(plans),
        "local_adapter_numel": local_numel,
        "tensor_parallel_size": int(plans[0][1].tp_size) if plans else 1,
    }


def materialize_lora_bf16_buffers_(transformer: torch.nn.Module) -> dict[str, Any]:
    adapters = [m for m in transformer.modules() if getattr(m, "_taomate_hd_inference_lora", False)]
    if not adapters:
        raise LoRAError("BF16 LoRA buffers require a loaded adapter")
    converted = 0
    for module in adapters:
        for name in ("lora_a", "lora_b"):
            value = getattr(module, name)
            if value.dtype != torch.bfloat16:
                converted += int(value.numel())
                setattr(module, name, value.to(dtype=torch.bfloat16))
    return {"target_count": len(adapters), "buffer_count": 2 * len(adapters),
            "converted_numel": converted, "dtype": "bfloat16"}


def enable_fused_lora_row_reduce_(transformer: torch.nn.Module) -> dict[str, Any]:
    rows = [m for m in transformer.modules()
            if getattr(m, "_taomate_hd_inference_lora", False) and getattr(m, "kind", None) == "row"]
    if not rows:
        raise LoRAError("fused row reduction requires a loaded adapter")
    for module in rows:
        module.fused_row_reduce_enabled = True
    return {"row_parallel_module_count": len(rows), "tp_all_reduce_calls_saved_per_forward": len(rows)}
