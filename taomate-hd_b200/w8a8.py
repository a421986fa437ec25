"""Selective-W8A8 operator adapter on the sm_100a kernels.

Mirrors src/taomate_hd/inference/w8a8.py with the vLLM operators replaced by
``torch.ops.taomate_w8a8`` (see :mod:`taomate_hd_b200.ops`):

* ``CutlassW8A8Workspace``          w8a8.py:12-73  grow-only per-stream buffers
* ``require_vllm_cutlass_w8a8``     w8a8.py:76-86  backend loader (returns ``ops``)
* ``resolve_h3_cutlass_w8a8_policy`` w8a8.py:89-114 interior QKV/FC1 selection
* ``cutlass_w8a8_linear``           w8a8.py:117-145 quant + scaled GEMM
* ``enable_h3_cutlass_w8a8_workspace_`` w8a8.py:148-172
* ``quantize_cutlass_w8a8_weight``  w8a8.py:175-179 (GPU kernel, bit-exact)
* streamed W8 loading               w8a8.py:182-242
* ``quantize_h3_interior_qkv_fc1_linears_cutlass_w8a8_`` w8a8.py:245-336

Function names, arguments, return values, receipts and error types follow the
reference so a caller can switch by changing the import.
"""
from __future__ import annotations

from typing import Any

INTERIOR_FC1_QKV_CUTLASS_W8A8_POLICY = "interior_fc1_qkv_v1"
H3_CUTLASS_W8A8_POLICIES = (INTERIOR_FC1_QKV_CUTLASS_W8A8_POLICY,)
STREAM_LOAD_TEMPORARY_BYTES = 8 * 1024 * 1024

_PROJECTION_SUFFIXES = (".attn.qkv_proj", ".mlp.fc1", ".mlp.fc2")
_ELIGIBLE_SUFFIXES = (".attn.qkv_proj", ".mlp.fc1")


class CutlassW8A8Workspace:
    """Reusable int8 / scale / output buffers, one set per (device, stream, width).

    Like the reference workspace (w8a8.py:12-73) the output buffer is reused
    across calls on a stream: a caller must consume it (enqueue its readers)
    before the next projection of the same width on that stream.  Buffers only
    grow.  Both operators run out-of-place into these buffers, so a call
    allocates nothing once the buffers reached their size.
    """

    def __init__(self, torch: Any) -> None:
        from . import ops  # noqa: F401  (registers torch.ops.taomate_w8a8)

        namespace = getattr(getattr(torch, "ops", None), "taomate_w8a8", None)
        dynamic_quant = getattr(namespace, "dynamic_scaled_int8_quant", None)
        scaled_mm = getattr(namespace, "cutlass_scaled_mm", None)
        if not callable(dynamic_quant) or not callable(scaled_mm):
            raise RuntimeError(
                "W8A8 workspace requires the taomate_w8a8 dynamic INT8 quant and scaled-mm operators"
            )
        self._torch = torch
        self._dynamic_quant = dynamic_quant
        self._scaled_mm = scaled_mm
        self._activation: dict[tuple[Any, ...], tuple[Any, Any]] = {}
        self._outputs: dict[tuple[Any, ...], Any] = {}

    def _stream_key(self, inputs: Any) -> tuple[Any, ...]:
        device = inputs.device
        if device.type != "cuda":
            return (device.type, device.index, 0)
        return (device.type, device.index, int(self._torch.cuda.current_stream(device).cuda_stream))

    def _activation_buffers(self, inputs: Any, key: tuple[Any, ...]) -> tuple[Any, Any]:
        rows, width = int(inputs.shape[0]), int(inputs.shape[1])
        slot = (*key, width)
        held = self._activation.get(slot)
        if held is None or int(held[0].shape[0]) < rows:
            held = (
                self._torch.empty((rows, width), device=inputs.device, dtype=self._torch.int8),
                self._torch.empty((rows, 1), device=inputs.device, dtype=self._torch.float32),
            )
            self._activation[slot] = held
        return held[0][:rows], held[1][:rows]

    def _output_buffer(self, inputs: Any, width: int, key: tuple[Any, ...]) -> Any:
        rows = int(inputs.shape[0])
        slot = (*key, int(width))
        held = self._outputs.get(slot)
        if held is None or int(held.shape[0]) < rows:
            held = self._torch.empty((rows, int(width)), device=inputs.device,
                                     dtype=self._torch.bfloat16)
            self._outputs[slot] = held
        return held[:rows]

    def linear(self, inputs: Any, weight_t: Any, weight_scale: Any) -> Any:
        key = self._stream_key(inputs)
        quantized, activation_scale = self._activation_buffers(inputs, key)
        output = self._output_buffer(inputs, int(weight_t.shape[1]), key)
        self._dynamic_quant(quantized, inputs, activation_scale, None)
        self._scaled_mm(output, quantized, weight_t, activation_scale, weight_scale, None)
        return output


def require_vllm_cutlass_w8a8() -> Any:
    """Return the W8A8 backend module (drop-in for w8a8.py:76-86).

    The reference imports ``vllm._custom_ops``; this returns
    :mod:`taomate_hd_b200.ops`, which exposes the same ``scaled_int8_quant``
    and ``cutlass_scaled_mm``.  Raises ``RuntimeError`` when the native
    extension is unavailable.
    """
    try:
        from . import ops
    except Exception as exc:  # the extension is missing or stale
        raise RuntimeError("W8A8 requires the taomate_hd_b200 CUDA extension") from exc
    for name in ("scaled_int8_quant", "cutlass_scaled_mm"):
        if not callable(getattr(ops, name, None)):
            raise RuntimeError(f"taomate_hd_b200 operators are missing {name}")
    return ops


require_w8a8_backend = require_vllm_cutlass_w8a8


def _block_index(name: str) -> int:
    return int(name.split(".", 2)[1])


def resolve_h3_cutlass_w8a8_policy(linear_names: list[str], *, policy: str) -> dict[str, Any]:
    """Pick the interior QKV/FC1 projections for W8A8 (w8a8.py:89-114).

    Among ``blocks.<i>.{attn.qkv_proj, mlp.fc1, mlp.fc2}`` names, the first two
    and last three block indices stay BF16; of the rest, QKV and FC1 are
    quantised and FC2 stays BF16.
    """
    if policy not in H3_CUTLASS_W8A8_POLICIES:
        raise ValueError("unsupported H3 CUTLASS W8A8 policy")
    candidates = [name for name in linear_names if name.endswith(_PROJECTION_SUFFIXES)]
    if not candidates:
        raise ValueError("H3 CUTLASS W8A8 policy requires projection candidates")
    blocks = sorted({_block_index(name) for name in candidates})
    boundary = tuple((*blocks[:2], *blocks[-3:]))
    chosen = [
        name for name in candidates
        if name.endswith(_ELIGIBLE_SUFFIXES) and _block_index(name) not in boundary
    ]
    chosen_set = set(chosen)
    return {
        "policy": policy,
        "quantized_linear_names": chosen,
        "bf16_protected_linear_names": [n for n in candidates if n not in chosen_set],
        "bf16_boundary_block_indices": list(boundary),
    }


def cutlass_w8a8_linear(
    torch: Any,
    inputs: Any,
    weight: Any,
    weight_scale: Any,
    *,
    bias: Any | None,
    workspace: CutlassW8A8Workspace | None = None,
    weight_t: Any | None = None,
    weight_scale_t: Any | None = None,
) -> Any:
    """Dynamic per-token A8 x per-channel W8 linear (w8a8.py:117-145).

    ``inputs [..., K]`` bf16, ``weight [N, K]`` int8, ``weight_scale [N, 1]``
    fp32; returns bf16 ``[..., N]``.  Bias is rejected as in the reference;
    :func:`w8a8_linear_fused` is the bias / GELU-capable entry.
    """
    if bias is not None:
        raise RuntimeError("H3 CUTLASS W8A8 currently supports bias-free linears")
    shape = (*inputs.shape[:-1], int(weight.shape[0]))
    flat = inputs.reshape(-1, int(inputs.shape[-1])).contiguous()
    w_t = weight.t() if weight_t is None else weight_t
    s_t = weight_scale.t() if weight_scale_t is None else weight_scale_t
    if workspace is not None:
        return workspace.linear(flat, w_t, s_t).reshape(shape)
    backend = require_vllm_cutlass_w8a8()
    quantized, activation_scale, _ = backend.scaled_int8_quant(flat)
    output = backend.cutlass_scaled_mm(quantized, w_t, activation_scale, s_t, torch.bfloat16)
    return output.reshape(shape)


def w8a8_linear_fused(
    inputs: Any,
    weight: Any,
    weight_scale: Any,
    *,
    bias: Any | None = None,
    gelu_tanh: bool = False,
    out: Any | None = None,
) -> Any:
    """W8A8 linear with the bias and GELU-tanh fused into the GEMM epilogue.

    Extends :func:`cutlass_w8a8_linear` for the BASELINE fc1 (bias + GELU);
    with neither option it computes the same values.
    """
    from . import ops

    shape = (*inputs.shape[:-1], int(weight.shape[0]))
    flat = inputs.reshape(-1, int(inputs.shape[-1]))
    quantized, activation_scale, _ = ops.scaled_int8_quant(flat)
    y = ops.scaled_mm(quantized, weight.t(), activation_scale, weight_scale.reshape(1, -1),
                      bias=bias, gelu_tanh=gelu_tanh, out=out)
    return y.reshape(shape)


def enable_h3_cutlass_w8a8_workspace_(torch: Any, transformer: Any) -> dict[str, Any]:
    """Attach one shared stream-aware workspace to every W8 linear (w8a8.py:148-172)."""
    require_vllm_cutlass_w8a8()
    modules = [
        (name, module) for name, module in transformer.named_modules()
        if name.startswith("blocks.") and getattr(module, "_cutlass_w8a8_weight_scale", None) is not None
    ]
    if not modules:
        raise RuntimeError("CUTLASS W8A8 workspace requires quantized H3 linears")
    workspace = CutlassW8A8Workspace(torch)
    for _, module in modules:
        module._cutlass_w8a8_workspace = workspace
        module._cutlass_w8a8_weight_t = module.weight.t()
        module._cutlass_w8a8_weight_scale_t = module._cutlass_w8a8_weight_scale.t()
    return {
        "schema": "taomate_hd.inference.cutlass_w8a8_workspace.v1",
        "linear_count": len(modules),
        "workspace_count_per_rank": 1,
        "allocation_policy": "grow_only_per_cuda_stream_and_shape",
        "activation_quantization": "unchanged_dynamic_per_token_symmetric",
        "weight_quantization": "unchanged_static_per_output_channel_symmetric",
        "arithmetic_order_changed": False,
    }


def quantize_cutlass_w8a8_weight(torch: Any, weight: Any) -> tuple[Any, Any]:
    """Per-output-channel symmetric int8 conversion on the GPU (w8a8.py:175-179).

    Bit-exact with the reference's torch expression; returns contiguous
    ``(int8 [N, K], fp32 [N, 1])``.  CPU tensors raise.
    """
    if not weight.is_cuda:
        raise RuntimeError("W8A8 weight conversion runs on the GPU; move the weight to CUDA first")
    from . import ops

    return ops.quantize_weight_int8(weight)


_quantize_cutlass_w8a8_weight = quantize_cutlass_w8a8_weight


def prepare_cutlass_w8a8_stream_load_slot_(torch: Any, module: Any, *, name: str) -> None:
    """Swap an uninitialised BF16 weight for its final int8 storage (w8a8.py:182-204)."""
    if module.weight.dtype not in {torch.bfloat16, torch.int8}:
        raise TypeError(f"{name} expected an uninitialized BF16 or INT8 weight")
    if getattr(module, "bias", None) is not None:
        raise RuntimeError(f"{name} expected a bias-free H3 projection")
    if getattr(module, "_cutlass_w8a8_weight_scale", None) is not None:
        raise RuntimeError(f"{name} already owns CUTLASS W8A8 storage")
    weight = module.weight
    if weight.dtype == torch.bfloat16:
        module.weight = torch.nn.Parameter(
            torch.empty(weight.shape, dtype=torch.int8, device=weight.device), requires_grad=False
        )
    elif weight.requires_grad:
        raise RuntimeError(f"{name} preallocated INT8 weight requires gradients")
    module.register_buffer(
        "_cutlass_w8a8_weight_scale",
        torch.empty((int(weight.shape[0]), 1), dtype=torch.float32, device=weight.device),
        persistent=False,
    )
    module._cutlass_w8a8_stream_load_pending = True
    module._cutlass_w8a8_stream_loaded = False
    module._cutlass_w8a8_source_weight_bytes = int(weight.numel() * 2)


def load_cutlass_w8a8_stream_weight_(
    torch: Any,
    module: Any,
    source_weight: Any,
    *,
    name: str,
    maximum_temporary_bytes: int = STREAM_LOAD_TEMPORARY_BYTES,
) -> None:
    """Quantise a BF16 source into a prepared W8 slot in bounded row chunks (w8a8.py:207-242).

    Scales are per output row, so chunking rows gives exactly the same result
    as converting the whole matrix while holding at most
    ``maximum_temporary_bytes`` of BF16 on the device.
    """
    if getattr(module, "_cutlass_w8a8_stream_load_pending", None) is not True:
        raise RuntimeError(f"{name} has no pending CUTLASS W8A8 stream load")
    if module.weight.dtype != torch.int8 or source_weight.dtype != torch.bfloat16:
        raise TypeError(f"{name} streamed CUTLASS W8A8 dtype differs")
    if tuple(module.weight.shape) != tuple(source_weight.shape):
        raise ValueError(f"{name} streamed CUTLASS W8A8 shape differs")
    if source_weight.ndim != 2:
        raise ValueError(f"{name} streamed CUTLASS W8A8 weight must be 2D")
    if maximum_temporary_bytes <= 0:
        raise ValueError("maximum_temporary_bytes must be positive")
    row_bytes = int(source_weight.shape[1]) * int(source_weight.element_size())
    chunk = max(1, maximum_temporary_bytes // row_bytes)
    rows = int(source_weight.shape[0])
    for start in range(0, rows, chunk):
        stop = min(start + chunk, rows)
        staged = source_weight[start:stop].to(device=module.weight.device, dtype=torch.bfloat16)
        q, s = quantize_cutlass_w8a8_weight(torch, staged)
        module.weight[start:stop].copy_(q)
        module._cutlass_w8a8_weight_scale[start:stop].copy_(s)
    module._cutlass_w8a8_stream_load_pending = False
    module._cutlass_w8a8_stream_loaded = True


def quantize_h3_interior_qkv_fc1_linears_cutlass_w8a8_(
    torch: Any, transformer: Any, *, policy: str
) -> dict[str, Any]:
    """Convert the policy-selected frozen QKV/FC1 base weights to W8 (w8a8.py:245-336)."""
    require_vllm_cutlass_w8a8()
    from .linear import ColumnParallelLinear, RowParallelLinear

    candidates: list[tuple[str, Any]] = []
    for name, module in transformer.named_modules():
        if not name.startswith("blocks.") or not name.endswith(_PROJECTION_SUFFIXES):
            continue
        base = getattr(module, "base", module)
        if isinstance(base, (ColumnParallelLinear, RowParallelLinear)):
            candidates.append((name, base))
    selection = resolve_h3_cutlass_w8a8_policy([n for n, _ in candidates], policy=policy)
    wanted = set(selection["quantized_linear_names"])
    selected = [(n, m) for n, m in candidates if n in wanted]
    if not selected:
        raise RuntimeError("H3 CUTLASS W8A8 policy selected no linears")
    streamed: list[str] = []
    for name, module in selected:
        if getattr(module, "_cutlass_w8a8_weight_scale", None) is not None:
            if (
                module.weight.dtype != torch.int8
                or getattr(module, "_cutlass_w8a8_stream_load_pending", None) is not False
                or getattr(module, "_cutlass_w8a8_stream_loaded", None) is not True
            ):
                raise RuntimeError(f"{name} has incomplete CUTLASS W8A8 storage")
            streamed.append(name)
        elif module.weight.dtype != torch.bfloat16:
            raise TypeError(f"{name} expected BF16 weight before W8A8 conversion")
        if getattr(module, "bias", None) is not None:
            raise RuntimeError(f"{name} expected a bias-free H3 projection")
    eligible_bytes = sum(
        int(getattr(m, "_cutlass_w8a8_source_weight_bytes",
                    m.weight.numel() * m.weight.element_size()))
        for _, m in candidates
    )
    converted: list[str] = []
    source_bytes = quantized_bytes = 0
    for name, module in selected:
        if name in streamed:
            source_bytes += int(module._cutlass_w8a8_source_weight_bytes)
            quantized_bytes += int(module.weight.numel() * module.weight.element_size())
        else:
            weight = module.weight.detach()
            q, s = quantize_cutlass_w8a8_weight(torch, weight)
            source_bytes += int(weight.numel() * weight.element_size())
            quantized_bytes += int(q.numel() * q.element_size())
            module.weight = torch.nn.Parameter(q, requires_grad=False)
            module.register_buffer("_cutlass_w8a8_weight_scale", s, persistent=False)
        converted.append(name)
    return {
        "schema": "taomate_hd.inference.cutlass_w8a8.v1",
        "format": "int8_w8a8",
        "scope": "frozen_main_dit_base_weights_only",
        "policy": policy,
        "projection_set": "interior_qkv_and_fc1",
        "quantized_projection_suffixes": ["attn.qkv_proj", "mlp.fc1"],
        "activation_scale": "dynamic_per_token_symmetric",
        "weight_scale": "static_per_output_channel_symmetric",
        "kernel": "taomate_hd_b200_tcgen05_scaled_mm_i8",
        "eligible_linear_count": len(candidates),
        "linear_count": len(converted),
        "stream_load_linear_count": len(streamed),
        "bf16_protected_linear_count": len(selection["bf16_protected_linear_names"]),
        "quantized_linear_names": converted,
        "bf16_protected_linear_names": selection["bf16_protected_linear_names"],
        "bf16_boundary_block_indices": selection["bf16_boundary_block_indices"],
        "source_weight_bytes": source_bytes,
        "quantized_weight_bytes": quantized_bytes,
        "eligible_source_weight_bytes": eligible_bytes,
        "eligible_weight_fraction": source_bytes / eligible_bytes,
        "bf16_projection_suffixes": ["attn.out_proj", "mlp.fc2"],
        "lora_branch": {"storage": "fp32_online_unmodified", "compute": "bf16"},
        "base_teacher_adapter_bypass": "lora_only",
        "base_teacher_base_precision": "int8_w8a8",
        "runtime_state": "transient_not_checkpoint_reconstructible",
    }
