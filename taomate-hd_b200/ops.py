"""Drop-in replacement for the ``vllm._custom_ops`` functions the reference uses.

The reference loads ``vllm._custom_ops`` (src/taomate_hd/inference/w8a8.py:76-86)
and calls ``scaled_int8_quant`` and ``cutlass_scaled_mm``
(src/taomate_hd/inference/w8a8.py:141-144); its workspace calls the
out-variant operators ``torch.ops._C.dynamic_scaled_int8_quant`` and
``torch.ops._C.cutlass_scaled_mm`` (w8a8.py:22-35, :71-72).  This module
exposes the same two functions with the same signatures, return values and
error behaviour, backed by ``torch.ops.taomate_w8a8`` (hand-written sm_100a
kernels), plus the fused variants this package adds.  Every function
requires CUDA tensors: there is no CPU path.
"""
from __future__ import annotations

import torch

from ._native import load_torch_ops

load_torch_ops()
_ops = torch.ops.taomate_w8a8

EPI_GELU_TANH = 0x1
EPI_SWIGLU = 0x2


def _require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("taomate_hd_b200 ops require CUDA tensors (there is no CPU path)")


def scaled_int8_quant(
    input: torch.Tensor,
    scale: torch.Tensor | None = None,
    azp: torch.Tensor | None = None,
    symmetric: bool = True,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """Quantise ``input`` to int8; returns ``(int8, scales, None)``.

    ``scale is None``: dynamic per-token symmetric quantisation, scales shaped
    ``[numel // input.shape[-1], 1]`` (vLLM ``scaled_int8_quant``, the call at
    w8a8.py:141).  Otherwise static per-tensor quantisation with ``scale``.
    Asymmetric quantisation (``azp`` / ``symmetric=False``) is not used by the
    reference and raises.
    """
    _require_cuda(input, scale)
    if azp is not None or not symmetric:
        raise NotImplementedError("asymmetric int8 quantisation is not supported")
    output = torch.empty_like(input, dtype=torch.int8)
    if scale is not None:
        _ops.static_scaled_int8_quant(output, input, scale, None)
        return output, scale, None
    input_scales = torch.empty(
        (input.numel() // input.shape[-1], 1), device=input.device, dtype=torch.float32
    )
    _ops.dynamic_scaled_int8_quant(output, input.contiguous(), input_scales, None)
    return output, input_scales, None


def cutlass_scaled_mm(
    a: torch.Tensor,
    b: torch.Tensor,
    scale_a: torch.Tensor,
    scale_b: torch.Tensor,
    out_dtype: torch.dtype,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """``out = (scale_a * a) @ (scale_b * b)`` in ``out_dtype`` (+ bias).

    ``a``: int8 ``[..., K]``; ``b``: int8 ``[K, N]`` column-major (the
    ``weight.t()`` view of an ``[N, K]`` weight); ``scale_a`` per-tensor or
    per-token fp32; ``scale_b`` per-tensor or per-channel fp32 (w8a8.py:142-144).
    Requires K and N to be multiples of 16 (vLLM's CUTLASS contract); vLLM's
    Triton fallback for other shapes is not provided.
    """
    _require_cuda(a, b, scale_a, scale_b, bias)
    if out_dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("out_dtype must be torch.bfloat16 or torch.float16")
    if bias is not None and (bias.numel() != b.shape[1] or bias.dtype != out_dtype):
        raise ValueError("bias must have b.shape[1] elements of out_dtype")
    if b.shape[0] % 16 or b.shape[1] % 16:
        raise ValueError("cutlass_scaled_mm requires K and N to be multiples of 16")
    target_shape = (*a.shape[:-1], b.shape[1])
    a2 = a.view(-1, a.shape[-1])
    out = torch.empty((a2.shape[0], b.shape[1]), dtype=out_dtype, device=a.device)
    _ops.cutlass_scaled_mm(out, a2, b, scale_a, scale_b, bias)
    return out.view(*target_shape)


def scaled_mm(
    a: torch.Tensor,
    b: torch.Tensor,
    scale_a: torch.Tensor,
    scale_b: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: torch.Tensor | None = None,
    *,
    gelu_tanh: bool = False,
    swiglu: bool = False,
    out: torch.Tensor | None = None,
    acc_debug: torch.Tensor | None = None,
    tile_n: int = 0,
) -> torch.Tensor:
    """:func:`cutlass_scaled_mm` with the fused epilogue options.

    ``gelu_tanh`` applies ``round(gelu_tanh(round(y)))`` to the dequantised
    (+bias) output.  ``swiglu`` expects ``b``'s N columns as interleaved
    (gate, up) blocks (:func:`interleave_gate_up`) and returns ``[M, N / 2]``
    ``round(round(g * sigmoid(g)) * u)`` (the reference's fused_swiglu after
    the merged fc1).  ``acc_debug`` (int32 ``[M, N]``) receives the raw
    accumulators; ``out`` makes the call allocation-free; ``tile_n`` forces
    the N-tile width (0 = heuristic).
    """
    _require_cuda(a, b, scale_a, scale_b, bias, out, acc_debug)
    if gelu_tanh and swiglu:
        raise ValueError("gelu_tanh and swiglu are exclusive")
    a2 = a.reshape(-1, a.shape[-1])
    if out is None:
        cols = b.shape[1] // 2 if swiglu else b.shape[1]
        out = torch.empty((a2.shape[0], cols), dtype=out_dtype, device=a.device)
    epi = (EPI_GELU_TANH if gelu_tanh else 0) | (EPI_SWIGLU if swiglu else 0)
    _ops.scaled_mm_i8_ex(out, a2, b, scale_a, scale_b, bias, epi, acc_debug, tile_n)
    return out


def interleave_gate_up(t: torch.Tensor, block: int = 16) -> torch.Tensor:
    """Reorder a merged ``[gate; up]`` tensor (rows, or a 1-D vector) into the
    SwiGLU epilogue's layout: ``block`` gate rows, then the matching ``block``
    up rows, repeated.  Per-row quantisation commutes with the reordering, so
    int8 weights and their scales can be interleaved before or after it."""
    rows = t.shape[0]
    if rows % (2 * block):
        raise ValueError(f"rows ({rows}) must be a multiple of {2 * block}")
    half = rows // 2
    gate = t[:half].reshape(half // block, block, *t.shape[1:])
    up = t[half:].reshape(half // block, block, *t.shape[1:])
    return torch.stack((gate, up), dim=1).reshape(t.shape).contiguous()


def scaled_mm_lora(
    a: torch.Tensor,
    b: torch.Tensor,
    scale_a: torch.Tensor,
    scale_b: torch.Tensor,
    lora_t: torch.Tensor,
    lora_b: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    bias: torch.Tensor | None = None,
    *,
    gelu_tanh: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """:func:`scaled_mm` plus a BF16 LoRA delta added in the epilogue.

    ``lora_t`` is ``x A^T`` (bf16 ``[M, r]``, r <= 64, a multiple of 8) and
    ``lora_b`` the adapter's B already multiplied by its scale (bf16
    ``[N, r]``); the result is ``epi(dequant(a b) (+bias) + lora_t lora_b^T)``
    with the update added in fp32 and rounded once together with the base
    output (GELU, when asked, applies to the sum).
    """
    _require_cuda(a, b, scale_a, scale_b, bias, out, lora_t, lora_b)
    a2 = a.reshape(-1, a.shape[-1])
    if out is None:
        out = torch.empty((a2.shape[0], b.shape[1]), dtype=out_dtype, device=a.device)
    _ops.scaled_mm_i8_lora(out, a2, b, scale_a, scale_b, bias, lora_t, lora_b,
                           EPI_GELU_TANH if gelu_tanh else 0)
    return out


def lora_down_proj(x: torch.Tensor, a: torch.Tensor, *,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """LoRA down-projection ``x @ a.T`` in bf16 (the inner linear of the
    reference's LoRA forward, lora_checkpoint.py:135-136 and 146-147): ``x``
    bf16 ``[..., K]``, ``a`` bf16 ``[r, K]`` with r in {8, 16, ..., 64};
    returns bf16 ``[M, r]`` (fp32 accumulation, one rounding), the
    ``lora_t`` operand of :func:`scaled_mm_lora`.  Row strides must be
    multiples of 8 elements."""
    _require_cuda(x, a, out)
    x2 = x.reshape(-1, x.shape[-1])
    if out is None:
        out = torch.empty((x2.shape[0], a.shape[0]), dtype=torch.bfloat16, device=x.device)
    _ops.lora_down_proj(out, x2, a)
    return out


def quantize_weight_int8(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel symmetric int8 weight conversion on the GPU.

    Bit-exact with ``_quantize_cutlass_w8a8_weight`` (w8a8.py:175-179);
    returns ``(int8 [N, K], fp32 scales [N, 1])``.
    """
    _require_cuda(weight)
    w = weight.contiguous()
    q = torch.empty_like(w, dtype=torch.int8)
    scales = torch.empty((w.shape[0], 1), device=w.device, dtype=torch.float32)
    _ops.quantize_weight_int8(q, scales, w)
    return q, scales


def quantize_weight_int8_into(
    q_out: torch.Tensor,
    scale_out: torch.Tensor,
    source: torch.Tensor,
    *,
    staging_bytes: int = 8 << 20,
) -> None:
    """Convert a ``[N, K]`` weight into preallocated int8 storage, in row chunks.

    For loaders that stream a checkpoint into already-allocated W8 slots (the
    reference's ``load_cutlass_w8a8_stream_weight_``, w8a8.py:207-242): the
    scales are per output row, so converting row chunks gives the same bytes
    as converting the whole matrix.  ``q_out`` is int8 ``[N, K]`` and
    ``scale_out`` fp32 with ``N`` elements, both contiguous on the GPU;
    ``source`` is bf16/fp16/fp32 ``[N, K]`` on the host or the GPU.

    A host source moves through two device staging buffers of at most
    ``staging_bytes`` each: the copy of chunk i+1 runs on a side stream while
    the kernel converts chunk i on the current stream, straight into the
    output rows (no int8 temporary).  A contiguous source already on the
    output's device is converted in one launch.  Stream-ordered; returns
    without synchronising.
    """
    _require_cuda(q_out, scale_out)
    if source.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise TypeError(f"source weight dtype {source.dtype} is not bf16, fp16 or fp32")
    if q_out.dtype != torch.int8 or scale_out.dtype != torch.float32:
        raise TypeError("q_out must be int8 and scale_out float32")
    if source.dim() != 2 or tuple(q_out.shape) != tuple(source.shape):
        raise ValueError(f"source {tuple(source.shape)} and q_out {tuple(q_out.shape)} "
                         "must be the same 2-D shape")
    if scale_out.numel() != source.shape[0]:
        raise ValueError("scale_out needs one element per output row")
    if not (q_out.is_contiguous() and scale_out.is_contiguous()):
        raise ValueError("q_out and scale_out must be contiguous")
    if staging_bytes <= 0:
        raise ValueError("staging_bytes must be positive")
    rows, cols = source.shape
    if rows == 0:
        return
    scales = scale_out.view(-1)
    device = q_out.device
    if source.device == device and source.is_contiguous():
        _ops.quantize_weight_int8(q_out, scales, source)
        return
    row_bytes = cols * source.element_size()
    chunk = max(1, min(rows, staging_bytes // row_bytes))
    staging = [torch.empty((chunk, cols), dtype=source.dtype, device=device) for _ in range(2)]
    main = torch.cuda.current_stream(device)
    side = torch.cuda.Stream(device)
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    for i, start in enumerate(range(0, rows, chunk)):
        stop = min(start + chunk, rows)
        b = i % 2
        dst = staging[b][: stop - start]
        with torch.cuda.stream(side):
            if i >= 2:
                side.wait_event(consumed[b])
            dst.copy_(source[start:stop], non_blocking=True)
            copied[b].record(side)
        main.wait_event(copied[b])
        _ops.quantize_weight_int8(q_out[start:stop], scales[start:stop], dst)
        consumed[b].record(main)
    # The staging buffers belong to the current stream, and their last use
    # is on it (every side-stream copy is waited on before its conversion),
    # so freeing them here is stream-ordered after the last conversion.


def modulate_int8_quant(
    x: torch.Tensor,
    shift: torch.Tensor,
    scale: torch.Tensor,
    index: torch.Tensor | None = None,
    *,
    return_hidden: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """adaLN modulate (fused_kernels.py:220-236) fused into the per-token quant.

    Returns ``(int8 like x, fp32 scales [rows, 1], hidden or None)`` where
    hidden is the bf16 modulated activation.
    """
    _require_cuda(x, shift, scale, index)
    rows = x.numel() // x.shape[-1]
    q = torch.empty_like(x, dtype=torch.int8)
    s = torch.empty((rows, 1), device=x.device, dtype=torch.float32)
    hidden = torch.empty_like(x) if return_hidden else None
    _ops.modulate_int8_quant(q, s, hidden, x, shift, scale, index)
    return q, s, hidden


def rms_norm_modulate_int8_quant(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    shift: torch.Tensor,
    scale: torch.Tensor,
    index: torch.Tensor | None = None,
    *,
    return_hidden: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """RMSNorm + adaLN modulate (fused_kernels.py:322-347) fused into the quant."""
    _require_cuda(x, weight, shift, scale, index)
    rows = x.numel() // x.shape[-1]
    q = torch.empty_like(x, dtype=torch.int8)
    s = torch.empty((rows, 1), device=x.device, dtype=torch.float32)
    hidden = torch.empty_like(x) if return_hidden else None
    _ops.rms_norm_modulate_int8_quant(q, s, hidden, x, weight, float(eps), shift, scale, index)
    return q, s, hidden


def residual_gate_rms_norm_modulate_int8_quant(
    residual: torch.Tensor,
    branch: torch.Tensor,
    gate: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    shift: torch.Tensor,
    scale: torch.Tensor,
    index: torch.Tensor | None = None,
    *,
    return_hidden: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor | None]:
    """``fused_residual_gate_rms_norm_modulate`` (fused_kernels.py:349-382,
    757-797) fused into the quant: returns the int8 rows and scales of the
    modulated hidden state, the updated residual ``bf16(residual +
    bf16(gate[t] * branch))`` and, if asked, the modulated hidden state."""
    _require_cuda(residual, branch, gate, weight, shift, scale, index)
    rows = residual.numel() // residual.shape[-1]
    q = torch.empty_like(residual, dtype=torch.int8)
    s = torch.empty((rows, 1), device=residual.device, dtype=torch.float32)
    residual_out = torch.empty_like(residual)
    hidden = torch.empty_like(residual) if return_hidden else None
    _ops.residual_gate_rms_norm_modulate_int8_quant(
        q, s, residual_out, hidden, residual, branch, gate, weight, float(eps), shift, scale, index)
    return q, s, residual_out, hidden
