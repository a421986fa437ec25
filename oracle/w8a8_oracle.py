"""CPU oracle for the selective-W8A8 tensor-parallel DiT linear path.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA path: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  The product package
(``taomate_hd_b200``) never imports or calls anything here.

Each function restates, in numpy (elementwise fp32 arithmetic, IEEE rounding)
and torch-on-CPU (bf16 rounding, exact int32 GEMM via ``torch._int_mm``), the
computation of one step of the reference path:

* activation quant  -> vLLM ``dynamic_scaled_int8_quant`` as called at
  src/taomate_hd/inference/w8a8.py:71 / :141 (third-party: vLLM, pinned by the
  reference at git commit c3a722fcb, README.md:62; its published algorithm is
  per-row amax, scale = amax / 127, q = round_half_even(x * (127 / amax))
  saturated to int8).  Pinned empirically by ``tests/golden/vllm_*.npz``,
  produced on a B200 by ``tests/golden/make_vllm_golden.py`` from the
  installed vLLM 0.22 operators.
* scaled GEMM       -> vLLM ``cutlass_scaled_mm`` (w8a8.py:72, :142-144):
  exact int32 accumulation, then ``scale_a * (scale_b * float(acc)) (+ bias)``.
* weight quant      -> ``_quantize_cutlass_w8a8_weight`` (w8a8.py:175-179),
  pinned against the reference function itself by
  ``tests/golden/reference_host.npz`` (``tests/golden/make_reference_golden.py``).
* adaLN producers   -> ``_modulate_kernel`` (fused_kernels.py:220-236),
  ``_rms_norm_modulate_kernel`` (fused_kernels.py:322-347) and
  ``_residual_gate_rms_norm_modulate_kernel`` (fused_kernels.py:349-382);
  with ``swiglu`` (:298-309), pinned against those Triton kernels run by
  Triton's CPU interpreter (``tests/golden/adaln_triton.npz``,
  ``tests/golden/make_adaln_golden.py``).
* LoRA composition  -> ``H3InferenceParallelLinearLoRA.forward``
  (lora_checkpoint.py:126-154).
* TP sharding       -> ``ColumnParallelLinear`` / ``MergedColumnParallelLinear`` /
  ``RowParallelLinear`` (distributed/linear.py:161-225, :291-296) and the LoRA
  shard helpers (lora_checkpoint.py:73-97).
"""
from __future__ import annotations

import math
from typing import Sequence

import numpy as np
import torch

F32 = np.float32


# ---------------------------------------------------------------- helpers
def to_f32(x: torch.Tensor | np.ndarray) -> np.ndarray:
    """Exact widening of bf16/fp16/fp32 values to a numpy float32 array."""
    if isinstance(x, np.ndarray):
        return x.astype(F32, copy=False)
    return x.detach().to(torch.float32).cpu().numpy()


def round_bf16(v: np.ndarray) -> np.ndarray:
    """Round-half-even to bf16 and back (fused_kernels.py:57-61 ``_round_bf16``)."""
    return torch.from_numpy(np.ascontiguousarray(v, dtype=F32)).to(torch.bfloat16).to(
        torch.float32).numpy()


def to_out_dtype(v: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(v, dtype=F32)).to(dtype)


def sat_round_int8(v: np.ndarray) -> np.ndarray:
    """Saturating round-half-even to int8 (``cvt.rni.sat.s8.f32``; NaN -> 0)."""
    r = np.rint(v.astype(F32))
    r = np.nan_to_num(r, nan=0.0, posinf=127.0, neginf=-128.0)
    return np.clip(r, -128, 127).astype(np.int8)


# ---------------------------------------------------------------- quant
def dynamic_scaled_int8_quant(x: torch.Tensor | np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-token dynamic symmetric int8 quant (vLLM op called at w8a8.py:71).

    Returns ``(q int8 [rows, K], scales float32 [rows])``.  NaN elements do not
    enter the row maximum and quantise to 0; infinities saturate.
    """
    xf = to_f32(x).reshape(-1, np.shape(x)[-1])
    # row maximum of |x| from 0 with NaN elements left out (an fmax
    # reduction; NaN handling is not pinned by golden vectors)
    amax = (np.fmax.reduce(np.abs(xf), axis=1, initial=F32(0.0)).astype(F32)
            if xf.shape[1] else np.zeros(xf.shape[0], F32))
    scales = (amax / F32(127.0)).astype(F32)
    with np.errstate(divide="ignore"):
        inv = np.where(amax == 0, F32(0.0), F32(127.0) / amax).astype(F32)
    q = sat_round_int8(xf * inv[:, None])
    return q, scales


def static_scaled_int8_quant(x: torch.Tensor | np.ndarray, scale: float) -> np.ndarray:
    """Static per-tensor quant: ``sat_int8(round(x / scale))``."""
    xf = to_f32(x).reshape(-1, np.shape(x)[-1])
    return sat_round_int8(xf / F32(scale))


def quantize_weight(w: torch.Tensor | np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-output-channel weight quant (w8a8.py:175-179).

    ``scale = max(amax_row(|W|) / 127, 1e-12)``; ``q = clamp(round(W / scale), -127, 127)``.
    Returns ``(q int8 [N, K], scales float32 [N])``.
    """
    wf = to_f32(w)
    amax = np.max(np.abs(wf), axis=1).astype(F32)
    scales = np.maximum(amax / F32(127.0), F32(1e-12)).astype(F32)
    q = np.clip(np.rint(wf / scales[:, None]), -127, 127).astype(np.int8)
    return q, scales


# ---------------------------------------------------------------- GEMM
def int_mm(a: np.ndarray, b_nk: np.ndarray) -> np.ndarray:
    """Exact int32 ``a[M,K] @ b[N,K]^T`` (no overflow for |int8| products at K < 2^17)."""
    a_t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.int8))
    b_t = torch.from_numpy(np.ascontiguousarray(b_nk, dtype=np.int8))
    if a_t.shape[0] == 0:
        return np.zeros((0, b_t.shape[0]), dtype=np.int32)
    try:
        return torch._int_mm(a_t, b_t.t()).numpy()
    except RuntimeError:
        return (a_t.to(torch.int64) @ b_t.to(torch.int64).t()).to(torch.int32).numpy()


def scaled_mm_epilogue(
    acc: np.ndarray,
    scale_a: np.ndarray,
    scale_b: np.ndarray,
    bias: torch.Tensor | np.ndarray | None,
    out_dtype: torch.dtype = torch.bfloat16,
    gelu: bool = False,
) -> torch.Tensor:
    """``cvt(scale_a[m] * (scale_b[n] * float(acc)) (+ bias[n]))`` (w8a8.py:142-144).

    The bias term is a fused multiply-add: the product is formed exactly in
    float64 and rounded once with the addend.  With ``gelu`` the output is
    ``round(gelu_tanh(round(y)))``.
    """
    accf = acc.astype(F32)
    sa = np.broadcast_to(np.asarray(scale_a, F32).reshape(-1, 1), (acc.shape[0], 1))
    sb = np.asarray(scale_b, F32).reshape(1, -1)
    t = (sb * accf).astype(F32)
    if bias is None:
        y = (sa * t).astype(F32)
    else:
        bf = to_f32(bias).reshape(1, -1)
        y = (sa.astype(np.float64) * t.astype(np.float64) + bf.astype(np.float64)).astype(F32)
    out = to_out_dtype(y, out_dtype)
    if gelu:
        out = torch.nn.functional.gelu(out.to(torch.float32), approximate="tanh").to(out_dtype)
    return out


def scaled_mm(
    a: np.ndarray,
    b_nk: np.ndarray,
    scale_a: np.ndarray,
    scale_b: np.ndarray,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    gelu: bool = False,
) -> tuple[torch.Tensor, np.ndarray]:
    """Full ``cutlass_scaled_mm``: returns ``(out, int32 accumulators)``."""
    acc = int_mm(a, b_nk)
    return scaled_mm_epilogue(acc, scale_a, scale_b, bias, out_dtype, gelu), acc


def w8a8_linear(
    x: torch.Tensor,
    w_q: np.ndarray,
    w_scale: np.ndarray,
    bias: torch.Tensor | None = None,
    gelu: bool = False,
) -> torch.Tensor:
    """``cutlass_w8a8_linear`` (w8a8.py:117-145): flatten, quant, scaled GEMM, reshape."""
    shape = (*x.shape[:-1], int(w_q.shape[0]))
    q, s = dynamic_scaled_int8_quant(x.reshape(-1, x.shape[-1]))
    out, _ = scaled_mm(q, w_q, s, w_scale, bias, torch.bfloat16, gelu)
    return out.reshape(shape)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.gelu(x.to(torch.float32), approximate="tanh").to(x.dtype)


def swiglu(value: torch.Tensor) -> torch.Tensor:
    """``fused_swiglu`` (fused_kernels.py:298-309, 694-704): gate, up = halves;
    ``round_bf16(round_bf16(gate * sigmoid(gate)) * up)`` in fp32."""
    v = to_f32(value).reshape(-1, value.shape[-1])
    half = v.shape[1] // 2
    gate, up = v[:, :half], v[:, half:]
    with np.errstate(over="ignore"):
        sig = (F32(1.0) / (F32(1.0) + np.exp(-gate).astype(F32))).astype(F32)
    act = round_bf16((gate * sig).astype(F32))
    out = round_bf16((act * up).astype(F32))
    return torch.from_numpy(out).to(torch.bfloat16).reshape(*value.shape[:-1], half)


# ---------------------------------------------------------------- adaLN producers
def modulate(
    x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, index: torch.Tensor | None = None
) -> torch.Tensor:
    """``bf16(bf16(x * bf16(1 + scale[t])) + shift[t])`` (fused_kernels.py:220-236)."""
    xf = to_f32(x).reshape(-1, x.shape[-1])
    rows = np.arange(xf.shape[0]) if index is None else index.cpu().numpy()
    sc = to_f32(scale)[rows]
    sh = to_f32(shift)[rows]
    m = round_bf16(xf * round_bf16(F32(1.0) + sc))
    h = round_bf16(m + sh)
    return torch.from_numpy(h).to(torch.bfloat16).reshape(x.shape)


def rms_norm_modulate(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    shift: torch.Tensor,
    scale: torch.Tensor,
    index: torch.Tensor | None = None,
) -> torch.Tensor:
    """RMSNorm then modulate (fused_kernels.py:322-347).

    ``n = bf16(x * rsqrt(mean(x^2) + eps) * w)`` with the mean accumulated in
    float64 and rounded to fp32, then ``1 / sqrt(var + eps)`` as two IEEE fp32
    steps (square root, then reciprocal), as the reference's Triton kernel
    evaluates it under the interpreter (pinned by ``adaln_triton.npz``).
    """
    xf = to_f32(x).reshape(-1, x.shape[-1])
    var = (xf.astype(np.float64) ** 2).mean(axis=1)
    rinv = (1.0 / np.sqrt(var.astype(F32) + F32(eps))).astype(F32)
    n = round_bf16((xf * rinv[:, None]).astype(F32) * to_f32(weight)[None, :])
    return modulate(torch.from_numpy(n).to(torch.bfloat16).reshape(x.shape), shift, scale, index)


def residual_gate_rms_norm_modulate(
    residual: torch.Tensor,
    branch: torch.Tensor,
    gate: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    shift: torch.Tensor,
    scale: torch.Tensor,
    index: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``_residual_gate_rms_norm_modulate_kernel`` (fused_kernels.py:349-382):
    ``x = bf16(residual + bf16(gate[t] * branch))`` (returned as the new
    residual), then :func:`rms_norm_modulate` of ``x``."""
    rf = to_f32(residual).reshape(-1, residual.shape[-1])
    bf = to_f32(branch).reshape(rf.shape)
    rows = np.arange(rf.shape[0]) if index is None else index.cpu().numpy()
    gt = to_f32(gate)[rows]
    x = round_bf16(rf + round_bf16(gt * bf))
    x_t = torch.from_numpy(x).to(torch.bfloat16).reshape(residual.shape)
    return x_t, rms_norm_modulate(x_t, weight, eps, shift, scale, index)


# ---------------------------------------------------------------- LoRA
def lora_column(
    base_out: torch.Tensor, x: torch.Tensor, a: torch.Tensor, b: torch.Tensor, scale: float
) -> torch.Tensor:
    """Column LoRA (lora_checkpoint.py:144-154): ``y + bf16(bf16(x A^T) B^T) * scale``."""
    dt = base_out.dtype
    update = torch.nn.functional.linear(
        torch.nn.functional.linear(x.to(dt), a.to(dt)), b.to(dt))
    return base_out + update * scale


def merged_qkv_send_layout(value: torch.Tensor, num_heads: int, head_dim: int,
                           world: int) -> torch.Tensor:
    """The send buffer of ``merged_qkv_sequence_to_heads`` (distributed/
    ulysses.py:166-204, ``_merged_qkv_send_layout`` :153-163):
    ``[tokens, 3 * heads * head_dim]`` -> ``[world, 3, tokens, local, head_dim]``,
    local = ceil(heads / world); when ``world`` does not divide ``heads`` the
    heads are first padded with zero heads (:188-193)."""
    tokens = value.shape[0]
    packed = value.reshape(tokens, 3, num_heads, head_dim)
    padding = -num_heads % world
    if padding:
        packed = torch.nn.functional.pad(packed, (0, 0, 0, padding))
    local = (num_heads + padding) // world
    return (packed.reshape(tokens, 3, world, local, head_dim)
            .permute(2, 1, 0, 3, 4).contiguous())


# ---------------------------------------------------------------- TP sharding
def column_shard(full: torch.Tensor, tp_size: int, tp_rank: int) -> torch.Tensor:
    """``ColumnParallelLinear.full_weight_slice`` (linear.py:161-166)."""
    n = full.shape[0] // tp_size
    return full.narrow(0, tp_rank * n, n).contiguous()


def merged_column_shard(
    full: torch.Tensor, output_sizes: Sequence[int], tp_size: int, tp_rank: int
) -> torch.Tensor:
    """``MergedColumnParallelLinear.full_weight_slice`` (linear.py:207-215)."""
    pieces, offset = [], 0
    for size in output_sizes:
        local = size // tp_size
        pieces.append(full.narrow(0, offset + tp_rank * local, local))
        offset += size
    return torch.cat(pieces, dim=0).contiguous()


def row_shard(full: torch.Tensor, tp_size: int, tp_rank: int) -> torch.Tensor:
    """``RowParallelLinear.full_weight_slice`` / ``_row_local_a`` (linear.py:291-296)."""
    k = full.shape[1] // tp_size
    return full.narrow(1, tp_rank * k, k).contiguous()


# ---------------------------------------------------------------- synthetic inputs
def activation(
    rows: int, cols: int, seed: int, outlier_channels: int | None = None, outlier_scale: float = 20.0
) -> torch.Tensor:
    """bf16 ~N(0,1) activations with a few outlier channels scaled by ``outlier_scale``.

    ``outlier_channels=None`` uses 0.1% of the channels (at least one).
    """
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g, dtype=torch.float32)
    count = max(1, math.ceil(cols * 0.001)) if outlier_channels is None else outlier_channels
    if count:
        idx = torch.randperm(cols, generator=g)[:count]
        x[:, idx] *= outlier_scale
    return x.to(torch.bfloat16)


def weight(n: int, k: int, seed: int, std: float = 0.02) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)
