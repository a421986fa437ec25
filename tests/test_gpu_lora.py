"""GPU parity: the W8A8 GEMM with the BF16 LoRA delta in its epilogue.

Reference behaviour: ``H3InferenceParallelLinearLoRA.forward``
(src/taomate_hd/inference/lora_checkpoint.py:126-154), column kind:
``output + bf16(bf16(x A^T) B^T) * scale`` on top of the W8A8 linear
(w8a8.py:117-145); BASELINE configs[3] puts the delta in the W8A8 epilogue
and, for fc1, GELU-tanh after it.  The kernel receives T = x A^T and
scale * B and adds T B^T in fp32 onto the rounded base output, rounding once:
compared with the oracle (which rounds the update to bf16 first) within the
bf16 tolerance, with a zero adapter bit-exact against the plain GEMM.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import w8a8_oracle as orc

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 1e-2


def _case(m, n, k, r, seed, b_std=0.002, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = orc.activation(m, k, seed=seed, outlier_channels=max(1, k // 1000))
    w = orc.weight(n, k, seed=seed + 1)
    wq, ws = orc.quantize_weight(w)
    q, s = orc.dynamic_scaled_int8_quant(x)
    a_lora = (torch.randn(r, k, generator=g) * 0.02).to(torch.bfloat16)
    b_lora = (torch.randn(n, r, generator=g) * b_std).to(torch.bfloat16)
    bias_t = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16) if bias else None
    return x, wq, ws, q, s, a_lora, b_lora, bias_t


def _run(tm_ops, cuda, q, s, wq, ws, t, b_scaled, bias, gelu):
    return tm_ops.scaled_mm_lora(
        torch.from_numpy(q).to(cuda), torch.from_numpy(wq).to(cuda).t(),
        torch.from_numpy(s).to(cuda).reshape(-1, 1), torch.from_numpy(ws).to(cuda).reshape(1, -1),
        t.to(cuda), b_scaled.to(cuda), torch.bfloat16,
        None if bias is None else bias.to(cuda), gelu_tanh=gelu).cpu()


@pytest.mark.parametrize("m,n,k,r,b_std", [
    (256, 256, 128, 64, 0.05),
    (512, 768, 1024, 64, 0.05),
    (300, 784, 512, 32, 0.05),     # ragged M and N, rank below the 64-column box
    (1024, 3072, 3072, 64, 0.002),  # BASELINE adapter distribution
    (130, 1536, 256, 8, 0.1),
])
def test_lora_epilogue_matches_reference(tm_ops, cuda, m, n, k, r, b_std):
    """Without an activation the result is the reference composition (1e-2);
    with GELU (BASELINE fc1), GELU-tanh of that same sum (the existing fused
    GELU bar).  The reference rounds the update to bf16 before the add; the
    kernel rounds the fp32 sum once, so pre-activation values may differ by one
    bf16 step, which GELU can widen to two: the activation is therefore checked
    against the kernel's own sum."""
    scale = 1.0  # alpha = r (BASELINE: alpha 64, rank 64)
    x, wq, ws, q, s, a_lora, b_lora, bias = _case(m, n, k, r, seed=m + n + r, b_std=b_std)
    base, _ = orc.scaled_mm(q, wq, s, ws, bias, torch.bfloat16)
    ref = orc.lora_column(base, x, a_lora, b_lora, scale)
    t = torch.nn.functional.linear(x.to(torch.bfloat16), a_lora)  # x A^T, bf16 as the reference
    b_scaled = (b_lora.float() * scale).to(torch.bfloat16)
    got = _run(tm_ops, cuda, q, s, wq, ws, t, b_scaled, bias, False)
    torch.testing.assert_close(got.float(), ref.float(), atol=ATOL, rtol=RTOL)
    got_gelu = _run(tm_ops, cuda, q, s, wq, ws, t, b_scaled, bias, True)
    torch.testing.assert_close(got_gelu.float(), orc.gelu_tanh(got).float(), atol=ATOL, rtol=RTOL)
    # the update really is in the output (not just within tolerance of the base)
    if b_std >= 0.05:
        delta = (got.float() - base.float()).abs().max().item()
        assert delta > 0.05, delta


@pytest.mark.parametrize("gelu", [False, True])
def test_zero_adapter_is_bit_exact_with_plain_gemm(tm_ops, cuda, gelu):
    m, n, k, r = 384, 1280, 768, 64
    x, wq, ws, q, s, a_lora, _, bias = _case(m, n, k, r, seed=7)
    t = torch.nn.functional.linear(x.to(torch.bfloat16), a_lora)
    zero_b = torch.zeros(n, r, dtype=torch.bfloat16)
    got = _run(tm_ops, cuda, q, s, wq, ws, t, zero_b, bias, gelu)
    plain = tm_ops.scaled_mm(
        torch.from_numpy(q).to(cuda), torch.from_numpy(wq).to(cuda).t(),
        torch.from_numpy(s).to(cuda).reshape(-1, 1), torch.from_numpy(ws).to(cuda).reshape(1, -1),
        torch.bfloat16, bias.to(cuda), gelu_tanh=gelu).cpu()
    assert torch.equal(got, plain)


def test_lora_update_in_fp32(tm_ops, cuda):
    """Against an fp32 restatement of what the kernel computes: round(y + T B^T)."""
    m, n, k, r = 512, 512, 256, 64
    x, wq, ws, q, s, a_lora, b_lora, bias = _case(m, n, k, r, seed=11, b_std=0.1)
    base, _ = orc.scaled_mm(q, wq, s, ws, bias, torch.bfloat16)
    t = torch.nn.functional.linear(x.to(torch.bfloat16), a_lora)
    want = (base.float() + t.float() @ b_lora.float().t()).to(torch.bfloat16)
    got = _run(tm_ops, cuda, q, s, wq, ws, t, b_lora, bias, False)
    # fp32 accumulation order differs from the CPU's: at most one bf16 step
    diff = (got.float() - want.float()).abs()
    step = want.float().abs().clamp_min(1e-3) * 2.0 ** -7
    assert bool((diff <= step).all()), float((diff / step).max())


def test_lora_through_c_abi_and_errors(capi, cuda):
    m, n, k, r = 256, 512, 256, 64
    x, wq, ws, q, s, a_lora, b_lora, _ = _case(m, n, k, r, seed=3, b_std=0.05)
    dev = [torch.from_numpy(v).to(cuda) for v in (q, wq, s, ws)]
    t = torch.nn.functional.linear(x.to(torch.bfloat16), a_lora).to(cuda)
    bl = b_lora.to(cuda)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call(rank=r, ldt=r, ldlb=r, t_ptr=None):
        return capi.tm_scaled_mm_i8_lora(
            out.data_ptr(), 0, dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), m,
            dev[3].data_ptr(), n, None, t.data_ptr() if t_ptr is None else t_ptr, ldt,
            bl.data_ptr(), ldlb, rank, m, n, k, k, k, n, 0, stream)

    assert call() == 0
    torch.cuda.synchronize()
    base, _ = orc.scaled_mm(q, wq, s, ws, None, torch.bfloat16)
    ref = orc.lora_column(base, x, a_lora, b_lora, 1.0)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)
    assert call(rank=72, ldt=72, ldlb=72) == 5   # rank above 64
    assert call(rank=12, ldt=64, ldlb=64) == 5   # rank not a multiple of 8
    assert call(ldt=60) == 2                     # row stride below the rank
    assert call(ldt=68, ldlb=64, rank=64) == 3   # row stride not a multiple of 8
    assert call(t_ptr=t.data_ptr() + 8) == 3     # misaligned T
    assert np.isfinite(out.cpu().float().numpy()).all()


@pytest.mark.parametrize("m,k,r,strided", [
    (1, 64, 64, False),
    (300, 1000, 8, False),      # K not a multiple of the 64-column k-block, smallest rank
    (257, 512, 24, True),       # rank between MMA widths; x a column slice of a wider tensor
    (1024, 3072, 48, False),
    (2048, 3072, 64, True),     # the 768p down-projection shape (x = QKV output's Q part)
    (640, 12288, 64, False),    # fc2's K
])
def test_down_projection_matches_fp32_reference(tm_ops, cuda, m, k, r, strided):
    """T = x A^T (lora_checkpoint.py:135-136, 146-147) on the tensor cores
    against a float64 product of the same bf16 operands: one bf16 rounding
    (2^-8 relative) plus an allowance of 2^-16 of sum |x_i a_i| for the
    order of the fp32 additions."""
    g = torch.Generator().manual_seed(m + k + r)
    width = k + 256 if strided else k
    x_full = torch.randn(m, width, generator=g).to(torch.bfloat16)
    x_full[:, 5] *= 20  # an outlier channel, as the DiT activations have
    x = x_full[:, 64:64 + k] if strided else x_full
    a = (torch.randn(r, k, generator=g) * 0.02).to(torch.bfloat16)
    got = tm_ops.lora_down_proj(x.to(cuda) if not strided else x_full.to(cuda)[:, 64:64 + k],
                                a.to(cuda)).cpu()
    assert got.shape == (m, r) and got.dtype == torch.bfloat16
    want = x.double() @ a.double().t()
    mag = x.double().abs() @ a.double().abs().t()
    bound = 2.0 ** -8 * want.abs() + 2.0 ** -16 * mag + 1e-30
    excess = ((got.double() - want).abs() / bound).max().item()
    assert excess <= 1.0, excess


def test_down_projection_through_c_abi_feeds_the_lora_gemm(tm_ops, capi, cuda):
    """The C-ABI call writes T into a strided buffer; the LoRA GEMM fed with
    it matches the oracle composition; calls twice in a row give the same
    bits."""
    m, n, k, r = 384, 512, 768, 64
    x, wq, ws, q, s, a_lora, b_lora, _ = _case(m, n, k, r, seed=21, b_std=0.05)
    xb = x.to(torch.bfloat16).to(cuda)
    al = a_lora.to(cuda)
    t_buf = torch.full((m, r + 16), float("nan"), dtype=torch.bfloat16, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = capi.tm_lora_down_proj(t_buf.data_ptr(), r + 16, xb.data_ptr(), k, al.data_ptr(), k, r,
                                m, k, stream)
    assert rc == 0
    first = t_buf.clone()
    assert capi.tm_lora_down_proj(t_buf.data_ptr(), r + 16, xb.data_ptr(), k, al.data_ptr(), k, r,
                                  m, k, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(first.view(torch.int16), t_buf.view(torch.int16))
    assert torch.isnan(t_buf[:, r:].float()).all()  # columns past the rank untouched
    t = t_buf[:, :r]
    qd, wqd, sd, wsd = (torch.from_numpy(v).to(cuda) for v in (q, wq, s, ws))
    out = tm_ops.scaled_mm_lora(qd, wqd.t(), sd.reshape(-1, 1), wsd.reshape(1, -1), t,
                                b_lora.to(cuda))
    base, _ = orc.scaled_mm(q, wq, s, ws, None, torch.bfloat16)
    ref = orc.lora_column(base, x, a_lora, b_lora, 1.0)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)

