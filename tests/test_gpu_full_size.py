"""GPU parity at the BASELINE configurations' full sizes.

The CPU oracle is too slow for full-size GEMMs, so these use properties that
hold at any size:

* int32 accumulators are exact, so the kernel's (acc_debug) must equal
  cuBLAS's int8 GEMM (``torch._int_mm``) element for element at the 480p MLP
  and 768p QKV shapes, through whichever tile configuration the heuristic
  picks;
* the activation quant is checked bit-exact against the oracle on a full
  480p fc1 input (numpy handles 25 M elements in seconds);
* the dequant epilogue is linear in the token scale: doubling ``scale_a``
  doubles every bf16 output exactly (a power-of-two factor commutes with
  fp32 and bf16 rounding while nothing overflows);
* the bf16 outputs of the full-size linears (bias, GELU) are compared with
  the oracle on a sample of rows: the oracle's exact int32 GEMM and fp32
  epilogue handle a few hundred rows in seconds.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w8a8_oracle as orc

pytestmark = pytest.mark.gpu


def _int8(shape, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randint(-127, 128, shape, generator=g, device=device, dtype=torch.int8)


@pytest.mark.parametrize("m,n,k", [
    (8192, 12288, 3072),   # 480p fc1
    (8192, 3072, 12288),   # 480p fc2
    (20480, 9216, 3072),   # 768p merged QKV
])
def test_full_size_accumulators_match_cublas_int8(tm_ops, cuda, m, n, k):
    a = _int8((m, k), m + k, cuda)
    b = _int8((n, k), n + k, cuda)
    sa = torch.ones(m, 1, device=cuda)
    sb = torch.ones(1, n, device=cuda)
    acc = torch.empty(m, n, dtype=torch.int32, device=cuda)
    tm_ops.scaled_mm(a, b.t(), sa, sb, torch.bfloat16, acc_debug=acc)
    ref = torch._int_mm(a, b.t())
    torch.cuda.synchronize()
    assert torch.equal(acc, ref)


def test_full_size_quant_bit_exact(tm_ops, cuda):
    x = orc.activation(8192, 3072, seed=11, outlier_channels=3).to(torch.bfloat16)
    q, s, _ = tm_ops.scaled_int8_quant(x.to(cuda))
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(x)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("gelu", [False])
def test_full_size_epilogue_linear_in_token_scale(tm_ops, cuda, gelu):
    m, n, k = 8192, 12288, 3072
    a = _int8((m, k), 5, cuda)
    b = _int8((n, k), 6, cuda)
    g = torch.Generator(device=cuda).manual_seed(7)
    sa = torch.rand(m, 1, generator=g, device=cuda) * 1e-3 + 1e-5
    sb = torch.rand(1, n, generator=g, device=cuda) * 1e-3 + 1e-5
    y1 = tm_ops.scaled_mm(a, b.t(), sa, sb, torch.bfloat16, gelu_tanh=gelu)
    y2 = tm_ops.scaled_mm(a, b.t(), sa * 2, sb, torch.bfloat16, gelu_tanh=gelu)
    torch.cuda.synchronize()
    assert torch.equal(y2.float(), y1.float() * 2)


@pytest.mark.parametrize("m,n,k,gelu", [
    (8192, 12288, 3072, True),    # 480p fc1, bias + GELU-tanh
    (8192, 3072, 12288, False),   # 480p fc2, bias
    (20480, 9216, 3072, False),   # 768p merged QKV, bias
])
def test_full_size_bf16_outputs_match_oracle_on_sampled_rows(tm_ops, cuda, m, n, k, gelu):
    x = orc.activation(m, k, seed=m + n)
    w = orc.weight(n, k, seed=n + k)
    g = torch.Generator().manual_seed(k)
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    q, s, _ = tm_ops.scaled_int8_quant(x.to(cuda))
    wq, ws = tm_ops.quantize_weight_int8(w.to(cuda))
    y = tm_ops.scaled_mm(q, wq.t(), s, ws.t(), torch.bfloat16, bias.to(cuda), gelu_tanh=gelu)
    torch.cuda.synchronize()
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(x)
    wq_ref, ws_ref = orc.quantize_weight(w)
    # rows on both sides of the first and last 128 / 256-row tile edges,
    # plus a random sample
    idx = np.unique(np.concatenate([
        np.array([0, 1, 127, 128, 255, 256, m - 257, m - 256, m - 1]),
        torch.randperm(m, generator=g)[:320].numpy()]))
    ref, _ = orc.scaled_mm(q_ref[idx], wq_ref, s_ref[idx], ws_ref, bias, torch.bfloat16, gelu)
    torch.testing.assert_close(y.cpu()[idx].float(), ref.float(), atol=1e-2, rtol=1e-2)
