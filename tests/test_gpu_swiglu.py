"""GPU parity: SwiGLU fused into the W8A8 fc1 epilogue.

Reference behaviour: the merged fc1 (MergedColumnParallelLinear with
[ffn, ffn] outputs, model/layers.py:502-533) quantised by the W8A8 path
(w8a8.py:117-145), followed by ``fused_swiglu`` (fused_kernels.py:298-309):
``round(round(gate * sigmoid(gate)) * up)``.  The kernel takes the weight rows
interleaved in blocks of 16 (ops.interleave_gate_up) and writes N / 2
columns; compared with the oracle chain within the bf16 tolerance (the
sigmoid uses the hardware exponential).
"""
from __future__ import annotations

import pytest
import torch

from oracle import w8a8_oracle as orc

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 1e-2


def _case(m, ffn, k, seed, bias):
    x = orc.activation(m, k, seed=seed, outlier_channels=max(1, k // 1000))
    w = orc.weight(2 * ffn, k, seed=seed + 1)  # [gate; up]
    g = torch.Generator().manual_seed(seed + 2)
    b = (torch.randn(2 * ffn, generator=g) * 0.01).to(torch.bfloat16) if bias else None
    return x, w, b


@pytest.mark.parametrize("m,ffn,k,bias,tile_n", [
    (256, 768, 1024, False, 0),
    (300, 512, 512, True, 0),      # ragged M, bias
    (2048, 1536, 3072, False, 0),  # CTA-pair path by the heuristic
    (512, 1024, 1024, False, 256),
    (512, 1024, 1024, False, 128),
    (512, 1024, 1024, True, 1256),
    (512, 1024, 1024, False, 1128),
    (64, 1536, 3072, False, 0),    # skinny M (split-K is not used with SwiGLU)
])
def test_swiglu_epilogue_matches_reference(tm_ops, cuda, m, ffn, k, bias, tile_n):
    x, w, b = _case(m, ffn, k, seed=m + ffn + k, bias=bias)
    q, s = orc.dynamic_scaled_int8_quant(x)
    wq, ws = orc.quantize_weight(w)
    projected, _ = orc.scaled_mm(q, wq, s, ws, b, torch.bfloat16)
    ref = orc.swiglu(projected)
    wq_i = tm_ops.interleave_gate_up(torch.from_numpy(wq))
    ws_i = tm_ops.interleave_gate_up(torch.from_numpy(ws))
    b_i = tm_ops.interleave_gate_up(b) if b is not None else None
    got = tm_ops.scaled_mm(
        torch.from_numpy(q).to(cuda), wq_i.to(cuda).t(), torch.from_numpy(s).to(cuda).reshape(-1, 1),
        ws_i.to(cuda).reshape(1, -1), torch.bfloat16, None if b_i is None else b_i.to(cuda),
        swiglu=True, tile_n=tile_n)
    torch.cuda.synchronize()
    assert got.shape == (m, ffn)
    torch.testing.assert_close(got.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)


def test_interleave_layout_and_errors(tm_ops, cuda):
    w = torch.arange(64 * 3).reshape(64, 3)
    wi = tm_ops.interleave_gate_up(w)
    assert torch.equal(wi[:16], w[:16]) and torch.equal(wi[16:32], w[32:48])
    assert torch.equal(wi[32:48], w[16:32]) and torch.equal(wi[48:], w[48:])
    a = torch.zeros(64, 256, dtype=torch.int8, device=cuda)
    b = torch.zeros(96, 256, dtype=torch.int8, device=cuda)  # 96 % 64 != 0
    with pytest.raises(RuntimeError):
        tm_ops.scaled_mm(a, b.t(), torch.ones(1, device=cuda), torch.ones(1, device=cuda),
                         torch.bfloat16, swiglu=True)
    with pytest.raises(ValueError):
        tm_ops.scaled_mm(a, b.t(), torch.ones(1, device=cuda), torch.ones(1, device=cuda),
                         torch.bfloat16, swiglu=True, gelu_tanh=True)
