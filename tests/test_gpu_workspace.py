"""GPU: the operator calls the reference's accelerated mode makes, checked
against the oracle.

Under ``--mode accelerated`` (generate.py:29, ``dit_w8a8_workspace=pipelined``)
every W8A8 linear goes through ``CutlassW8A8Workspace.linear``
(src/taomate_hd/inference/w8a8.py:12-73): per (device, stream, width) it keeps
grow-only int8, scale and bf16 output buffers and passes ``[:rows]`` prefix
views of them to the two out-variant operators, with the weight as
``weight.t()`` and its scales as ``weight_scale.t()``.  Weights reach their
int8 slots through the streamed loader (w8a8.py:182-242), row chunk by row
chunk.  These tests drive ``torch.ops.taomate_w8a8`` and
``ops.quantize_weight_int8_into`` in exactly those forms.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w8a8_oracle as orc

pytestmark = pytest.mark.gpu

TOL = dict(atol=1e-2, rtol=1e-2)  # bf16 output tolerance of the BASELINE parity bar


@pytest.mark.parametrize("n", [3072, 12288])  # configs[0] weight; the 480p fc1 weight
def test_workspace_call_pattern_matches_oracle(tm_ops, cuda, n):
    k = 3072
    w = orc.weight(n, k, seed=n)
    wq, ws = tm_ops.quantize_weight_int8(w.to(cuda))  # [n, k] int8, [n, 1] fp32
    wq_ref, ws_ref = orc.quantize_weight(w)
    q_buf = s_buf = out_buf = None
    # token counts in the order a serving loop might see them: the buffers
    # grow twice and are otherwise reused through prefix views
    for rows in (1024, 64, 1024, 8192 if n == 12288 else 2048, 300):
        if q_buf is None or q_buf.shape[0] < rows:
            q_buf = torch.empty(rows, k, dtype=torch.int8, device=cuda)
            s_buf = torch.empty(rows, 1, dtype=torch.float32, device=cuda)
            out_buf = torch.empty(rows, n, dtype=torch.bfloat16, device=cuda)
        q, s, out = q_buf[:rows], s_buf[:rows], out_buf[:rows]
        x = orc.activation(rows, k, seed=rows + n)
        torch.ops.taomate_w8a8.dynamic_scaled_int8_quant(q, x.to(cuda), s, None)
        torch.ops.taomate_w8a8.cutlass_scaled_mm(out, q, wq.t(), s, ws.t(), None)
        torch.cuda.synchronize()
        q_ref, s_ref = orc.dynamic_scaled_int8_quant(x)
        np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
        np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)
        # the GEMM on up to 512 sampled rows (the oracle's int32 GEMM is exact)
        g = torch.Generator().manual_seed(rows)
        idx = torch.randperm(rows, generator=g)[:512].sort().values.numpy()
        ref, _ = orc.scaled_mm(q_ref[idx], wq_ref, s_ref[idx], ws_ref, None, torch.bfloat16)
        torch.testing.assert_close(out.cpu()[idx].float(), ref.float(), **TOL)


@pytest.mark.parametrize("staging", [8 << 20, 100_000, 1 << 40])
def test_streamed_weight_conversion_bit_exact(tm_ops, cuda, staging):
    """A host bf16 checkpoint tensor converted into preallocated int8 storage
    in row chunks (8 MiB as the reference's default, an odd 100 kB that does
    not divide the rows, and one chunk) equals the whole-matrix conversion."""
    w = orc.weight(12288, 3072, seed=5)
    w[7] = 0.0  # zero row: scale clamps at 1e-12
    q = torch.empty(12288, 3072, dtype=torch.int8, device=cuda)
    s = torch.empty(12288, 1, dtype=torch.float32, device=cuda)
    tm_ops.quantize_weight_int8_into(q, s, w, staging_bytes=staging)
    torch.cuda.synchronize()
    q_ref, s_ref = orc.quantize_weight(w)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)


def test_streamed_weight_conversion_sources(tm_ops, cuda):
    """A device source converts in one launch; a non-contiguous host view
    (a column slice of a wider tensor) goes through the staging buffers."""
    wide = orc.weight(640, 4096, seed=6)
    view = wide[:, 512:3584]  # [640, 3072], row stride 4096
    q = torch.empty(640, 3072, dtype=torch.int8, device=cuda)
    s = torch.empty(640, dtype=torch.float32, device=cuda)
    tm_ops.quantize_weight_int8_into(q, s, view, staging_bytes=3072 * 2 * 100)
    torch.cuda.synchronize()
    q_ref, s_ref = orc.quantize_weight(view.contiguous())
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    q2 = torch.zeros_like(q)
    s2 = torch.zeros_like(s)
    tm_ops.quantize_weight_int8_into(q2, s2, view.contiguous().to(cuda))
    torch.cuda.synchronize()
    assert torch.equal(q2, q) and torch.equal(s2, s)
