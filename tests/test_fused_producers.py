"""The reference-shaped adaLN producers with the quant fused in
(taomate_hd_b200.fused_kernels; reference fused_kernels.py:723-797).

CPU: argument errors as the reference raises them, and the wrappers'
plumbing (flattening, returned shapes, table handling, the prequantised
linear) through a fake of the operators built from the oracle.
GPU: the real operators against the oracle chain producer -> quant -> GEMM.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w8a8_oracle as orc


def _case(batch, tokens, cols, seed):
    g = torch.Generator().manual_seed(seed)
    bf = lambda *s, sd=1.0: (torch.randn(*s, generator=g) * sd).to(torch.bfloat16)
    return dict(residual=bf(batch, tokens, cols), branch=bf(batch, tokens, cols),
                gate=bf(3, cols, sd=0.5), weight=(1.0 + 0.1 * torch.randn(cols, generator=g))
                .to(torch.bfloat16), scale=bf(3, cols, sd=0.1), shift=bf(3, cols, sd=0.1),
                indices=torch.randint(0, 3, (batch, tokens), generator=g))


def test_index_coverage_errors_match_reference():
    from taomate_hd_b200 import fused_kernels as fk

    c = _case(2, 8, 64, seed=1)
    short = c["indices"].reshape(-1)[:-1]
    with pytest.raises(ValueError, match="do not cover every row"):
        fk.fused_rms_norm_modulate_quant(c["residual"], c["weight"], c["scale"], c["shift"],
                                         short, 1e-6)
    with pytest.raises(ValueError, match="do not cover every row"):
        fk.fused_residual_gate_rms_norm_modulate_quant(
            c["residual"], c["branch"], c["gate"], c["weight"], c["scale"], c["shift"], short,
            1e-6)


def test_wrapper_plumbing_with_oracle_backed_ops(monkeypatch):
    from taomate_hd_b200 import fused_kernels as fk

    seen = {}

    def fake_rg(residual, branch, gate, weight, eps, shift, scale, index, *, return_hidden):
        seen["rg"] = (residual.shape, index.shape, gate.is_contiguous(), scale.is_contiguous())
        value, hidden = orc.residual_gate_rms_norm_modulate(residual, branch, gate, weight, eps,
                                                            shift, scale, index)
        q, s = orc.dynamic_scaled_int8_quant(hidden)
        return (torch.from_numpy(q), torch.from_numpy(s).reshape(-1, 1), value,
                hidden if return_hidden else None)

    def fake_mm(a, b, scale_a, scale_b, out_dtype, bias, *, gelu_tanh, swiglu, out):
        seen["mm"] = (a.shape, b.shape, swiglu)
        y, _ = orc.scaled_mm(a.numpy(), b.t().contiguous().numpy(), scale_a.numpy().reshape(-1),
                             scale_b.numpy().reshape(-1), bias, out_dtype)
        return orc.swiglu(y) if swiglu else y

    monkeypatch.setattr(fk.ops, "residual_gate_rms_norm_modulate_int8_quant", fake_rg)
    monkeypatch.setattr(fk.ops, "scaled_mm", fake_mm)
    c = _case(2, 8, 64, seed=2)
    scale_t = c["scale"].t().contiguous().t()   # a table with stride(-1) != 1
    value, act = fk.fused_residual_gate_rms_norm_modulate_quant(
        c["residual"], c["branch"], c["gate"], c["weight"], scale_t, c["shift"], c["indices"],
        1e-6, return_hidden=True)
    assert seen["rg"] == (torch.Size([16, 64]), torch.Size([16]), True, True)
    assert value.shape == (2, 8, 64) and act.shape == (2, 8, 64) and act.hidden.shape == (2, 8, 64)
    v_ref, h_ref = orc.residual_gate_rms_norm_modulate(
        c["residual"].reshape(16, 64), c["branch"].reshape(16, 64), c["gate"], c["weight"], 1e-6,
        c["shift"], c["scale"], c["indices"].reshape(-1))
    assert torch.equal(value.reshape(16, 64), v_ref)
    wq, ws = orc.quantize_weight(orc.weight(96, 64, seed=3))
    wq_i = fk.ops.interleave_gate_up(torch.from_numpy(wq))
    ws_i = fk.ops.interleave_gate_up(torch.from_numpy(ws))
    y = fk.w8a8_linear_prequantized(act, wq_i, ws_i, swiglu=True)
    assert seen["mm"] == (torch.Size([16, 64]), torch.Size([64, 96]), True)
    assert y.shape == (2, 8, 48)
    with pytest.raises(ValueError):
        fk.w8a8_linear_prequantized(act, wq_i[:, :32], ws_i)


@pytest.mark.gpu
def test_producers_then_prequantized_linear_match_oracle(tm_ops, cuda):
    from taomate_hd_b200 import fused_kernels as fk

    c = _case(2, 64, 1024, seed=4)
    dev = {k: v.to(cuda) for k, v in c.items()}
    value, act = fk.fused_residual_gate_rms_norm_modulate_quant(
        dev["residual"], dev["branch"], dev["gate"], dev["weight"], dev["scale"], dev["shift"],
        dev["indices"], 1e-6, return_hidden=True)
    v_ref, h_ref = orc.residual_gate_rms_norm_modulate(
        c["residual"].reshape(128, 1024), c["branch"].reshape(128, 1024), c["gate"],
        c["weight"], 1e-6, c["shift"], c["scale"], c["indices"].reshape(-1))
    assert torch.equal(value.cpu().reshape(128, 1024), v_ref)
    hidden = act.hidden.cpu().reshape(128, 1024)
    torch.testing.assert_close(hidden.float(), h_ref.float(), atol=1e-2, rtol=1e-2)
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(hidden)
    np.testing.assert_array_equal(act.q.cpu().numpy(), q_ref)
    wq, ws = orc.quantize_weight(orc.weight(512, 1024, seed=5))
    y = fk.w8a8_linear_prequantized(act, torch.from_numpy(wq).to(cuda),
                                    torch.from_numpy(ws).to(cuda))
    ref, _ = orc.scaled_mm(q_ref, wq, s_ref, ws, None, torch.bfloat16)
    assert y.shape == (2, 64, 512)
    torch.testing.assert_close(y.cpu().reshape(128, 512).float(), ref.float(), atol=1e-2,
                               rtol=1e-2)
    act2 = fk.fused_rms_norm_modulate_quant(dev["residual"], dev["weight"], dev["scale"],
                                            dev["shift"], dev["indices"], 1e-6)
    h2_ref = orc.rms_norm_modulate(c["residual"].reshape(128, 1024), c["weight"], 1e-6,
                                   c["shift"], c["scale"], c["indices"].reshape(-1))
    q2_ref, _ = orc.dynamic_scaled_int8_quant(h2_ref)
    # within one int8 step where the RMSNorm output sits one bf16 step away
    assert np.abs(act2.q.cpu().numpy().astype(np.int32) - q2_ref.astype(np.int32)).max() <= 1
