"""CPU: pin the oracle against golden vectors from the reference path itself.

* ``vllm_quant.npz``      vLLM 0.22 ``scaled_int8_quant`` run on a B200
                          (tests/golden/make_vllm_golden.py)
* ``vllm_scaled_mm.npz``  vLLM's scaled GEMM on a B200 (CUTLASS int8 is refused
                          on sm_100, so vLLM's Triton implementation of the op)
* ``reference_host.npz``  the reference's own torch code run on CPU
                          (tests/golden/make_reference_golden.py)
* ``adaln_triton.npz``    the reference's Triton adaLN producers and SwiGLU run
                          by Triton's CPU interpreter
                          (tests/golden/make_adaln_golden.py)
* ``ulysses_send.npz``    the reference's ``merged_qkv_sequence_to_heads``
                          send buffers and outputs, zero-head padding
                          included (tests/golden/make_ulysses_golden.py)
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import w8a8_oracle as orc

from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"


def _tensor(bits: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "torch.bfloat16":
        return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
    if dtype == "torch.float16":
        return torch.from_numpy(bits.view(np.int16).copy()).view(torch.float16)
    return torch.from_numpy(bits.copy())


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return _tensor(bits, "torch.bfloat16")


@pytest.fixture(scope="module")
def vllm_quant():
    return np.load(GOLDEN / "vllm_quant.npz")


@pytest.fixture(scope="module")
def ref_host():
    return np.load(GOLDEN / "reference_host.npz"), json.loads((GOLDEN / "reference_host.json").read_text())


def test_vllm_quant_fixture_provenance(vllm_quant):
    meta = json.loads(str(vllm_quant["meta"]))
    assert meta["vllm"] == "0.22.0" and "B200" in meta["device"]


@pytest.mark.parametrize("case", ["normal_bf16", "normal_fp16", "normal_fp32", "odd_width_bf16",
                                  "ties_bf16", "special_bf16", "special_fp32"])
def test_oracle_quant_matches_vllm(vllm_quant, case):
    x = _tensor(vllm_quant[f"{case}.x"], str(vllm_quant[f"{case}.dtype"]))
    q, s = orc.dynamic_scaled_int8_quant(x)
    np.testing.assert_array_equal(s, vllm_quant[f"{case}.s"])
    np.testing.assert_array_equal(q, vllm_quant[f"{case}.q"])


def test_vllm_rounds_half_to_even(vllm_quant):
    """The tie case pins round-half-even (x * 127/amax with 127/amax == 1)."""
    x = _tensor(vllm_quant["ties_bf16.x"], "torch.bfloat16").float().numpy()
    q = vllm_quant["ties_bf16.q"]
    halves = np.abs(x - np.trunc(x)) == 0.5
    assert halves.sum() > 100
    np.testing.assert_array_equal(q[halves], np.rint(x[halves]).astype(np.int8))
    assert not np.array_equal(q[halves], np.round(x[halves] + 1e-3 * np.sign(x[halves])).astype(np.int8))


def test_vllm_zero_row_scale_is_zero(vllm_quant):
    s = vllm_quant["special_bf16.s"]
    q = vllm_quant["special_bf16.q"]
    assert s[0] == 0.0 and not q[0].any()


def test_oracle_scaled_mm_matches_vllm():
    path = GOLDEN / "vllm_scaled_mm.npz"
    if not path.exists():
        pytest.skip("vllm_scaled_mm.npz not generated")
    d = np.load(path)
    for i in range(int(d["count"])):
        dtype = getattr(torch, str(d[f"{i}.dtype"]).split(".")[-1])
        bias = _tensor(d[f"{i}.bias"], str(d[f"{i}.dtype"])) if f"{i}.bias" in d.files else None
        y, _ = orc.scaled_mm(d[f"{i}.a"], d[f"{i}.b"], d[f"{i}.sa"], d[f"{i}.sb"], bias, dtype)
        ref = _tensor(d[f"{i}.out"], str(d[f"{i}.dtype"]))
        torch.testing.assert_close(y.float(), ref.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("name", ["w_small", "w_wide"])
def test_oracle_weight_quant_matches_reference(ref_host, name):
    arrays, _ = ref_host
    q, s = orc.quantize_weight(_bf16(arrays[f"{name}.w"]))
    np.testing.assert_array_equal(s, arrays[f"{name}.s"])
    np.testing.assert_array_equal(q, arrays[f"{name}.q"])


def test_streamed_load_equals_whole_conversion(ref_host):
    arrays, _ = ref_host
    q, s = orc.quantize_weight(_bf16(arrays["stream.src"]))
    np.testing.assert_array_equal(q, arrays["stream.q"])
    np.testing.assert_array_equal(s, arrays["stream.s"])


def test_oracle_linear_matches_reference_composition(ref_host):
    """The reference's cutlass_w8a8_linear (w8a8.py:117-145) on an oracle backend."""
    arrays, meta = ref_host
    x = _bf16(arrays["linear.x"])
    y = orc.w8a8_linear(x, arrays["linear.wq"], arrays["linear.ws"])
    assert y.shape == (2, 5, 128)
    assert torch.equal(y, _bf16(arrays["linear.y"]).reshape(2, 5, 128))
    assert meta["linear_bias_rejected"] is True


def test_int_mm_exact_against_int64():
    g = torch.Generator().manual_seed(0)
    a = torch.randint(-128, 128, (37, 4096), generator=g, dtype=torch.int8).numpy()
    b = torch.randint(-128, 128, (19, 4096), generator=g, dtype=torch.int8).numpy()
    np.testing.assert_array_equal(orc.int_mm(a, b), a.astype(np.int64) @ b.astype(np.int64).T)


def test_epilogue_order_and_rounding():
    acc = np.array([[100000, -7, 0, 2 ** 24 + 1]], dtype=np.int32)
    sa = np.array([0.013], np.float32)
    sb = np.array([0.5, 2.0, 1.0, 1e-6], np.float32)
    y = orc.scaled_mm_epilogue(acc, sa, sb, None, torch.bfloat16)
    expect = np.float32(0.013) * (sb * acc.astype(np.float32))
    assert torch.equal(y, torch.from_numpy(expect.astype(np.float32)).to(torch.bfloat16))


def test_modulate_rounding_steps():
    x = torch.tensor([[1.0, -2.0, 0.3]]).to(torch.bfloat16)
    shift = torch.tensor([[0.1, 0.0, -0.2]]).to(torch.bfloat16)
    scale = torch.tensor([[0.05, -0.5, 0.0]]).to(torch.bfloat16)
    h = orc.modulate(x, shift, scale)
    xf, sf, shf = x.float(), scale.float(), shift.float()
    expect = ((xf * (1 + sf).to(torch.bfloat16).float()).to(torch.bfloat16).float() + shf).to(torch.bfloat16)
    assert torch.equal(h, expect)


def _ulysses_cases():
    data = np.load(GOLDEN / "ulysses_send.npz")
    i = 0
    while f"case{i}_shape" in data:
        tokens, heads, head_dim, degree = (int(v) for v in data[f"case{i}_shape"])
        send = _bf16(data[f"case{i}_send"]) if f"case{i}_send" in data else None
        yield (tokens, heads, head_dim, degree, _bf16(data[f"case{i}_value"]),
               _bf16(data[f"case{i}_qkv"]), send)
        i += 1


def test_oracle_ulysses_send_layout_matches_reference():
    seen_padding = False
    for tokens, heads, head_dim, degree, value, qkv, send in _ulysses_cases():
        if send is None:
            continue
        got = orc.merged_qkv_send_layout(value, heads, head_dim, degree)
        assert got.shape == send.shape
        assert torch.equal(got.view(torch.int16), send.view(torch.int16))
        seen_padding |= heads % degree != 0
    assert seen_padding


def test_ulysses_receive_layout_matches_reference():
    """The reference's outputs were taken with an identity exchange, so its
    (q, k, v) are the receive layout of its own send buffer."""
    from taomate_hd_b200.ulysses import exchange_qkv, receive_layout

    for tokens, heads, head_dim, degree, value, qkv, send in _ulysses_cases():
        if send is None:  # degree 1: no exchange, q/k/v straight from the projection
            got = exchange_qkv(orc.merged_qkv_send_layout(value, heads, head_dim, 1))
        else:
            got = receive_layout(send)
        assert torch.equal(torch.stack(got).view(torch.int16), qkv.view(torch.int16))


def test_oracle_adaln_and_swiglu_match_reference_triton_kernels():
    """fused_modulate / fused_gate_add / fused_rms_norm_modulate /
    fused_residual_gate_rms_norm_modulate / fused_swiglu
    (fused_kernels.py:643-797), executed by Triton's interpreter: the
    oracle reproduces every output bit, including bf16 overflow to inf and
    widths that leave a masked tail in the kernel's block."""
    data = np.load(GOLDEN / "adaln_triton.npz")
    for i in range(int(data["n_shapes"][0])):
        g = lambda k: _bf16(data[f"s{i}_{k}"])
        idx = torch.from_numpy(data[f"s{i}_indices"])
        eps = float(data[f"s{i}_eps"][0])
        x, branch, residual = g("x"), g("branch"), g("residual")
        scale, shift, gate, weight = g("scale"), g("shift"), g("gate"), g("weight")

        def same(got, name):
            assert torch.equal(got.view(torch.int16), g(f"out_{name}").view(torch.int16)), name

        with np.errstate(over="ignore", invalid="ignore"):
            same(orc.modulate(x, shift, scale, idx), "modulate")
            value, _ = orc.residual_gate_rms_norm_modulate(residual, branch, gate, weight, eps,
                                                           shift, scale, idx)
            same(value, "gate_add")
            same(orc.rms_norm_modulate(x.clamp(-100, 100), weight, eps, shift, scale, idx),
                 "rms_norm_modulate")
            value, hidden = orc.residual_gate_rms_norm_modulate(
                residual.clamp(-100, 100), branch, gate, weight, eps, shift, scale, idx)
            same(value, "residual_gate_value")
            same(hidden, "residual_gate_hidden")
            same(orc.swiglu(g("swiglu_in")), "swiglu")
