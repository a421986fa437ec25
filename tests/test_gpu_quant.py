"""GPU parity: int8 quantisation kernels vs the CPU oracle (bit-exact).

Reference behaviour: vLLM ``dynamic_scaled_int8_quant`` as called at
src/taomate_hd/inference/w8a8.py:71 / :141, weight conversion at
w8a8.py:175-179, adaLN producers at fused_kernels.py:220-236 / :322-347.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import w8a8_oracle as orc

pytestmark = pytest.mark.gpu


def _rand(rows, cols, dtype, seed, outliers=None):
    x = orc.activation(rows, cols, seed, outlier_channels=outliers)
    return x.to(dtype)


@pytest.mark.parametrize(
    "rows,cols",
    [(1, 16), (7, 384), (64, 3072), (33, 5376), (130, 12288), (5, 1536), (3, 40000), (9, 1000),
     (300, 24), (2, 8)],
)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_dynamic_quant_bit_exact(tm_ops, cuda, rows, cols, dtype):
    x = _rand(rows, cols, dtype, seed=rows * 7919 + cols)
    q, s, azp = tm_ops.scaled_int8_quant(x.to(cuda))
    assert azp is None and q.dtype == torch.int8 and s.shape == (rows, 1)
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(x)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


def test_dynamic_quant_edge_rows(tm_ops, cuda):
    x = torch.randn(8, 512)
    x[0] = 0.0                          # padding row -> scale 0, q 0
    x[1] = 0.0
    x[1, 3] = -5.0                      # single nonzero -> -127 there
    x[2] = 2.5                          # constant row
    x[3, ::2] = 1e4
    # exact ties: amax 127 -> inverse scale 1, so k + 0.5 rounds half-even
    x[4] = 0.0
    x[4, :254] = torch.arange(-126.5, 127.0, 1.0)[:254]
    x[4, 300] = 127.0
    xb = x.to(torch.bfloat16)
    q, s, _ = tm_ops.scaled_int8_quant(xb.to(cuda))
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(xb)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    assert s[0].item() == 0.0 and (q[0] == 0).all()
    assert q[1, 3].item() == -127


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_dynamic_quant_non_finite_rows(tm_ops, cuda, dtype):
    """Rows whose maximum is inf, NaN or subnormal (127 / amax overflows) take
    the conversion-instruction path; finite rows the FP32-pipe rounding: both
    bit-exact with the oracle (NaN -> 0, saturation at -128 / 127)."""
    x = torch.randn(8, 1024) * 3
    x[0, 5] = float("inf")
    x[1, 7] = float("-inf")
    x[2, 9] = float("nan")
    x[3] = 0.0
    x[3, :4] = torch.tensor([1e-40, -2e-40, 3e-41, 0.0])  # subnormal row maximum
    x[4, 11] = 1e30  # large but finite
    xd = x.to(dtype)
    q, s, _ = tm_ops.scaled_int8_quant(xd.to(cuda))
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(xd)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)


def test_dynamic_quant_3d_and_strided(tm_ops, cuda):
    x = _rand(6 * 5, 768, torch.bfloat16, seed=5).reshape(6, 5, 768).to(cuda)
    q, s, _ = tm_ops.scaled_int8_quant(x)
    assert q.shape == x.shape and s.shape == (30, 1)
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(x.cpu().reshape(-1, 768))
    np.testing.assert_array_equal(q.cpu().numpy().reshape(-1, 768), q_ref)
    # a row-strided 2-D view goes through the out-variant op without a copy
    big = _rand(40, 1024, torch.bfloat16, seed=6).to(cuda)
    view = big[:, :512]
    out = torch.empty(40, 512, dtype=torch.int8, device=cuda)
    sc = torch.empty(40, 1, dtype=torch.float32, device=cuda)
    torch.ops.taomate_w8a8.dynamic_scaled_int8_quant(out, view, sc, None)
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(view.cpu())
    np.testing.assert_array_equal(out.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(sc.cpu().numpy().reshape(-1), s_ref)


def test_static_quant_bit_exact(tm_ops, cuda):
    x = _rand(50, 3072, torch.bfloat16, seed=11)
    scale = torch.tensor([0.0371], dtype=torch.float32)
    q, s, _ = tm_ops.scaled_int8_quant(x.to(cuda), scale.to(cuda))
    np.testing.assert_array_equal(q.cpu().numpy(), orc.static_scaled_int8_quant(x, 0.0371))


@pytest.mark.parametrize("n,k", [(96, 200), (3072, 3072), (17, 16), (256, 12288)])
def test_weight_quant_bit_exact(tm_ops, cuda, n, k):
    w = orc.weight(n, k, seed=n + k)
    w[0] = 0.0  # zero row -> scale clamps at 1e-12
    q, s = tm_ops.quantize_weight_int8(w.to(cuda))
    q_ref, s_ref = orc.quantize_weight(w)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("rows,cols,indexed", [(64, 3072, False), (37, 1536, True), (5, 12288, True)])
def test_modulate_quant_bit_exact(tm_ops, cuda, rows, cols, indexed):
    g = torch.Generator().manual_seed(rows + cols)
    x = _rand(rows, cols, torch.bfloat16, seed=rows)
    table = 3 if indexed else rows
    shift = (torch.randn(table, cols, generator=g) * 0.1).to(torch.bfloat16)
    scale = (torch.randn(table, cols, generator=g) * 0.1).to(torch.bfloat16)
    index = torch.randint(0, table, (rows,), generator=g) if indexed else None
    q, s, h = tm_ops.modulate_int8_quant(
        x.to(cuda), shift.to(cuda), scale.to(cuda),
        index.to(cuda) if index is not None else None, return_hidden=True)
    h_ref = orc.modulate(x, shift, scale, index)
    assert torch.equal(h.cpu(), h_ref)
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(h_ref)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


def test_rms_norm_modulate_quant(tm_ops, cuda):
    rows, cols = 48, 3072
    g = torch.Generator().manual_seed(3)
    x = _rand(rows, cols, torch.bfloat16, seed=9)
    w = (1.0 + 0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16)
    shift = (torch.randn(3, cols, generator=g) * 0.1).to(torch.bfloat16)
    scale = (torch.randn(3, cols, generator=g) * 0.1).to(torch.bfloat16)
    index = torch.randint(0, 3, (rows,), generator=g)
    q, s, h = tm_ops.rms_norm_modulate_int8_quant(
        x.to(cuda), w.to(cuda), 1e-6, shift.to(cuda), scale.to(cuda), index.to(cuda),
        return_hidden=True)
    h_ref = orc.rms_norm_modulate(x, w, 1e-6, shift, scale, index)
    # the correctly rounded mean / sqrt / reciprocal chain reproduces the
    # reference arithmetic bit for bit, and so do int8 rows and scales
    assert torch.equal(h.cpu(), h_ref)
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(h_ref)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("with_index", [True, False])
def test_residual_gate_rms_norm_modulate_quant(tm_ops, cuda, with_index):
    """The fc1-input producer after attention (fused_kernels.py:349-382):
    gated residual update, RMSNorm + modulate and the int8 rows and scales,
    all bit-exact against the oracle chain."""
    rows, cols = 40, 3072
    g = torch.Generator().manual_seed(31)
    residual = _rand(rows, cols, torch.bfloat16, seed=32)
    branch = _rand(rows, cols, torch.bfloat16, seed=33)
    w = (1.0 + 0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16)
    table_rows = 3 if with_index else rows
    gate = (torch.randn(table_rows, cols, generator=g) * 0.5).to(torch.bfloat16)
    shift = (torch.randn(table_rows, cols, generator=g) * 0.1).to(torch.bfloat16)
    scale = (torch.randn(table_rows, cols, generator=g) * 0.1).to(torch.bfloat16)
    index = torch.randint(0, 3, (rows,), generator=g) if with_index else None
    q, s, res_out, h = tm_ops.residual_gate_rms_norm_modulate_int8_quant(
        residual.to(cuda), branch.to(cuda), gate.to(cuda), w.to(cuda), 1e-6, shift.to(cuda),
        scale.to(cuda), None if index is None else index.to(cuda), return_hidden=True)
    res_ref, h_ref = orc.residual_gate_rms_norm_modulate(residual, branch, gate, w, 1e-6, shift,
                                                         scale, index)
    assert torch.equal(res_out.cpu(), res_ref)
    assert torch.equal(h.cpu(), h_ref)
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(h_ref)
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), s_ref)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    # the modulated state from the kernel's own residual equals the plain
    # RMSNorm + modulate producer's
    _, _, h2 = tm_ops.rms_norm_modulate_int8_quant(
        res_out, w.to(cuda), 1e-6, shift.to(cuda), scale.to(cuda),
        None if index is None else index.to(cuda), return_hidden=True)
    assert torch.equal(h2, h)


@pytest.mark.parametrize("gated", [False, True])
def test_rms_norm_producers_full_768p_bit_exact(tm_ops, cuda, gated):
    """The 768p QKV / fc1 input (20480 x 3072, three modality rows in the
    adaLN tables): every hidden element, int8 value and scale of every row
    equals the oracle chain's; the mismatching-row count is in the message."""
    rows, cols = 20480, 3072
    g = torch.Generator().manual_seed(41 + gated)
    x = _rand(rows, cols, torch.bfloat16, seed=42 + gated)
    w = (1.0 + 0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16)
    shift = (torch.randn(3, cols, generator=g) * 0.1).to(torch.bfloat16)
    scale = (torch.randn(3, cols, generator=g) * 0.1).to(torch.bfloat16)
    index = torch.randint(0, 3, (rows,), generator=g)
    if gated:
        branch = _rand(rows, cols, torch.bfloat16, seed=43)
        gate = (torch.randn(3, cols, generator=g) * 0.5).to(torch.bfloat16)
        q, s, _, h = tm_ops.residual_gate_rms_norm_modulate_int8_quant(
            x.to(cuda), branch.to(cuda), gate.to(cuda), w.to(cuda), 1e-6, shift.to(cuda),
            scale.to(cuda), index.to(cuda), return_hidden=True)
        _, h_ref = orc.residual_gate_rms_norm_modulate(x, branch, gate, w, 1e-6, shift, scale,
                                                       index)
    else:
        q, s, h = tm_ops.rms_norm_modulate_int8_quant(
            x.to(cuda), w.to(cuda), 1e-6, shift.to(cuda), scale.to(cuda), index.to(cuda),
            return_hidden=True)
        h_ref = orc.rms_norm_modulate(x, w, 1e-6, shift, scale, index)
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(h_ref)
    h_bad = (h.cpu().view(torch.int16) != h_ref.view(torch.int16)).any(dim=1)
    q_bad = torch.from_numpy((q.cpu().numpy() != q_ref).any(axis=1)
                             | (s.cpu().numpy().reshape(-1) != s_ref))
    assert int(h_bad.sum()) == 0 and int(q_bad.sum()) == 0, (
        f"{int(h_bad.sum())} of {rows} hidden rows and {int(q_bad.sum())} int8 rows differ")


@pytest.mark.parametrize("case", ["normal_bf16", "normal_fp16", "normal_fp32", "odd_width_bf16",
                                  "ties_bf16", "special_bf16", "special_fp32"])
def test_quant_kernel_matches_vllm_golden_bytes(tm_ops, cuda, case):
    """The kernel fed the exact inputs of the vLLM golden vectors (vLLM 0.22
    scaled_int8_quant run on a B200) returns vLLM's int8 bytes and scales."""
    data = np.load(orc_golden_path())
    dtype = str(data[f"{case}.dtype"])
    bits = data[f"{case}.x"]
    if dtype == "torch.bfloat16":
        x = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)
    elif dtype == "torch.float16":
        x = torch.from_numpy(bits.view(np.int16).copy()).view(torch.float16)
    else:
        x = torch.from_numpy(bits.copy())
    q, s, _ = tm_ops.scaled_int8_quant(x.to(cuda))
    np.testing.assert_array_equal(q.cpu().numpy(), data[f"{case}.q"])
    np.testing.assert_array_equal(s.cpu().numpy().reshape(-1), data[f"{case}.s"])


def orc_golden_path():
    from pathlib import Path

    return Path(__file__).resolve().parent / "golden" / "vllm_quant.npz"


def test_quant_through_c_abi(capi, cuda):
    x = _rand(100, 3072, torch.bfloat16, seed=21).to(cuda)
    q = torch.empty(100, 3072, dtype=torch.int8, device=cuda)
    s = torch.empty(100, dtype=torch.float32, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = capi.tm_dynamic_scaled_int8_quant(q.data_ptr(), x.data_ptr(), 0, s.data_ptr(), None,
                                           100, 3072, 3072, stream)
    assert rc == 0
    torch.cuda.synchronize()
    q_ref, s_ref = orc.dynamic_scaled_int8_quant(x.cpu())
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    # argument errors are reported before any launch
    assert capi.tm_dynamic_scaled_int8_quant(q.data_ptr(), x.data_ptr(), 0, s.data_ptr(), None,
                                             100, 3072, 100, stream) == 2  # ld < cols
    assert capi.tm_dynamic_scaled_int8_quant(q.data_ptr(), x.data_ptr(), 9, s.data_ptr(), None,
                                             100, 3072, 3072, stream) == 4  # dtype
    assert capi.tm_dynamic_scaled_int8_quant(q.data_ptr(), x.data_ptr(), 0, s.data_ptr(),
                                             ctypes.c_void_p(16), 100, 3072, 3072, stream) == 5


def test_cpu_tensors_raise(tm_ops):
    with pytest.raises(RuntimeError):
        tm_ops.scaled_int8_quant(torch.randn(4, 16, dtype=torch.bfloat16))
