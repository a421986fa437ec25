"""GPU parity: tcgen05 scaled int8 GEMM vs the CPU oracle.

Reference behaviour: vLLM ``cutlass_scaled_mm`` as called at
src/taomate_hd/inference/w8a8.py:72 and :142-144.  int32 accumulators are
compared bit-exactly through the kernel's debug output; bf16/fp16 outputs
within |diff| <= 1e-2 + 1e-2 * |ref| (the BASELINE.json tolerance).
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


def _operands(m, n, k, seed, per_tok=True, per_ch=True, bias_dtype=None):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    sa = torch.rand(m if per_tok else 1, 1, generator=g) * 0.02 + 1e-4
    sb = torch.rand(1, n if per_ch else 1, generator=g) * 0.002 + 1e-5
    bias = (torch.randn(n, generator=g) * 0.01).to(bias_dtype) if bias_dtype else None
    return a, b, sa, sb, bias


def _run(tm_ops, cuda, a, b, sa, sb, bias, out_dtype, gelu=False, tile_n=0):
    m, n = a.shape[0], b.shape[0]
    acc = torch.empty(m, n, dtype=torch.int32, device=cuda)
    out = tm_ops.scaled_mm(a.to(cuda), b.to(cuda).t(), sa.to(cuda), sb.to(cuda), out_dtype,
                           bias.to(cuda) if bias is not None else None, gelu_tanh=gelu,
                           acc_debug=acc, tile_n=tile_n)
    torch.cuda.synchronize()
    return out.cpu(), acc.cpu().numpy()


@pytest.mark.parametrize(
    "m,n,k",
    [(128, 256, 128), (1, 16, 16), (100, 48, 32), (300, 1008, 208), (257, 512, 3072),
     (64, 3072, 3072), (1024, 3072, 3072), (513, 1152, 12288), (8192, 3072, 1536),
     (2560, 2304, 3072)],
)
def test_scaled_mm_acc_and_output(tm_ops, cuda, m, n, k):
    a, b, sa, sb, _ = _operands(m, n, k, seed=m * 31 + n * 7 + k)
    out, acc = _run(tm_ops, cuda, a, b, sa, sb, None, torch.bfloat16)
    acc_ref = orc.int_mm(a.numpy(), b.numpy())
    np.testing.assert_array_equal(acc, acc_ref)
    ref = orc.scaled_mm_epilogue(acc_ref, sa.numpy(), sb.numpy(), None, torch.bfloat16)
    torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("tile_n", [256, 128, 64, 1256, 1192, 1128])
@pytest.mark.parametrize("m,n,k", [(200, 400, 256), (129, 272, 640), (384, 1024, 1024),
                                   (1000, 2112, 384)])
def test_every_tile_width(tm_ops, cuda, tile_n, m, n, k):
    a, b, sa, sb, bias = _operands(m, n, k, seed=tile_n + m, bias_dtype=torch.bfloat16)
    out, acc = _run(tm_ops, cuda, a, b, sa, sb, bias, torch.bfloat16, tile_n=tile_n)
    acc_ref = orc.int_mm(a.numpy(), b.numpy())
    np.testing.assert_array_equal(acc, acc_ref)
    ref = orc.scaled_mm_epilogue(acc_ref, sa.numpy(), sb.numpy(), bias, torch.bfloat16)
    torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("per_tok,per_ch", [(True, True), (False, False), (True, False), (False, True)])
def test_scale_broadcast_bias_dtype(tm_ops, cuda, out_dtype, per_tok, per_ch):
    a, b, sa, sb, bias = _operands(160, 384, 512, seed=3, per_tok=per_tok, per_ch=per_ch,
                                   bias_dtype=out_dtype)
    out, acc = _run(tm_ops, cuda, a, b, sa, sb, bias, out_dtype)
    ref = orc.scaled_mm_epilogue(acc, sa.numpy(), sb.numpy(), bias, out_dtype)
    assert out.dtype == out_dtype
    torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)


def test_gelu_epilogue(tm_ops, cuda):
    a, b, sa, sb, bias = _operands(256, 768, 1024, seed=17, bias_dtype=torch.bfloat16)
    sb *= 20  # outputs of order 1 so that GELU's curvature matters
    out, acc = _run(tm_ops, cuda, a, b, sa, sb, bias, torch.bfloat16, gelu=True)
    ref = orc.scaled_mm_epilogue(acc, sa.numpy(), sb.numpy(), bias, torch.bfloat16, gelu=True)
    torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)


def test_vllm_surface_cutlass_scaled_mm(tm_ops, cuda):
    """The drop-in wrapper: a 3-D activation, weight.t() view, [M,1]/[1,N] scales."""
    x = orc.activation(2 * 96, 1024, seed=4).reshape(2, 96, 1024)
    w = orc.weight(512, 1024, seed=5)
    wq, ws = orc.quantize_weight(w)
    q, s, _ = tm_ops.scaled_int8_quant(x.to(cuda))
    wq_t = torch.from_numpy(wq).to(cuda)
    ws_t = torch.from_numpy(ws).reshape(-1, 1).to(cuda)
    y = tm_ops.cutlass_scaled_mm(q, wq_t.t(), s, ws_t.t(), torch.bfloat16)
    assert y.shape == (2, 96, 512)
    ref = orc.w8a8_linear(x, wq, ws)
    torch.testing.assert_close(y.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)


def test_scaled_mm_through_c_abi(capi, cuda):
    m, n, k = 256, 512, 768
    a, b, sa, sb, bias = _operands(m, n, k, seed=8, bias_dtype=torch.bfloat16)
    a_d, b_d, sa_d, sb_d, bias_d = (t.to(cuda) for t in (a, b, sa, sb, bias))
    out = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = capi.tm_cutlass_scaled_mm(out.data_ptr(), 0, a_d.data_ptr(), b_d.data_ptr(),
                                   sa_d.data_ptr(), m, sb_d.data_ptr(), n, bias_d.data_ptr(),
                                   m, n, k, k, k, n, stream)
    assert rc == 0
    torch.cuda.synchronize()
    acc_ref = orc.int_mm(a.numpy(), b.numpy())
    ref = orc.scaled_mm_epilogue(acc_ref, sa.numpy(), sb.numpy(), bias, torch.bfloat16)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=ATOL, rtol=RTOL)
    # host-side argument errors: K not a multiple of 16, misaligned pointer, bad scales
    assert capi.tm_cutlass_scaled_mm(out.data_ptr(), 0, a_d.data_ptr(), b_d.data_ptr(),
                                     sa_d.data_ptr(), m, sb_d.data_ptr(), n, None,
                                     m, n, 760, k, k, n, stream) == 2
    assert capi.tm_cutlass_scaled_mm(out.data_ptr(), 0, a_d.data_ptr() + 8, b_d.data_ptr(),
                                     sa_d.data_ptr(), m, sb_d.data_ptr(), n, None,
                                     m, n, k, k, k, n, stream) == 3
    assert capi.tm_cutlass_scaled_mm(out.data_ptr(), 0, a_d.data_ptr(), b_d.data_ptr(),
                                     sa_d.data_ptr(), 3, sb_d.data_ptr(), n, None,
                                     m, n, k, k, k, n, stream) == 2


def test_empty_m(tm_ops, cuda):
    a = torch.empty(0, 64, dtype=torch.int8, device=cuda)
    b = torch.zeros(32, 64, dtype=torch.int8, device=cuda)
    y = tm_ops.cutlass_scaled_mm(a, b.t(), torch.ones(1, device=cuda), torch.ones(1, device=cuda),
                                 torch.bfloat16)
    assert y.shape == (0, 32)


def _splitk_call(capi, cuda, a, b, sa, sb, bias, tile_n, splits, ws):
    m, k = a.shape
    n = b.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    acc = torch.empty(m, n, dtype=torch.int32, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = capi.tm_scaled_mm_i8_splitk(
        out.data_ptr(), 0, a.data_ptr(), b.data_ptr(), sa.data_ptr(), sa.numel(), sb.data_ptr(),
        sb.numel(), None if bias is None else bias.data_ptr(), m, n, k, k, k, n, 0, acc.data_ptr(),
        tile_n, splits, ws.data_ptr(), ws.numel(), stream)
    assert rc == 0, capi.tm_status_string(rc)
    torch.cuda.synchronize()
    return out.cpu(), acc.cpu().numpy()


@pytest.mark.parametrize("tile_n,splits", [(64, 3), (128, 2), (256, 5), (64, 8)])
@pytest.mark.parametrize("m,n,k", [(64, 3072, 3072), (200, 1024, 1280), (1, 48, 512),
                                   (300, 400, 2048)])
def test_split_k_bit_exact_two_calls(capi, cuda, tile_n, splits, m, n, k):
    """Split-K partial sums are exact int32: identical accumulators to the unsplit GEMM.

    Two calls on one workspace check that the per-tile counters return to zero.
    """
    a, b, sa, sb, bias = _operands(m, n, k, seed=m + n + splits, bias_dtype=torch.bfloat16)
    need = ctypes.c_uint64()
    assert capi.tm_scaled_mm_i8_splitk_workspace_size(m, n, k, tile_n, splits, ctypes.byref(need)) == 0
    ws = torch.zeros(max(int(need.value), 16), dtype=torch.uint8, device=cuda)
    d = [t.to(cuda) for t in (a, b, sa, sb, bias)]
    acc_ref = orc.int_mm(a.numpy(), b.numpy())
    ref = orc.scaled_mm_epilogue(acc_ref, sa.numpy(), sb.numpy(), bias, torch.bfloat16)
    for _ in range(2):
        out, acc = _splitk_call(capi, cuda, *d, tile_n, splits, ws)
        np.testing.assert_array_equal(acc, acc_ref)
        torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)
    # too small a workspace for a forced split is an error, not a silent fallback
    if need.value > 256:
        small = torch.zeros(256, dtype=torch.uint8, device=cuda)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        rc = capi.tm_scaled_mm_i8_splitk(
            out.data_ptr(), 0, d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[2].numel(),
            d[3].data_ptr(), d[3].numel(), None, m, n, k, k, k, n, 0, None, tile_n, splits,
            small.data_ptr(), small.numel(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 8


@pytest.mark.parametrize("m,n,k", [(64, 3072, 3072), (256, 12288, 3072), (16, 3072, 12288)])
def test_skinny_m_heuristic_path(tm_ops, cuda, capi, m, n, k):
    """The torch op picks split-K for skinny M on its own; results stay exact."""
    need = ctypes.c_uint64()
    assert capi.tm_scaled_mm_i8_workspace_size(m, n, k, ctypes.byref(need)) == 0
    a, b, sa, sb, bias = _operands(m, n, k, seed=m * 3 + k, bias_dtype=torch.bfloat16)
    for gelu in (False, True):
        out, acc = _run(tm_ops, cuda, a, b, sa, sb, bias, torch.bfloat16, gelu=gelu)
        acc_ref = orc.int_mm(a.numpy(), b.numpy())
        np.testing.assert_array_equal(acc, acc_ref)
        ref = orc.scaled_mm_epilogue(acc_ref, sa.numpy(), sb.numpy(), bias, torch.bfloat16, gelu=gelu)
        torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)


def test_split_workspace_reuse_with_more_tiles(tm_ops, cuda):
    """Two split-K calls through the torch op's cached workspace, the second
    with more tiles (48 then 72 one-CTA tiles of 64 columns): the second call's
    counters must not start on the first call's partials.  Bit-exact with the
    unsplit kernel."""
    for (m, n, k) in [(16, 3072, 12288), (128, 4608, 12288)]:
        a, b, sa, sb, bias = _operands(m, n, k, seed=m + n, bias_dtype=torch.bfloat16)
        a_d, b_d, sa_d, sb_d, bias_d = (t.to(cuda) for t in (a, b, sa, sb, bias))
        split = tm_ops.scaled_mm(a_d, b_d.t(), sa_d, sb_d, torch.bfloat16, bias_d)
        whole = tm_ops.scaled_mm(a_d, b_d.t(), sa_d, sb_d, torch.bfloat16, bias_d, tile_n=64)
        torch.cuda.synchronize()
        torch.testing.assert_close(split, whole, atol=0, rtol=0)
