"""GPU: the allocation-free split-K entry point against the ordinary GEMM entry.

``tm_scaled_mm_i8_splitk_noalloc`` keeps its int32 partials and tile counters
in a fixed array inside the library instead of a caller workspace.  Its
outputs must agree with ``tm_scaled_mm_i8_ex`` (no split, no scratch) on the
same operands, on consecutive calls that reuse the array, and requests whose
split needs more than the array holds must be refused before any launch.
The file name keeps it last in collection, so it also runs after every other
GPU test has used the library in the same process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 1e-2
TM_ERR_UNSUPPORTED = 5
TM_ERR_TOO_LARGE = 8


def _operands(m, n, k, seed, cuda, with_bias):
    g = torch.Generator().manual_seed(seed)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    sa = torch.rand(m, generator=g) * 0.02 + 1e-4
    sb = torch.rand(n, generator=g) * 0.002 + 1e-5
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16) if with_bias else None
    return tuple(None if t is None else t.to(cuda) for t in (a, b, sa, sb, bias))


def _gemm_args(out, a, b, sa, sb, bias):
    m, k = a.shape
    n = b.shape[0]
    return (out.data_ptr(), 0, a.data_ptr(), b.data_ptr(), sa.data_ptr(), sa.numel(),
            sb.data_ptr(), sb.numel(), None if bias is None else bias.data_ptr(),
            m, n, k, k, k, n)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m,n,k,tile_n,splits,with_bias,epilogue", [
    (64, 3072, 12288, 64, 3, False, 0),
    (16, 1536, 12288, 64, 6, True, 0),
    (200, 768, 6144, 128, 4, True, 1),
])
def test_no_alloc_matches_ordinary_entry_two_calls(capi, cuda, m, n, k, tile_n, splits,
                                                   with_bias, epilogue):
    for call in range(2):
        a, b, sa, sb, bias = _operands(m, n, k, seed=100 * call + m, cuda=cuda,
                                       with_bias=with_bias)
        ref = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        got = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
        rc = capi.tm_scaled_mm_i8_ex(*_gemm_args(ref, a, b, sa, sb, bias), epilogue, None,
                                     _stream())
        assert rc == 0, capi.tm_status_string(rc)
        rc = capi.tm_scaled_mm_i8_splitk_noalloc(*_gemm_args(got, a, b, sa, sb, bias), epilogue,
                                                 tile_n, splits, _stream())
        assert rc == 0, capi.tm_status_string(rc)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float().cpu(), ref.float().cpu(), atol=ATOL, rtol=RTOL,
                                   msg=f"call {call}")


def test_no_alloc_refuses_oversized_and_bad_arguments(capi, cuda):
    a, b, sa, sb, _ = _operands(256, 128, 1024, seed=1, cuda=cuda, with_bias=False)
    out = torch.empty(256, 128, dtype=torch.bfloat16, device=cuda)
    base = list(_gemm_args(out, a, b, sa, sb, None))
    # 2 slices x 256 x 12288 x 4 bytes = 24 MiB of partials: above the array
    big = base.copy()
    big[9:15] = [256, 12288, 12288, 12288, 12288, 12288]
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*big, 0, 64, 2, _stream()) == TM_ERR_TOO_LARGE
    # sizes whose m * n * splits * 4 leaves 64 bits are refused, not wrapped
    huge = base.copy()
    huge[9:15] = [1 << 30, 1 << 30, 1 << 20, 1 << 20, 1 << 20, 1 << 30]
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*huge, 0, 64, 64, _stream()) == TM_ERR_TOO_LARGE
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*base, 0, 96, 2, _stream()) == TM_ERR_UNSUPPORTED
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*base, 0, 64, 0, _stream()) == TM_ERR_UNSUPPORTED
    torch.cuda.synchronize()
