"""GPU: the allocation-free split-K entry point against the ordinary GEMM entry.

``tm_scaled_mm_i8_splitk_noalloc`` keeps its int32 partials and tile counters
in a fixed array inside the library instead of a caller workspace, for callers
that must not allocate device memory.  The split sums exact int32 partials and
runs the same epilogue, so its outputs must equal ``tm_scaled_mm_i8_ex`` (no
split, no scratch) bit for bit on the same operands, on consecutive calls that
reuse the array; requests whose split needs more than the array holds, and bad
arguments, must be refused before anything is enqueued.
The file name keeps it last in collection, so it also runs after every other
GPU test has used the library in the same process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TM_ERR_SHAPE = 2
TM_ERR_ALIGNMENT = 3
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
        assert torch.equal(got, ref), f"call {call}: split-K output differs from the unsplit GEMM"


def test_no_alloc_refuses_oversized_and_bad_arguments(capi, cuda):
    a, b, sa, sb, _ = _operands(256, 128, 1024, seed=1, cuda=cuda, with_bias=False)
    out = torch.empty(256, 128, dtype=torch.bfloat16, device=cuda)
    base = list(_gemm_args(out, a, b, sa, sb, None))
    # 2 slices x 256 x 12288 x 4 bytes = 24 MiB of partials: above the array
    # (per-tensor scales keep the oversized requests valid in every other way)
    big = base.copy()
    big[5], big[7] = 1, 1
    big[9:15] = [256, 12288, 12288, 12288, 12288, 12288]
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*big, 0, 64, 2, _stream()) == TM_ERR_TOO_LARGE
    # sizes whose m * n * splits * 4 leaves 64 bits are refused, not wrapped
    huge = base.copy()
    huge[5], huge[7] = 1, 1
    huge[9:15] = [1 << 30, 1 << 30, 1 << 20, 1 << 20, 1 << 20, 1 << 30]
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*huge, 0, 64, 64, _stream()) == TM_ERR_TOO_LARGE
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*base, 0, 96, 2, _stream()) == TM_ERR_UNSUPPORTED
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*base, 0, 64, 0, _stream()) == TM_ERR_UNSUPPORTED
    torch.cuda.synchronize()


def test_no_alloc_checks_arguments_before_enqueueing(capi, cuda):
    """Refused calls return their error before the counters are cleared on
    the stream: an output left as NaN stays NaN, and the next valid call on
    the same stream is exact."""
    a, b, sa, sb, _ = _operands(64, 768, 12288, seed=3, cuda=cuda, with_bias=False)
    got = torch.full((64, 768), float("nan"), dtype=torch.bfloat16, device=cuda)
    args = list(_gemm_args(got, a, b, sa, sb, None))
    bad_ld = args.copy()
    bad_ld[12] = 12280  # lda < k
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*bad_ld, 0, 64, 4, _stream()) == TM_ERR_SHAPE
    bad_align = args.copy()
    bad_align[2] = a.data_ptr() + 8
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*bad_align, 0, 64, 4, _stream()) == TM_ERR_ALIGNMENT
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*args, 2, 64, 4, _stream()) == TM_ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert torch.isnan(got.float()).all()
    ref = torch.empty_like(got)
    assert capi.tm_scaled_mm_i8_ex(*_gemm_args(ref, a, b, sa, sb, None), 0, None, _stream()) == 0
    assert capi.tm_scaled_mm_i8_splitk_noalloc(*args, 0, 64, 4, _stream()) == 0
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
