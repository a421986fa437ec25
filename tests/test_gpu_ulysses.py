"""GPU: the merged QKV projection written in the Ulysses all-to-all send layout.

Reference behaviour: ``merged_qkv_sequence_to_heads`` / ``_merged_qkv_send_layout``
(src/taomate_hd/distributed/ulysses.py:153-212) permutes the merged QKV output
``[tokens, 3 * heads * head_dim]`` into ``[world, 3, tokens, ceil(heads /
world), head_dim]`` before the all-to-all, padding with zero heads when the
degree does not divide the heads (:188-193).  The fused epilogue writes that buffer
directly: it must equal the reference permute of the ordinary GEMM output bit
for bit (same epilogue arithmetic, different store coordinates).
"""
from __future__ import annotations

import pytest
import torch

from oracle import w8a8_oracle as orc

pytestmark = pytest.mark.gpu


def _operands(tokens, d, n, seed, cuda):
    g = torch.Generator(device=cuda).manual_seed(seed)
    q = torch.randint(-127, 128, (tokens, d), generator=g, device=cuda, dtype=torch.int8)
    w = torch.randint(-127, 128, (n, d), generator=g, device=cuda, dtype=torch.int8)
    sq = torch.rand(tokens, 1, generator=g, device=cuda) * 1e-2 + 1e-4
    sw = torch.rand(n, generator=g, device=cuda) * 1e-3 + 1e-5
    bias = (torch.randn(n, generator=g, device=cuda) * 0.01).to(torch.bfloat16)
    return q, w, sq, sw, bias


@pytest.mark.parametrize("tokens,d,heads,world,with_bias", [
    (256, 512, 8, 1, False),
    (256, 512, 8, 2, True),
    (320, 1024, 8, 4, False),     # tokens not a multiple of the 128-row tile
    (2048, 3072, 24, 8, True),    # 768p head layout at Ulysses 8
    (320, 512, 6, 4, True),       # zero-padded head shards (local 2, 2 padded heads)
    (256, 1024, 24, 5, False),    # one padded head in the last shard
    (128, 256, 2, 4, False),      # fewer heads than ranks: whole shards of zeros
])
def test_send_layout_matches_reference_permute(tm_ops, cuda, tokens, d, heads, world, with_bias):
    from taomate_hd_b200.ulysses import qkv_send_buffer

    hd = 128
    n = 3 * heads * hd
    q, w, sq, sw, bias = _operands(tokens, d, n, seed=tokens + world, cuda=cuda)
    b = bias if with_bias else None
    send = qkv_send_buffer(q, sq, w, sw, b, num_heads=heads, head_dim=hd, world=world)
    plain = tm_ops.scaled_mm(q, w.t(), sq, sw.reshape(1, -1), torch.bfloat16, b)
    ref = orc.merged_qkv_send_layout(plain, heads, hd, world)
    torch.cuda.synchronize()
    assert send.shape == ref.shape
    assert torch.equal(send, ref)


def test_send_layout_world_one_returns_qkv(tm_ops, cuda):
    from taomate_hd_b200.ulysses import merged_qkv_sequence_to_heads_w8a8

    q, w, sq, sw, bias = _operands(128, 256, 3 * 4 * 128, seed=3, cuda=cuda)
    qq, kk, vv = merged_qkv_sequence_to_heads_w8a8(q, sq, w, sw, bias, num_heads=4, head_dim=128)
    plain = tm_ops.scaled_mm(q, w.t(), sq, sw.reshape(1, -1), torch.bfloat16, bias)
    packed = plain.view(128, 3, 4, 128)
    for got, ref in zip((qq, kk, vv), packed.unbind(1)):
        assert torch.equal(got, ref)


def test_send_layout_argument_errors(tm_ops, cuda):
    from taomate_hd_b200.ulysses import qkv_send_buffer

    q, w, sq, sw, _ = _operands(100, 256, 3 * 4 * 128, seed=4, cuda=cuda)
    with pytest.raises(RuntimeError):  # 100 tokens: not a multiple of 32
        qkv_send_buffer(q, sq, w, sw, None, num_heads=4, head_dim=128, world=2)
    q2, w2, sq2, sw2, _ = _operands(128, 256, 3 * 4 * 128, seed=5, cuda=cuda)
    with pytest.raises(RuntimeError):  # head_dim 64 x 3 x 4 != the weight's 1536 rows
        qkv_send_buffer(q2, sq2, w2, sw2, None, num_heads=4, head_dim=64, world=2)
    from taomate_hd_b200.ulysses import merged_qkv_sequence_to_heads_w8a8
    with pytest.raises(ValueError):  # the reference's width check
        merged_qkv_sequence_to_heads_w8a8(q2, sq2, w2, sw2, None, num_heads=4, head_dim=64)


@pytest.mark.parametrize("tokens,d,heads", [(256, 512, 8), (320, 1024, 24), (2560, 3072, 24)])
def test_nvlink_exchange_on_one_rank_matches_send_layout(tm_ops, cuda, tokens, d, heads):
    """The exchange form (tm_scaled_mm_i8_ulysses_exchange) at one rank: the
    kernel stores into its own receive buffer, counts its stores and waits
    for them, so its (q, k, v) equal the send-layout path's bit for bit, over
    three calls (both buffer sets, a second use of one)."""
    from taomate_hd_b200.parallel import ParallelContext
    from taomate_hd_b200.ulysses import PeerUlyssesExchange, merged_qkv_sequence_to_heads_w8a8

    head_dim = 128
    ex = PeerUlyssesExchange.from_context(ParallelContext(), tokens, heads, head_dim, cuda)
    try:
        for call in range(3):
            q, w, sq, sw, bias = _operands(tokens, d, 3 * heads * head_dim, seed=call + tokens,
                                           cuda=cuda)
            want = merged_qkv_sequence_to_heads_w8a8(q, sq, w, sw, bias, num_heads=heads,
                                                     head_dim=head_dim)
            got = ex(q, sq, w, sw, bias)
            torch.cuda.synchronize()
            for a, b in zip(got, want):
                assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        ex.check()
    finally:
        ex.close()


def test_nvlink_exchange_argument_errors(capi, cuda):
    """Host checks of the exchange entry point, before any launch."""
    import ctypes

    p = ctypes.c_void_p(1 << 20)
    arr = (ctypes.c_void_p * 2)(p, p)
    call = capi.tm_scaled_mm_i8_ulysses_exchange
    #     a  b  sa  n   sb  n     bias  m    n     k    lda  ldb  heads hd   recv flags world rank ep st
    assert call(p, p, p, 256, p, 3072, None, 256, 3072, 512, 512, 512, 8, 128, None, arr, 2, 0, 1,
                None) == 1  # no receive buffers
    assert call(p, p, p, 256, p, 3072, None, 256, 3072, 512, 512, 512, 8, 128, arr, arr, 9, 0, 1,
                None) == 8  # more than 8 ranks
    assert call(p, p, p, 256, p, 3072, None, 256, 3072, 512, 512, 512, 8, 128, arr, arr, 2, 2, 1,
                None) == 2  # rank outside the group
    assert call(p, p, p, 256, p, 1536, None, 256, 1536, 512, 512, 512, 16, 32, arr, arr, 2, 0, 1,
                None) == 2  # head_dim not a multiple of 64
