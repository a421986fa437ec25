"""Ulysses sequence-to-heads exchange of a W8A8 merged QKV projection.

The reference's inference path (src/taomate_hd/distributed/ulysses.py:166-212,
``merged_qkv_sequence_to_heads``) runs the merged QKV linear, permutes its
``[tokens, 3 * heads * head_dim]`` output into the all-to-all send layout
``[world, 3, tokens, ceil(heads / world), head_dim]`` (zero heads pad the last
shards when ``world`` does not divide ``heads``, ulysses.py:188-193) and
exchanges it.  Here the
scaled GEMM's epilogue writes the send layout directly
(``torch.ops.taomate_w8a8.scaled_mm_i8_ulysses_send``), so the projection
output is never materialised in token-major order; the exchange and the
receive layout are the reference's.
"""
from __future__ import annotations

import torch

from . import ops  # noqa: F401  (registers torch.ops.taomate_w8a8)


def qkv_send_buffer(q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
                    w_scale: torch.Tensor, bias: torch.Tensor | None, *, num_heads: int,
                    head_dim: int, world: int, out_dtype: torch.dtype = torch.bfloat16
                    ) -> torch.Tensor:
    """The merged QKV projection of int8 ``q`` ([tokens, d], per-token scales)
    with int8 ``w_q`` ([3 * heads * head_dim, d], per-channel scales) as the
    send buffer ``[world, 3, tokens, ceil(heads / world), head_dim]`` (padded
    head slots zero)."""
    tokens = q.shape[0]
    local = -(-num_heads // world)
    send = torch.empty((world, 3, tokens, local, head_dim), dtype=out_dtype, device=q.device)
    torch.ops.taomate_w8a8.scaled_mm_i8_ulysses_send(
        send, q, w_q.t(), q_scale, w_scale.reshape(-1), bias, num_heads, head_dim, world)
    return send


def receive_layout(received: torch.Tensor) -> tuple[torch.Tensor, ...]:
    """The all-to-all output ``[world, 3, tokens, local, head_dim]`` (chunk s
    from rank s) as (q, k, v), each ``[tokens * world, local, head_dim]``
    (distributed/ulysses.py:209-212)."""
    world, three, tokens, local, head_dim = received.shape
    exchanged = received.movedim(0, 1).contiguous().view(three, tokens * world, local, head_dim)
    return tuple(exchanged.unbind(0))


def exchange_qkv(send: torch.Tensor, *, group=None) -> tuple[torch.Tensor, ...]:
    """All-to-all of a send buffer ``[world, 3, tokens, local, head_dim]`` over
    ``group`` (world == its size), returning (q, k, v) as the reference does
    (distributed/ulysses.py:194-212)."""
    world = send.shape[0]
    if world == 1:
        return tuple(send[0].unbind(0))
    if not torch.distributed.is_available() or not torch.distributed.is_initialized():
        raise RuntimeError("Ulysses all-to-all requires initialized torch.distributed")
    received = torch.empty_like(send)
    torch.distributed.all_to_all_single(received, send, group=group)
    return receive_layout(received)


def merged_qkv_sequence_to_heads_w8a8(q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
                                      w_scale: torch.Tensor, bias: torch.Tensor | None, *,
                                      num_heads: int, head_dim: int, group=None,
                                      world: int = 1) -> tuple[torch.Tensor, ...]:
    """Project and exchange: returns (q, k, v), each
    ``[tokens * world, ceil(heads / world), head_dim]`` (the reference's
    output).  Same errors as the reference: ValueError when the weight is not
    3 x heads x head_dim rows, RuntimeError without torch.distributed."""
    if int(w_q.shape[0]) != 3 * num_heads * head_dim:
        raise ValueError("merged QKV width differs from heads * head_dim")
    if world > 1 and (not torch.distributed.is_available()
                      or not torch.distributed.is_initialized()):
        raise RuntimeError("Ulysses all-to-all requires initialized torch.distributed")
    send = qkv_send_buffer(q, q_scale, w_q, w_scale, bias, num_heads=num_heads,
                           head_dim=head_dim, world=world)
    return exchange_qkv(send, group=group)
