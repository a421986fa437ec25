"""Ulysses sequence-to-heads exchange of a W8A8 merged QKV projection.

The reference's inference path (src/taomate_hd/distributed/ulysses.py:166-212,
``merged_qkv_sequence_to_heads``) runs the merged QKV linear, permutes its
``[tokens, 3 * heads * head_dim]`` output into the all-to-all send layout
``[world, 3, tokens, ceil(heads / world), head_dim]`` (zero heads pad the last
shards when ``world`` does not divide ``heads``, ulysses.py:188-193) and
exchanges it.  Two forms here:

* ``merged_qkv_sequence_to_heads_w8a8``: the scaled GEMM's epilogue writes
  the send layout directly (``torch.ops.taomate_w8a8.scaled_mm_i8_ulysses_send``),
  so the projection output is never materialised in token-major order; the
  exchange is NCCL's all-to-all, and the receive layout the reference's.
* ``PeerUlyssesExchange``: the epilogue stores each head block straight into
  the receive buffer of the rank that holds the head, over NVLink
  (``tm_scaled_mm_i8_ulysses_exchange``); the launch returns with every
  rank's receive buffer complete, so there is no separate exchange.
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


class PeerUlyssesExchange:
    """The merged QKV projection and its Ulysses all-to-all in one launch.

    Per rank of the Ulysses ``group`` (``world`` ranks, this one ``rank``;
    the reference passes the group to ``merged_qkv_sequence_to_heads``),
    two receive buffer sets ``[world, 3, tokens, local, head_dim]``
    (``local = ceil(heads / world)``, zeroed once, so padded head slots stay
    zero) and their counters, shared across the group by CUDA IPC
    (``peer_reduce``'s buffers).  Every rank calls with its own ``tokens``
    rows, in the same order.  ``__call__`` returns the reference's
    ``(q, k, v)``, each ``[tokens * world, local, head_dim]`` (copies; with
    ``world == 1`` views valid until the second call after).  Waits inside
    the kernel are bounded; :meth:`check` raises when one ran out.
    :meth:`from_context` takes the Ulysses axis of a ``ParallelContext``.
    """

    def __init__(self, tokens: int, num_heads: int, head_dim: int, device: torch.device, *,
                 group=None, world: int = 1, rank: int = 0):
        from .parallel import ParallelContext
        from .peer_reduce import _PeerBuffers

        self.world, self.tokens = world, tokens
        self.num_heads, self.head_dim = num_heads, head_dim
        self.local = -(-num_heads // world)

        class _Buffers(_PeerBuffers):
            @staticmethod
            def _check_shape(rows: int, cols: int, world: int) -> None:
                if tokens % 32:
                    raise ValueError("tokens must be a multiple of 32")
                if head_dim % 64:
                    raise ValueError("head_dim must be a multiple of 64")

        # the buffer machinery is written over a TP-style context: here the
        # Ulysses group plays that role
        axis = ParallelContext(tp_world_size=world, tp_rank=rank, tp_group=group)
        self._buf = _Buffers(axis, world * 3 * tokens, self.local * head_dim, device)
        self.rank = rank
        self.device = device

    @classmethod
    def from_context(cls, ctx, tokens: int, num_heads: int, head_dim: int,
                     device: torch.device) -> "PeerUlyssesExchange":
        """Over the Ulysses axis of ``ctx`` (``ulysses_group``,
        ``ulysses_world_size``, ``ulysses_rank``)."""
        return cls(tokens, num_heads, head_dim, device, group=ctx.ulysses_group,
                   world=ctx.ulysses_world_size, rank=ctx.ulysses_rank)

    def __call__(self, q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
                 w_scale: torch.Tensor, bias: torch.Tensor | None) -> tuple[torch.Tensor, ...]:
        """(q, k, v) of int8 ``q`` ([tokens, d], per-token scales) against int8
        ``w_q`` ([3 * heads * head_dim, d], per-channel ``w_scale``)."""
        from .peer_reduce import _check_operands

        if int(w_q.shape[0]) != 3 * self.num_heads * self.head_dim:
            raise ValueError("merged QKV width differs from heads * head_dim")
        _check_operands(q, q_scale, w_q, w_scale, bias, self.tokens,
                        3 * self.num_heads * self.head_dim)
        buf = self._buf
        half, stream = buf._next_set()
        m, k = q.shape
        rc = buf._lib.tm_scaled_mm_i8_ulysses_exchange(
            q.data_ptr(), w_q.data_ptr(), q_scale.data_ptr(), q_scale.numel(),
            w_scale.data_ptr(), w_scale.numel(), None if bias is None else bias.data_ptr(),
            m, w_q.shape[0], k, q.stride(0), w_q.stride(0), self.num_heads, self.head_dim,
            buf._part[half], buf._counts[half], self.world, self.rank, buf._uses[half], stream)
        if rc != 0:
            buf._raise("tm_scaled_mm_i8_ulysses_exchange", rc)
        buf._after_call()
        from .peer_reduce import _wrap_bf16

        flat = _wrap_bf16(buf._part[half][self.rank], self.world * 3 * self.tokens,
                          self.local * self.head_dim, self.device)
        received = flat.view(self.world, 3, self.tokens, self.local, self.head_dim)
        if self.world == 1:
            return tuple(received[0].unbind(0))
        return receive_layout(received)

    def check(self) -> None:
        self._buf.check()

    def close(self) -> None:
        self._buf.close()
