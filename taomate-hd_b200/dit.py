"""W8A8 tensor-parallel DiT linear stages on preallocated buffers.

These are the shapes of the BASELINE configurations, built from the
package's operators (no reference counterpart as a class: the reference runs
the same linears inside its DiT block, model/layers.py:346-368, :502-523):

* ``TPW8A8MLP``        fc1 column-parallel (+bias, GELU-tanh in the GEMM
                       epilogue) -> per-token quant over the local K ->
                       fc2 row-parallel, partials summed by a row reduce-scatter
                       (NCCL, or fused into the GEMM epilogue over NVLink peer
                       memory) or an all-reduce.  ``reduce(partial) + bias``
                       (linear.py:284-289): the fused path adds the bias on the
                       owner after the sum; the NCCL paths let TP rank 0 add it
                       in its GEMM epilogue so that it enters the sum once.
* ``TPW8A8AttnProj``   merged QKV column-parallel (each of Q, K, V sharded
                       separately, linear.py:207-215) and the row-parallel
                       out-projection with an all-reduce (NCCL, or fused into
                       the GEMM launch over NVLink peer memory).
* ``TPW8A8BlockChain`` QKV, out-proj, fc1, fc2 of one block in sequence.

Every ``forward`` writes into buffers allocated at construction, so a step
allocates nothing and can be captured in a CUDA graph.  Weights are random
(``N(0, 0.02)``) and quantised per output channel on the GPU; row-parallel
weights are quantised after K-sharding, as the reference does.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops
from .collectives import all_reduce_sum_inplace_, reduce_scatter_rows
from .parallel import ParallelContext


@dataclass
class W8Weight:
    """int8 weight [N, K] with fp32 per-output-channel scales [N] and optional bias [N]."""

    q: torch.Tensor
    scale: torch.Tensor
    bias: torch.Tensor | None

    @property
    def q_t(self) -> torch.Tensor:
        return self.q.t()


def random_bf16(shape: tuple[int, ...], std: float, seed: int, device: torch.device) -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


def column_slice(full: torch.Tensor, world: int, rank: int,
                 output_sizes: tuple[int, ...] | None = None) -> torch.Tensor:
    """This rank's output rows of a column-parallel weight, bias or LoRA B.

    ``full`` stacks one or more logical projections along dim 0 (their row
    counts in ``output_sizes``; one projection when None).  Every projection
    is split into ``world`` equal parts on its own and the rank's parts are
    stacked in projection order, so a merged QKV shard is ``[Q_r; K_r; V_r]``
    and heads stay whole (the reference's per-projection merged sharding,
    distributed/linear.py:207-215, lora_checkpoint.py:73-88).
    """
    sizes = output_sizes or (int(full.shape[0]),)
    if sum(sizes) != full.shape[0]:
        raise ValueError(f"output sizes {sizes} do not add up to {full.shape[0]} rows")
    if any(s % world for s in sizes):
        raise ValueError(f"every output size must divide by the TP degree {world}")
    starts = torch.tensor([0, *sizes[:-1]]).cumsum(0).tolist()
    parts = [full[start + rank * (s // world): start + (rank + 1) * (s // world)]
             for start, s in zip(starts, sizes)]
    return torch.cat(parts, 0).contiguous() if len(parts) > 1 else parts[0].contiguous()


def row_slice(full: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's input columns (the K slice) of a row-parallel weight or LoRA A
    (distributed/linear.py:291-296, lora_checkpoint.py:91-97)."""
    k = int(full.shape[-1])
    if k % world:
        raise ValueError(f"K ({k}) must divide by the TP degree {world}")
    return full[..., rank * (k // world):(rank + 1) * (k // world)].contiguous()


def column_weight(
    n: int, k: int, ctx: ParallelContext, seed: int, device: torch.device, *,
    bias: bool, output_sizes: tuple[int, ...] | None = None,
) -> W8Weight:
    """Column-parallel shard of a random [n, k] weight (per-projection for merged)."""
    t, r = ctx.tp_world_size, ctx.tp_rank
    local_w = column_slice(random_bf16((n, k), 0.02, seed, device), t, r, output_sizes)
    q, s = ops.quantize_weight_int8(local_w)
    b = (column_slice(random_bf16((n,), 0.01, seed + 1, device), t, r, output_sizes)
         if bias else None)
    return W8Weight(q, s.reshape(-1), b)


def row_weight(
    n: int, k: int, ctx: ParallelContext, seed: int, device: torch.device, *, bias: bool
) -> W8Weight:
    """Row-parallel K-shard of a random [n, k] weight, quantised after sharding."""
    local_w = row_slice(random_bf16((n, k), 0.02, seed, device), ctx.tp_world_size, ctx.tp_rank)
    q, s = ops.quantize_weight_int8(local_w)
    b = random_bf16((n,), 0.01, seed + 1, device) if bias else None
    return W8Weight(q, s.reshape(-1), b)


class _Quant:
    """Preallocated per-token int8 activation buffers."""

    def __init__(self, rows: int, cols: int, device: torch.device):
        self.q = torch.empty(rows, cols, dtype=torch.int8, device=device)
        self.s = torch.empty(rows, 1, dtype=torch.float32, device=device)

    def __call__(self, x: torch.Tensor) -> None:
        torch.ops.taomate_w8a8.dynamic_scaled_int8_quant(self.q, x, self.s, None)


def _gemm(q: _Quant, w: W8Weight, out: torch.Tensor, *, bias: torch.Tensor | None,
          gelu: bool = False) -> torch.Tensor:
    torch.ops.taomate_w8a8.scaled_mm_i8_ex(out, q.q, w.q_t, q.s, w.scale, bias,
                                           ops.EPI_GELU_TANH if gelu else 0, None, 0)
    return out


_MLP_REDUCE = ("reduce_scatter", "fused_reduce_scatter", "all_reduce", "fused_all_reduce")


class TPW8A8MLP:
    """480p LOW-stage MLP, fc1 column + fc2 row (reduce-scatter)."""

    def __init__(self, tokens: int, d: int, ffn: int, ctx: ParallelContext, device: torch.device,
                 *, seed: int = 0, reduce: str = "reduce_scatter"):
        t = ctx.tp_world_size
        if ffn % t or (reduce == "reduce_scatter" and tokens % t):
            raise ValueError("ffn and tokens must divide by the TP degree")
        if reduce not in _MLP_REDUCE:
            raise ValueError(f"reduce must be one of {_MLP_REDUCE}")
        self.ctx, self.tokens, self.d, self.ffn, self.reduce = ctx, tokens, d, ffn, reduce
        self.fc1 = column_weight(ffn, d, ctx, seed + 10, device, bias=True)
        self.fc2 = row_weight(d, ffn, ctx, seed + 20, device, bias=True)
        local_ffn = ffn // t
        self.q1 = _Quant(tokens, d, device)
        self.h = torch.empty(tokens, local_ffn, dtype=torch.bfloat16, device=device)
        self.q2 = _Quant(tokens, local_ffn, device)
        self.partial = torch.empty(tokens, d, dtype=torch.bfloat16, device=device)
        scatter = reduce in ("reduce_scatter", "fused_reduce_scatter")
        rows_out = tokens // t if scatter and t > 1 else tokens
        self.out = torch.empty(rows_out, d, dtype=torch.bfloat16, device=device)
        self.peer = None
        if reduce == "fused_reduce_scatter" and t > 1:
            from .peer_reduce import PeerReduceScatter

            self.peer = PeerReduceScatter(ctx, tokens, d, device)
        self.peer_ar = None
        if reduce == "fused_all_reduce" and t > 1:
            from .peer_reduce import PeerAllReduce

            self.peer_ar = PeerAllReduce(ctx, tokens, d, device)

    @property
    def int8_ops(self) -> int:
        """Whole-job int8 GEMM operations of one forward (2 M N K per linear)."""
        return 2 * 2 * self.tokens * self.d * self.ffn

    # this package's kernel launches per forward: 2 quant + 2 GEMM (the fused
    # reduce-scatter runs inside the fc2 GEMM launch)
    launches_per_step = 4

    def forward(self, x: torch.Tensor, gemm_events: list | None = None) -> torch.Tensor:
        self.q1(x)
        if gemm_events is not None:
            gemm_events[0].record()
        _gemm(self.q1, self.fc1, self.h, bias=self.fc1.bias, gelu=True)
        if gemm_events is not None:
            gemm_events[1].record()
        self.q2(self.h)
        if gemm_events is not None:
            gemm_events[2].record()
        if self.peer is not None:
            # fc2 partial blocks go straight to their owners; bias added once there
            self.peer(self.q2.q, self.q2.s, self.fc2.q, self.fc2.scale, self.fc2.bias, self.out)
            if gemm_events is not None:
                gemm_events[3].record()
            return self.out
        if self.peer_ar is not None:
            y = self.peer_ar(self.q2.q, self.q2.s, self.fc2.q, self.fc2.scale, self.fc2.bias)
            if gemm_events is not None:
                gemm_events[3].record()
            return y
        bias2 = self.fc2.bias if self.ctx.tp_rank == 0 else None
        _gemm(self.q2, self.fc2, self.partial, bias=bias2)
        if gemm_events is not None:
            gemm_events[3].record()
        t = self.ctx.tp_world_size
        if t == 1:
            return self.partial
        if self.reduce == "reduce_scatter":
            return reduce_scatter_rows(self.partial, group=self.ctx.tp_group, world_size=t,
                                       out=self.out)
        return all_reduce_sum_inplace_(self.partial, group=self.ctx.tp_group, world_size=t)


class TPW8A8AttnProj:
    """merged QKV column-parallel + out-proj row-parallel (all-reduce)."""

    def __init__(self, tokens: int, d: int, heads: int, head_dim: int, ctx: ParallelContext,
                 device: torch.device, *, seed: int = 0, reduce: str = "all_reduce"):
        t = ctx.tp_world_size
        width = heads * head_dim
        if heads % t:
            raise ValueError("heads must divide by the TP degree")
        if reduce not in ("all_reduce", "fused_all_reduce"):
            raise ValueError("reduce must be 'all_reduce' or 'fused_all_reduce'")
        self.ctx, self.tokens, self.d, self.width = ctx, tokens, d, width
        self.qkv = column_weight(3 * width, d, ctx, seed + 30, device, bias=True,
                                 output_sizes=(width, width, width))
        self.out_proj = row_weight(d, width, ctx, seed + 40, device, bias=True)
        self.q_in = _Quant(tokens, d, device)
        self.qkv_out = torch.empty(tokens, 3 * width // t, dtype=torch.bfloat16, device=device)
        self.q_attn = _Quant(tokens, width // t, device)
        self.partial = torch.empty(tokens, d, dtype=torch.bfloat16, device=device)
        self.peer_ar = None
        if reduce == "fused_all_reduce" and t > 1:
            from .peer_reduce import PeerAllReduce

            self.peer_ar = PeerAllReduce(ctx, tokens, d, device)

    @property
    def int8_ops(self) -> int:
        return 2 * self.tokens * self.d * 3 * self.width + 2 * self.tokens * self.width * self.d

    launches_per_step = 4

    def forward(self, x: torch.Tensor, attn: torch.Tensor | None = None) -> torch.Tensor:
        """QKV of ``x``; out-proj of ``attn`` (the attention output; defaults to Q's shard)."""
        self.q_in(x)
        _gemm(self.q_in, self.qkv, self.qkv_out, bias=self.qkv.bias)
        a = self.qkv_out[:, : self.width // self.ctx.tp_world_size] if attn is None else attn
        self.q_attn(a)
        if self.peer_ar is not None:
            # partial blocks go to their row owners, reduced rows to every rank
            return self.peer_ar(self.q_attn.q, self.q_attn.s, self.out_proj.q,
                                self.out_proj.scale, self.out_proj.bias)
        bias = self.out_proj.bias if self.ctx.tp_rank == 0 else None
        _gemm(self.q_attn, self.out_proj, self.partial, bias=bias)
        t = self.ctx.tp_world_size
        if t == 1:
            return self.partial
        return all_reduce_sum_inplace_(self.partial, group=self.ctx.tp_group, world_size=t)


class TPW8A8BlockChain:
    """BASELINE configs[3] linear chain of one DiT block: QKV, out-proj, fc1, fc2."""

    def __init__(self, tokens: int, d: int, heads: int, head_dim: int, ffn: int,
                 ctx: ParallelContext, device: torch.device, *, seed: int = 0,
                 fused: bool = False):
        reduce = "fused_all_reduce" if fused else "all_reduce"
        self.attn = TPW8A8AttnProj(tokens, d, heads, head_dim, ctx, device, seed=seed,
                                   reduce=reduce)
        self.mlp = TPW8A8MLP(tokens, d, ffn, ctx, device, seed=seed + 100, reduce=reduce)

    @property
    def int8_ops(self) -> int:
        return self.attn.int8_ops + self.mlp.int8_ops

    launches_per_step = 8

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.attn.forward(x)
        return self.mlp.forward(h)


# ---------------------------------------------------------------- LoRA block stack
@dataclass
class LoRAShard:
    """This rank's LoRA factors: ``a`` bf16 ``[r, K_local]``; ``b`` bf16
    ``[N_local, r]`` already multiplied by the adapter scale alpha / r."""

    a: torch.Tensor
    b: torch.Tensor


def column_lora(n: int, k: int, rank: int, alpha: float, ctx: ParallelContext, seed: int,
                device: torch.device, output_sizes: tuple[int, ...] | None = None) -> LoRAShard:
    """Column LoRA shards (lora_checkpoint.py:73-88): full A, B sharded per projection."""
    a = random_bf16((rank, k), 0.02, seed, device)
    b_full = random_bf16((n, rank), 0.002, seed + 1, device)
    b_local = column_slice(b_full, ctx.tp_world_size, ctx.tp_rank, output_sizes)
    b = (b_local.float() * (alpha / rank)).to(torch.bfloat16).contiguous()
    return LoRAShard(a, b)


def row_lora(n: int, k: int, rank: int, alpha: float, ctx: ParallelContext, seed: int,
             device: torch.device) -> LoRAShard:
    """Row LoRA shards (lora_checkpoint.py:91-97): A sliced along K, full B."""
    a = row_slice(random_bf16((rank, k), 0.02, seed, device), ctx.tp_world_size, ctx.tp_rank)
    b = (random_bf16((n, rank), 0.002, seed + 1, device).float() * (alpha / rank)).to(torch.bfloat16)
    return LoRAShard(a, b.contiguous())


@dataclass
class _BlockWeights:
    qkv: W8Weight
    qkv_lora: LoRAShard
    out: W8Weight
    out_lora: LoRAShard
    fc1: W8Weight
    fc1_lora: LoRAShard
    fc2: W8Weight
    fc2_lora: LoRAShard


class TPW8A8LoRABlockStack:
    """``n_blocks`` chained 768p DiT block linear chains.

    Per block: adaLN modulate (per-token shift/scale) fused into the
    activation quant -> merged QKV (+bias, LoRA) -> out-projection of the
    attention output (the Q shard stands in for attention, which is outside
    the W8A8 path) (+bias, LoRA) and its row reduction -> modulate fused into
    the quant -> fc1 (+bias, LoRA, GELU-tanh) -> quant -> fc2 (+bias, LoRA)
    and its row reduction.  Every W8A8 linear adds its BF16 LoRA delta
    (rank 64, alpha 64) in the GEMM epilogue; the LoRA down-projection
    T = x A^T is this package's tcgen05 bf16 kernel (``lora_down_proj``).
    Row-parallel linears follow the reference's fused-row-reduce LoRA
    (lora_checkpoint.py:127-143): reduce(partial + update) + bias.  With
    ``fused=True`` (TP > 1) that reduction runs inside the LoRA GEMM launch
    over NVLink (``PeerAllReduce.lora``; one buffer pair serves the
    out-projection and fc2, which have the same shape); otherwise the bias
    goes on TP rank 0 and NCCL all-reduces.  Each block has its own random
    weights; activation buffers are shared by all blocks, so a forward
    allocates nothing.
    """

    def __init__(self, n_blocks: int, tokens: int, d: int, heads: int, head_dim: int, ffn: int,
                 ctx: ParallelContext, device: torch.device, *, rank: int = 64,
                 alpha: float = 64.0, seed: int = 0, fused: bool = False):
        t = ctx.tp_world_size
        width = heads * head_dim
        if heads % t or ffn % t:
            raise ValueError("heads and ffn must divide by the TP degree")
        self.ctx, self.tokens, self.d, self.width, self.ffn = ctx, tokens, d, width, ffn
        self.rank = rank
        self.blocks: list[_BlockWeights] = []
        for i in range(n_blocks):
            s = seed + 1000 * i
            sizes = (width, width, width)
            self.blocks.append(_BlockWeights(
                qkv=column_weight(3 * width, d, ctx, s + 30, device, bias=True, output_sizes=sizes),
                qkv_lora=column_lora(3 * width, d, rank, alpha, ctx, s + 35, device, sizes),
                out=row_weight(d, width, ctx, s + 40, device, bias=True),
                out_lora=row_lora(d, width, rank, alpha, ctx, s + 45, device),
                fc1=column_weight(ffn, d, ctx, s + 50, device, bias=True),
                fc1_lora=column_lora(ffn, d, rank, alpha, ctx, s + 55, device),
                fc2=row_weight(d, ffn, ctx, s + 60, device, bias=True),
                fc2_lora=row_lora(d, ffn, rank, alpha, ctx, s + 65, device)))
        # adaLN shift/scale, per token, shared by the blocks
        self.shift1 = random_bf16((tokens, d), 0.1, seed + 1, device)
        self.scale1 = random_bf16((tokens, d), 0.1, seed + 2, device)
        self.shift2 = random_bf16((tokens, d), 0.1, seed + 3, device)
        self.scale2 = random_bf16((tokens, d), 0.1, seed + 4, device)
        bf = dict(dtype=torch.bfloat16, device=device)
        self.q_in = _Quant(tokens, d, device)
        self.hidden = torch.empty(tokens, d, **bf)
        self.t_buf = torch.empty(tokens, rank, **bf)
        self.qkv_out = torch.empty(tokens, 3 * width // t, **bf)
        self.q_attn = _Quant(tokens, width // t, device)
        self.attn_out = torch.empty(tokens, d, **bf)
        self.h = torch.empty(tokens, ffn // t, **bf)
        self.q2 = _Quant(tokens, ffn // t, device)
        self.y = [torch.empty(tokens, d, **bf) for _ in range(2)]
        self.peer_ar = None
        if fused and t > 1:
            from .peer_reduce import PeerAllReduce

            self.peer_ar = PeerAllReduce(ctx, tokens, d, device)

    @property
    def int8_ops_per_block(self) -> int:
        """Whole-job int8 GEMM operations of one block (2 M N K per linear)."""
        m, d, w, f = self.tokens, self.d, self.width, self.ffn
        return 2 * m * (d * 3 * w + w * d + d * f + f * d)

    @property
    def lora_flops_per_block(self) -> int:
        """Whole-job bf16 LoRA flops of one block: 2 M r (K + N) per linear."""
        m, d, w, f, r = self.tokens, self.d, self.width, self.ffn, self.rank
        return 2 * m * r * ((d + 3 * w) + (w + d) + (d + f) + (f + d))

    # this package's kernel launches per block: 2 modulate-quant + 2 quant + 4
    # LoRA down-projections + 4 LoRA GEMMs
    launches_per_block = 12

    def _lora_linear(self, q: _Quant, w: W8Weight, lora: LoRAShard, x: torch.Tensor,
                     out: torch.Tensor, bias: torch.Tensor | None, gelu: bool = False) -> None:
        torch.ops.taomate_w8a8.lora_down_proj(self.t_buf, x, lora.a)
        torch.ops.taomate_w8a8.scaled_mm_i8_lora(out, q.q, w.q_t, q.s, w.scale, bias, self.t_buf,
                                                 lora.b, ops.EPI_GELU_TANH if gelu else 0)

    def _row_lora_linear(self, q: _Quant, w: W8Weight, lora: LoRAShard, x: torch.Tensor,
                         out: torch.Tensor) -> torch.Tensor:
        """Row-parallel LoRA linear and its reduction over the TP group."""
        if self.peer_ar is not None:
            torch.ops.taomate_w8a8.lora_down_proj(self.t_buf, x, lora.a)
            return self.peer_ar.lora(q.q, q.s, w.q, w.scale, w.bias, self.t_buf, lora.b)
        self._lora_linear(q, w, lora, x, out, w.bias if self.ctx.tp_rank == 0 else None)
        return self._reduce(out)

    def close(self) -> None:
        """Release the fused reduction's peer buffers (collective: every rank)."""
        if self.peer_ar is not None:
            self.peer_ar.check()
            self.peer_ar.close()
            self.peer_ar = None

    def _reduce(self, y: torch.Tensor) -> torch.Tensor:
        t = self.ctx.tp_world_size
        if t == 1:
            return y
        return all_reduce_sum_inplace_(y, group=self.ctx.tp_group, world_size=t)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for i, blk in enumerate(self.blocks):
            torch.ops.taomate_w8a8.modulate_int8_quant(self.q_in.q, self.q_in.s, self.hidden, x,
                                                       self.shift1, self.scale1, None)
            self._lora_linear(self.q_in, blk.qkv, blk.qkv_lora, self.hidden, self.qkv_out,
                              blk.qkv.bias)
            attn = self.qkv_out[:, : self.width // self.ctx.tp_world_size]
            self.q_attn(attn)
            a = self._row_lora_linear(self.q_attn, blk.out, blk.out_lora, attn, self.attn_out)
            torch.ops.taomate_w8a8.modulate_int8_quant(self.q_in.q, self.q_in.s, self.hidden, a,
                                                       self.shift2, self.scale2, None)
            self._lora_linear(self.q_in, blk.fc1, blk.fc1_lora, self.hidden, self.h, blk.fc1.bias,
                              gelu=True)
            self.q2(self.h)
            x = self._row_lora_linear(self.q2, blk.fc2, blk.fc2_lora, self.h, self.y[i % 2])
        return x
