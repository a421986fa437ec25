"""GPU: the BASELINE configs[3] block stack (modulate-fused quant, W8A8 + LoRA
epilogue, GELU) against the CPU oracle chained the same way.

Each stage of the oracle chain follows the reference: adaLN modulate
(fused_kernels.py:220-236), per-token quant (w8a8.py:71), the scaled GEMM
(w8a8.py:72), the LoRA composition (lora_checkpoint.py:144-154) and GELU.
Small shapes, TP=1, two chained blocks with their own weights.  Bf16
roundings may differ by a step where the kernel rounds the LoRA sum once, and
a step can move a token's int8 quantisation in the next layer, so the chain is
compared relative to its output scale.
"""
from __future__ import annotations

import pytest
import torch

from oracle import w8a8_oracle as orc

pytestmark = pytest.mark.gpu


def _linear_lora(x_bf16, w, lora, bias, gelu=False):
    q, s = orc.dynamic_scaled_int8_quant(x_bf16)
    y, _ = orc.scaled_mm(q, w.q.cpu().numpy(), s, w.scale.cpu().numpy(),
                         None if bias is None else bias.cpu(), torch.bfloat16)
    y = orc.lora_column(y, x_bf16, lora.a.cpu(), lora.b.cpu(), 1.0)  # b carries alpha / r
    return orc.gelu_tanh(y) if gelu else y


def test_lora_block_stack_matches_oracle_chain(cuda):
    from taomate_hd_b200.dit import TPW8A8LoRABlockStack
    from taomate_hd_b200.parallel import ParallelContext

    tokens, d, heads, head_dim, ffn = 512, 256, 2, 128, 1024
    ctx = ParallelContext(tp_world_size=1, tp_rank=0, tp_group=None)
    stack = TPW8A8LoRABlockStack(2, tokens, d, heads, head_dim, ffn, ctx, cuda, seed=5)
    x = orc.activation(tokens, d, seed=9, outlier_channels=1).to(torch.bfloat16)
    got = stack.forward(x.to(cuda)).cpu().float()

    width = heads * head_dim
    h = x
    for blk in stack.blocks:
        m1 = orc.modulate(h, stack.shift1.cpu(), stack.scale1.cpu(), None)
        qkv = _linear_lora(m1, blk.qkv, blk.qkv_lora, blk.qkv.bias)
        attn = qkv[:, :width].contiguous()
        a = _linear_lora(attn, blk.out, blk.out_lora, blk.out.bias)
        m2 = orc.modulate(a, stack.shift2.cpu(), stack.scale2.cpu(), None)
        f = _linear_lora(m2, blk.fc1, blk.fc1_lora, blk.fc1.bias, gelu=True)
        h = _linear_lora(f, blk.fc2, blk.fc2_lora, blk.fc2.bias)
    ref = h.float()
    scale = ref.abs().max().item()
    err = (got - ref).abs()
    assert err.max().item() <= 2e-2 * scale, (err.max().item(), scale)
    assert err.mean().item() <= 2e-3 * scale, (err.mean().item(), scale)
    assert stack.int8_ops_per_block == 2 * tokens * (d * 3 * width + width * d + 2 * d * ffn)
