"""Generate golden vectors by running the reference's own (pure-torch) code.

Runs only where the reference tree is available (``TAOMATE_REFERENCE_SRC`` =
its ``src`` directory); its output files are committed so the tests never
need the reference at run time.

Captured, each from the reference function named:

* ``_quantize_cutlass_w8a8_weight``        inference/w8a8.py:175-179
* streamed loading in bounded chunks       inference/w8a8.py:182-242
* ``resolve_h3_cutlass_w8a8_policy``       inference/w8a8.py:89-114
* column / merged-column / row sharding    distributed/linear.py:161-225, :291-296
* LoRA shard helpers                       inference/lora_checkpoint.py:73-97
* ``cutlass_w8a8_linear`` host composition inference/w8a8.py:117-145, with its
  vLLM backend replaced by a stub whose arithmetic is the CPU oracle (the
  vLLM operators need a GPU)
* the inference LoRA wrapper forward       inference/lora_checkpoint.py:100-154,
  through ``apply_h3_lora_checkpoint`` on a synthetic adapter

Usage: ``python tests/golden/make_reference_golden.py [outdir]``.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
_REFERENCE_SRC = os.environ.get("TAOMATE_REFERENCE_SRC")
if not _REFERENCE_SRC:
    raise SystemExit("set TAOMATE_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, _REFERENCE_SRC)

from oracle import w8a8_oracle as orc  # noqa: E402


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def main(outdir: str) -> int:
    from taomate_hd.distributed import linear as ref_linear
    from taomate_hd.distributed.parallel import ParallelContext
    from taomate_hd.inference import lora_checkpoint as ref_lora
    from taomate_hd.inference import w8a8 as ref_w8a8

    out = Path(outdir)
    out.mkdir(parents=True, exist_ok=True)
    arrays: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(2024)

    # --- weight conversion (w8a8.py:175-179)
    for name, (n, k) in {"w_small": (96, 200), "w_wide": (64, 3072)}.items():
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        w[0] = 0.0                                    # zero row -> 1e-12 clamp
        w[1, :4] = torch.tensor([0.5, -0.5, 1.5, -127.0 * 0.01]).to(torch.bfloat16)
        q, s = ref_w8a8._quantize_cutlass_w8a8_weight(torch, w)
        arrays[f"{name}.w"] = bf16_bits(w)
        arrays[f"{name}.q"] = q.numpy()
        arrays[f"{name}.s"] = s.numpy().reshape(-1)

    # --- streamed loading in tiny chunks equals whole-matrix conversion
    src = (torch.randn(40, 96, generator=g) * 0.02).to(torch.bfloat16)
    mod = torch.nn.Module()
    mod.weight = torch.nn.Parameter(torch.empty(40, 96, dtype=torch.bfloat16), requires_grad=False)
    mod.bias = None
    ref_w8a8.prepare_cutlass_w8a8_stream_load_slot_(torch, mod, name="probe")
    ref_w8a8.load_cutlass_w8a8_stream_weight_(torch, mod, src, name="probe",
                                              maximum_temporary_bytes=1000)
    arrays["stream.src"] = bf16_bits(src)
    arrays["stream.q"] = mod.weight.detach().numpy()
    arrays["stream.s"] = mod._cutlass_w8a8_weight_scale.numpy().reshape(-1)

    # --- policy (w8a8.py:89-114)
    names = [f"blocks.{i}.{s}" for i in range(50)
             for s in ("attn.qkv_proj", "attn.out_proj", "mlp.fc1", "mlp.fc2")]
    names += ["final_layer.linear"]
    policy = ref_w8a8.resolve_h3_cutlass_w8a8_policy(
        names, policy=ref_w8a8.INTERIOR_FC1_QKV_CUTLASS_W8A8_POLICY)
    policy_errors = {}
    for label, bad in {"refiner_name": names + ["token_refiner.blocks.0.attn.qkv_proj"],
                       "no_candidates": ["final_layer.linear"]}.items():
        try:
            ref_w8a8.resolve_h3_cutlass_w8a8_policy(
                bad, policy=ref_w8a8.INTERIOR_FC1_QKV_CUTLASS_W8A8_POLICY)
            policy_errors[label] = None
        except Exception as exc:
            policy_errors[label] = type(exc).__name__
    try:
        ref_w8a8.resolve_h3_cutlass_w8a8_policy(names, policy="other")
        policy_errors["unknown_policy"] = None
    except Exception as exc:
        policy_errors["unknown_policy"] = type(exc).__name__
    shuffled = names[::-1]
    policy_shuffled = ref_w8a8.resolve_h3_cutlass_w8a8_policy(
        shuffled, policy=ref_w8a8.INTERIOR_FC1_QKV_CUTLASS_W8A8_POLICY)

    # --- TP sharding (linear.py) and LoRA shard helpers (lora_checkpoint.py)
    full_qkv = torch.randn(3 * 48, 32, generator=g).to(torch.bfloat16)
    full_row = torch.randn(24, 64, generator=g).to(torch.bfloat16)
    full_bias = torch.randn(3 * 48, generator=g).to(torch.bfloat16)
    arrays["shard.full_qkv"] = bf16_bits(full_qkv)
    arrays["shard.full_row"] = bf16_bits(full_row)
    arrays["shard.full_bias"] = bf16_bits(full_bias)
    lora_b = torch.randn(3 * 48, 4, generator=g)
    lora_a = torch.randn(4, 64, generator=g)
    arrays["shard.lora_b"] = lora_b.numpy()
    arrays["shard.lora_a"] = lora_a.numpy()
    for tp in (1, 2, 4):
        for rank in range(tp):
            ctx = ParallelContext(tp_world_size=tp, tp_rank=rank,
                                  tp_group=object() if tp > 1 else None)
            merged = ref_linear.MergedColumnParallelLinear(
                32, (48, 48, 48), bias=True, gather_output=False, dtype=torch.bfloat16, context=ctx)
            col = ref_linear.ColumnParallelLinear(
                32, 144, bias=True, gather_output=False, dtype=torch.bfloat16, context=ctx)
            row = ref_linear.RowParallelLinear(
                64, 24, bias=False, input_is_parallel=True, dtype=torch.bfloat16, context=ctx)
            arrays[f"shard.tp{tp}.r{rank}.merged_w"] = bf16_bits(merged.full_weight_slice(full_qkv))
            arrays[f"shard.tp{tp}.r{rank}.merged_b"] = bf16_bits(merged.full_bias_slice(full_bias))
            arrays[f"shard.tp{tp}.r{rank}.column_w"] = bf16_bits(col.full_weight_slice(full_qkv))
            arrays[f"shard.tp{tp}.r{rank}.row_w"] = bf16_bits(row.full_weight_slice(full_row))
            arrays[f"shard.tp{tp}.r{rank}.lora_b"] = ref_lora._column_local_b(lora_b, merged).numpy()
            arrays[f"shard.tp{tp}.r{rank}.lora_a"] = ref_lora._row_local_a(lora_a, row).numpy()

    # --- cutlass_w8a8_linear host composition with an oracle-backed backend
    def stub_quant(x):
        q, s = orc.dynamic_scaled_int8_quant(x)
        return torch.from_numpy(q), torch.from_numpy(s).reshape(-1, 1), None

    def stub_mm(q, w_t, sa, sb, dtype, bias=None):
        y, _ = orc.scaled_mm(q.numpy(), w_t.t().contiguous().numpy(), sa.numpy(), sb.numpy(),
                             bias, dtype)
        return y

    stub = SimpleNamespace(scaled_int8_quant=stub_quant, cutlass_scaled_mm=stub_mm)
    original = ref_w8a8.require_vllm_cutlass_w8a8
    ref_w8a8.require_vllm_cutlass_w8a8 = lambda: stub
    try:
        x = orc.activation(2 * 5, 256, seed=77).reshape(2, 5, 256)
        w = (torch.randn(128, 256, generator=g) * 0.02).to(torch.bfloat16)
        wq, ws = ref_w8a8._quantize_cutlass_w8a8_weight(torch, w)
        y = ref_w8a8.cutlass_w8a8_linear(torch, x, wq, ws, bias=None)
        try:
            ref_w8a8.cutlass_w8a8_linear(torch, x, wq, ws, bias=torch.zeros(128))
            bias_rejected = False
        except RuntimeError:
            bias_rejected = True
    finally:
        ref_w8a8.require_vllm_cutlass_w8a8 = original
    arrays["linear.x"] = bf16_bits(x)
    arrays["linear.wq"] = wq.numpy()
    arrays["linear.ws"] = ws.numpy().reshape(-1)
    arrays["linear.y"] = bf16_bits(y)

    # --- LoRA wrapper forward through apply_h3_lora_checkpoint (TP=1, BF16 base)
    d, ffn, rank_r, alpha = 32, 64, 4, 8.0
    model = torch.nn.Module()
    lora_state = {}
    for target in ref_lora.canonical_h3_lora_targets():
        parts = target.split(".")
        parent = model
        for part in parts[:-1]:
            if not hasattr(parent, part):
                parent.add_module(part, torch.nn.Module())
            parent = getattr(parent, part)
        suffix = ".".join(parts[-2:])
        if suffix in ("attn.qkv_proj", "mlp.fc1"):
            sizes = (d, d, d) if suffix == "attn.qkv_proj" else (ffn,)
            layer = ref_linear.MergedColumnParallelLinear(
                d, sizes, bias=False, gather_output=False, dtype=torch.bfloat16)
        else:
            in_size = d if suffix == "attn.out_proj" else ffn
            layer = ref_linear.RowParallelLinear(
                in_size, d, bias=False, input_is_parallel=True, dtype=torch.bfloat16)
        with torch.no_grad():
            layer.weight.copy_((torch.randn(layer.weight.shape, generator=g) * 0.05).to(torch.bfloat16))
        parent.add_module(parts[-1], layer)
        lora_state[f"{target}.lora_a"] = torch.randn(rank_r, layer.input_size, generator=g) * 0.02
        lora_state[f"{target}.lora_b"] = torch.randn(layer.output_size, rank_r, generator=g) * 0.002
    from safetensors.torch import save_file

    with tempfile.TemporaryDirectory() as adapter_dir:
        save_file(lora_state, str(Path(adapter_dir) / "adapter_model.safetensors"))
        (Path(adapter_dir) / "config.json").write_text(json.dumps({"rank": rank_r, "alpha": alpha}))
        receipt = ref_lora.apply_h3_lora_checkpoint(model, adapter_dir)
    ref_lora.materialize_h3_lora_bf16_buffers_(model)
    xl = torch.randn(6, d, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        qkv_wrapper = model.get_submodule("blocks.3.attn.qkv_proj")
        out_wrapper = model.get_submodule("blocks.3.attn.out_proj")
        y_qkv = qkv_wrapper(xl)
        y_out = out_wrapper(xl)
    arrays["lora.x"] = bf16_bits(xl)
    arrays["lora.qkv_w"] = bf16_bits(qkv_wrapper.base.weight.detach())
    arrays["lora.qkv_a"] = bf16_bits(qkv_wrapper.lora_a)
    arrays["lora.qkv_b"] = bf16_bits(qkv_wrapper.lora_b)
    arrays["lora.qkv_y"] = bf16_bits(y_qkv)
    arrays["lora.out_w"] = bf16_bits(out_wrapper.base.weight.detach())
    arrays["lora.out_a"] = bf16_bits(out_wrapper.lora_a)
    arrays["lora.out_b"] = bf16_bits(out_wrapper.lora_b)
    arrays["lora.out_y"] = bf16_bits(y_out)
    arrays["lora.scale"] = np.array(receipt["scale"], dtype=np.float64)

    np.savez_compressed(out / "reference_host.npz", **arrays)
    meta = {
        "source": "TaoLiveAIGC/TaoMate-HD reference functions, run on CPU by this script",
        "policy": policy,
        "policy_input_names": names,
        "policy_reversed_input": policy_shuffled,
        "policy_errors": policy_errors,
        "linear_bias_rejected": bias_rejected,
        "lora_receipt": {k: receipt[k] for k in ("rank", "alpha", "scale", "target_count")},
    }
    (out / "reference_host.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"wrote {out / 'reference_host.npz'} and {out / 'reference_host.json'}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1] if len(sys.argv) > 1 else str(HERE)))
