"""Generate golden vectors from the installed vLLM W8A8 operators (run on a GPU).

The reference's activation quantisation and scaled GEMM are vLLM's compiled
operators (src/taomate_hd/inference/w8a8.py:71-72, :141-144).  Their source
is not in the reference tree, so the CPU oracle's rounding is pinned against
the operators themselves: this script calls ``vllm._custom_ops`` on seeded
inputs and writes the inputs and outputs to ``<outdir>/vllm_quant.npz`` and
``<outdir>/vllm_scaled_mm.npz``.  bf16/fp16 tensors are stored as their raw
uint16 bits.

Cases include exact .5 rounding ties (to pin round-half-even), all-zero
rows, single-nonzero rows, saturating values and non-multiple-of-16 widths.

Usage (on the GPU box): ``python tests/golden/make_vllm_golden.py <outdir>``.
Exits 0 and writes ``vllm_unavailable.txt`` when vLLM's operators do not load.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def quant_cases() -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(1234)
    cases: dict[str, torch.Tensor] = {}
    x = torch.randn(64, 3072, generator=g)
    x[:, torch.randperm(3072, generator=g)[:8]] *= 20
    cases["normal_bf16"] = x.to(torch.bfloat16)
    cases["normal_fp16"] = torch.randn(40, 1536, generator=g).to(torch.float16)
    cases["normal_fp32"] = torch.randn(24, 640, generator=g)
    cases["odd_width_bf16"] = torch.randn(17, 1000, generator=g).to(torch.bfloat16)
    # Ties: amax = 127 makes 127/amax exactly 1, so k + 0.5 is an exact tie.
    ties = torch.zeros(8, 256)
    vals = torch.arange(-126.5, 127.0, 1.0)  # 254 exact halves
    ties[:, :254] = vals[torch.randperm(254, generator=g)]
    ties[:, 254] = 127.0
    ties[1] = -ties[1]
    cases["ties_bf16"] = ties.to(torch.bfloat16)
    special = torch.randn(6, 512, generator=g)
    special[0] = 0.0                      # all-zero row (padding tokens)
    special[1] = 0.0
    special[1, 17] = -3.0                 # single nonzero
    special[2] *= 1e-30                   # subnormal-range magnitudes (fp32)
    special[3] = torch.full((512,), 2.0)  # constant row
    special[4, ::2] = 1e4                 # large values
    cases["special_fp32"] = special
    cases["special_bf16"] = special.to(torch.bfloat16)
    return cases


def mm_cases() -> list[dict[str, object]]:
    g = torch.Generator().manual_seed(4321)
    out = []
    for (m, n, k, per_tok, per_ch, bias, dt) in [
        (200, 384, 512, True, True, False, torch.bfloat16),
        (200, 384, 512, True, True, True, torch.bfloat16),
        (96, 256, 3072, True, True, True, torch.bfloat16),
        (130, 272, 384, False, False, False, torch.float16),
        (64, 128, 1024, True, False, True, torch.float16),
    ]:
        a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
        b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
        sa = torch.rand(m if per_tok else 1, 1, generator=g) * 0.05 + 1e-3
        sb = torch.rand(1, n if per_ch else 1, generator=g) * 0.01 + 1e-4
        bb = (torch.randn(n, generator=g) * 0.01).to(dt) if bias else None
        out.append(dict(m=m, n=n, k=k, a=a, b=b, sa=sa, sb=sb, bias=bb, dtype=dt))
    return out


def main(outdir: str) -> int:
    root = Path(outdir)
    root.mkdir(parents=True, exist_ok=True)
    try:
        import vllm
        from vllm import _custom_ops as ops

        probe = torch.zeros(1, 16, device="cuda", dtype=torch.bfloat16)
        ops.scaled_int8_quant(probe)
    except Exception as exc:  # vLLM absent or its CUDA ops do not load here
        (root / "vllm_unavailable.txt").write_text(f"{type(exc).__name__}: {exc}\n")
        print(f"vLLM operators unavailable: {type(exc).__name__}: {exc}")
        return 0
    meta = {"vllm": vllm.__version__, "torch": torch.__version__,
            "device": torch.cuda.get_device_name(0)}
    quant = {}
    for name, x in quant_cases().items():
        q, s, _ = ops.scaled_int8_quant(x.cuda())
        quant[f"{name}.x"] = bits(x)
        quant[f"{name}.dtype"] = np.array(str(x.dtype))
        quant[f"{name}.q"] = q.cpu().numpy()
        quant[f"{name}.s"] = s.cpu().numpy().reshape(-1)
    np.savez_compressed(root / "vllm_quant.npz", meta=np.array(json.dumps(meta)), **quant)
    # vLLM's CUTLASS int8 kernels refuse sm_100 ("Int8 not supported on
    # SM100"); the scaled-GEMM vectors then come from vLLM's own Triton
    # implementation of the same operator (its fallback for other shapes).
    mm_impl = "cutlass_scaled_mm"
    scaled_mm = ops.cutlass_scaled_mm
    try:
        c0 = mm_cases()[0]
        scaled_mm(c0["a"].cuda(), c0["b"].cuda().t(), c0["sa"].cuda(), c0["sb"].cuda(),
                  c0["dtype"])
    except RuntimeError as exc:
        from vllm.model_executor.layers.quantization.compressed_tensors.triton_scaled_mm import (
            triton_scaled_mm,
        )

        mm_impl = f"triton_scaled_mm (cutlass_scaled_mm raised: {str(exc).splitlines()[0][:160]})"

        def scaled_mm(a, b, sa, sb, dtype, bias=None):
            # the Triton entry point takes per-channel scales as [N, 1]
            return triton_scaled_mm(a, b, sa, sb.reshape(-1, 1), dtype, bias)
    meta["scaled_mm_impl"] = mm_impl
    mm = {}
    for i, c in enumerate(mm_cases()):
        a, b = c["a"].cuda(), c["b"].cuda()
        bias = c["bias"].cuda() if c["bias"] is not None else None
        y = scaled_mm(a, b.t(), c["sa"].cuda(), c["sb"].cuda(), c["dtype"], bias)
        mm[f"{i}.a"] = c["a"].numpy()
        mm[f"{i}.b"] = c["b"].numpy()
        mm[f"{i}.sa"] = c["sa"].numpy().reshape(-1)
        mm[f"{i}.sb"] = c["sb"].numpy().reshape(-1)
        if bias is not None:
            mm[f"{i}.bias"] = bits(c["bias"])
        mm[f"{i}.dtype"] = np.array(str(c["dtype"]))
        mm[f"{i}.out"] = bits(y)
    np.savez_compressed(root / "vllm_scaled_mm.npz", meta=np.array(json.dumps(meta)),
                        count=np.array(len(mm_cases())), **mm)
    print(f"wrote {root / 'vllm_quant.npz'} and {root / 'vllm_scaled_mm.npz'} ({meta})")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1] if len(sys.argv) > 1 else str(Path(__file__).resolve().parent)))
