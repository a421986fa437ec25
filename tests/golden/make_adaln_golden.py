"""Golden vectors for the adaLN producers and SwiGLU from the reference's own
Triton kernels, run on the CPU by Triton's interpreter.

The reference implements the W8A8 producers as Triton kernels
(src/taomate_hd/inference/fused_kernels.py): ``fused_modulate`` (:643-655,
kernel :219-235), ``fused_gate_add`` (:658-670, kernel :237-254),
``fused_rms_norm_modulate`` (:723-754, kernel :322-347),
``fused_residual_gate_rms_norm_modulate`` (:757-797, kernel :349-382) and
``fused_swiglu`` (:694-704, kernel :298-309).  With ``TRITON_INTERPRET=1``
Triton executes them in Python on CPU tensors, so their outputs can be
recorded here without a GPU.  The interpreter evaluates each operation in
numpy fp32; the elementwise steps (``_round_bf16`` of sums and products) are
therefore the kernels' own, while ``tl.rsqrt`` and ``tl.sum`` follow numpy
(the GPU's approximate rsqrt and reduction tree may differ in the last bit),
and ``tl.sigmoid`` is numpy's.

Needs the reference tree (``TAOMATE_REFERENCE_SRC`` = its ``src``
directory); the output ``adaln_triton.npz`` is committed so
the tests never need the reference or Triton.

Usage: ``python tests/golden/make_adaln_golden.py [outdir]``.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"  # before Triton is imported

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
_REFERENCE_SRC = os.environ.get("TAOMATE_REFERENCE_SRC")
if not _REFERENCE_SRC:
    raise SystemExit("set TAOMATE_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, _REFERENCE_SRC)

# (rows, columns): a masked tail (200 of a 256-wide block) and a full block
SHAPES = [(7, 200), (5, 256)]


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def main(outdir: str) -> int:
    from taomate_hd.inference import fused_kernels as ref

    if not ref._TRITON_AVAILABLE:
        raise SystemExit("Triton is not importable: cannot run the reference kernels")
    g = torch.Generator().manual_seed(808)
    arrays: dict[str, np.ndarray] = {}

    def bf(*shape, sd=1.0):
        return (torch.randn(*shape, generator=g) * sd).to(torch.bfloat16)

    for i, (rows, cols) in enumerate(SHAPES):
        x, branch, residual = bf(rows, cols), bf(rows, cols, sd=2.0), bf(rows, cols)
        # large magnitudes: products and sums that round to +-inf in bf16
        x[0, :4] = torch.tensor([3.0e38, -3.0e38, 1.0e-38, 0.0]).to(torch.bfloat16)
        residual[1, :2] = torch.tensor([3.3e38, -3.3e38]).to(torch.bfloat16)
        scale, shift, gate = bf(3, cols, sd=0.1), bf(3, cols, sd=0.1), bf(3, cols, sd=0.5)
        scale[2, :4] = torch.tensor([1.5, -1.0, 0.5, 3.0]).to(torch.bfloat16)
        weight = (1.0 + 0.1 * torch.randn(cols, generator=g)).to(torch.bfloat16)
        indices = torch.randint(0, 3, (rows,), generator=g)
        eps = 1e-6
        outputs = {
            "modulate": ref.fused_modulate(x, shift, scale, indices),
            "gate_add": ref.fused_gate_add(residual, gate, branch, indices),
            "rms_norm_modulate": ref.fused_rms_norm_modulate(
                x.clamp(-100, 100), weight, scale, shift, indices, eps),
        }
        res_value, res_hidden = ref.fused_residual_gate_rms_norm_modulate(
            residual.clamp(-100, 100), branch, gate, weight, scale, shift, indices, eps)
        outputs["residual_gate_value"] = res_value
        outputs["residual_gate_hidden"] = res_hidden
        swiglu_in = bf(rows, 2 * cols, sd=3.0)
        outputs["swiglu"] = ref.fused_swiglu(swiglu_in)
        inputs = {"x": x, "branch": branch, "residual": residual, "scale": scale,
                  "shift": shift, "gate": gate, "weight": weight, "swiglu_in": swiglu_in}
        for k, v in inputs.items():
            arrays[f"s{i}_{k}"] = bf16_bits(v)
        arrays[f"s{i}_indices"] = indices.numpy()
        arrays[f"s{i}_eps"] = np.array([eps], dtype=np.float64)
        for k, v in outputs.items():
            arrays[f"s{i}_out_{k}"] = bf16_bits(v)
    out_path = Path(outdir) / "adaln_triton.npz"
    np.savez_compressed(out_path, n_shapes=np.array([len(SHAPES)]), **arrays)
    print(f"wrote {out_path} ({len(SHAPES)} shapes)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main(sys.argv[1] if len(sys.argv) > 1 else str(HERE)))
