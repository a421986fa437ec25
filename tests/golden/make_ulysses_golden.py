"""Golden vectors for the Ulysses send layout, from the reference's own code.

Runs ``merged_qkv_sequence_to_heads`` (src/taomate_hd/distributed/
ulysses.py:166-212) in a one-process ``gloo`` group with its ``_all_to_all``
(:12-16) replaced by an identity copy, and records the send buffer the
reference builds (``_merged_qkv_send_layout`` :153-163, with the zero-head
padding of :188-193 when the degree does not divide the heads) and the
(q, k, v) it returns from that buffer.  Needs the reference tree
(``TAOMATE_REFERENCE_SRC`` = its ``src`` directory); the output
``ulysses_send.npz`` is committed so the tests never need the reference.

Usage: ``python tests/golden/make_ulysses_golden.py [outdir]``.
"""
from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
_REFERENCE_SRC = os.environ.get("TAOMATE_REFERENCE_SRC")
if not _REFERENCE_SRC:
    raise SystemExit("set TAOMATE_REFERENCE_SRC to the reference checkout's src directory")
sys.path.insert(0, _REFERENCE_SRC)

# (tokens, heads, head_dim, degree): divisible, padded by 2, padded by 1, degree 1
CASES = [(6, 4, 4, 2), (5, 6, 8, 4), (3, 24, 2, 5), (4, 3, 4, 1)]


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def main(outdir: str) -> int:
    from taomate_hd.distributed import ulysses as ref

    captured: list[torch.Tensor] = []

    def identity_all_to_all(outputs, inputs, group):
        captured.append(inputs.clone())
        outputs.copy_(inputs)

    ref._all_to_all = identity_all_to_all
    with tempfile.TemporaryDirectory() as tmp:
        torch.distributed.init_process_group(
            "gloo", init_method=f"file://{tmp}/store", rank=0, world_size=1)
        arrays: dict[str, np.ndarray] = {}
        g = torch.Generator().manual_seed(77)
        for i, (tokens, heads, head_dim, degree) in enumerate(CASES):
            value = torch.randn(tokens, 3 * heads * head_dim, generator=g).to(torch.bfloat16)
            context = SimpleNamespace(ulysses_world_size=degree, ulysses_group=object())
            captured.clear()
            out = ref.merged_qkv_sequence_to_heads(value, num_heads=heads, head_dim=head_dim,
                                                   context=context)
            arrays[f"case{i}_shape"] = np.array([tokens, heads, head_dim, degree], dtype=np.int64)
            arrays[f"case{i}_value"] = bf16_bits(value)
            arrays[f"case{i}_qkv"] = bf16_bits(torch.stack(out))
            if degree > 1:
                assert len(captured) == 1
                arrays[f"case{i}_send"] = bf16_bits(captured[0])
        torch.distributed.destroy_process_group()
    out_path = Path(outdir) / "ulysses_send.npz"
    np.savez_compressed(out_path, **arrays)
    print(f"wrote {out_path} ({len(CASES)} cases)")
    return 0


if __name__ == "__main__":
    raise SystemExit(main(sys.argv[1] if len(sys.argv) > 1 else str(HERE)))
