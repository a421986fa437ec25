"""taomate_hd_b200: B200-native selective-W8A8 tensor-parallel DiT linear path.

A from-scratch sm_100a implementation of the path TaoMate-HD runs under
``--mode accelerated``: per-token dynamic int8 activation quantisation and
the scaled int8 GEMM (tcgen05 ``kind::i8``) behind the reference's operator
surface, the column/row tensor-parallel linears around them, and the LoRA
and adaLN pieces adjacent to the GEMM.

Modules
-------
ops          vLLM-compatible ``scaled_int8_quant`` / ``cutlass_scaled_mm`` and fused variants
w8a8         mirror of ``inference/w8a8.py`` (workspace, linear, weight conversion, policy)
parallel     ``ParallelContext`` (``distributed/parallel.py``)
collectives  NCCL reductions (``distributed/collectives.py``)
linear       Column / MergedColumn / Row parallel linears (``distributed/linear.py``)
lora         TP-aware LoRA wrapper (``inference/lora_checkpoint.py``)
capi         ctypes binding of the C ABI (``include/taomate_w8a8.h``)
build        in-tree build of the native libraries
"""
from __future__ import annotations

__version__ = "0.1.0"
