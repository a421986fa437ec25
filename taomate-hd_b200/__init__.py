"""taomate_hd_b200: B200-native selective-W8A8 tensor-parallel DiT linear path.

A from-scratch sm_100a implementation of the path TaoMate-HD runs under
``--mode accelerated``: per-token dynamic int8 activation quantisation and
the scaled int8 GEMM (tcgen05 ``kind::i8``) behind the reference's operator
surface, the column/row tensor-parallel linears around them, and the LoRA
and adaLN pieces adjacent to the GEMM.

Modules
-------
ops            vLLM-compatible ``scaled_int8_quant`` / ``cutlass_scaled_mm``, the
               out-variant torch ops the reference's workspace calls, streamed
               weight conversion and the fused variants
fused_kernels  the reference's adaLN producer wrappers with the quant fused in
peer_reduce    row-parallel GEMM with its reduce-scatter / all-reduce in the launch
ulysses        merged QKV projection written in the Ulysses all-to-all send layout
dit            TP-sharded DiT linear stages on preallocated buffers (bench workloads)
parallel       ``ParallelContext`` (``distributed/parallel.py``)
collectives    NCCL reductions (``distributed/collectives.py``)
capi           ctypes binding of the C ABI (``include/taomate_w8a8.h``)
build          in-tree build of the native libraries

The reference's own host modules (``inference/w8a8.py``,
``distributed/linear.py``, ``inference/lora_checkpoint.py``) run unchanged on
top of ``ops``: they bind it by module name.
"""
from __future__ import annotations

__version__ = "0.1.0"
