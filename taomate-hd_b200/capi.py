"""ctypes signatures of the C ABI in ``include/taomate_w8a8.h``.

This is the binding a non-torch host (or a test) uses to call the library
directly with device pointers, sizes and a CUDA stream handle.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

HEADER = Path(__file__).resolve().parent.parent / "include" / "taomate_w8a8.h"

c_int, c_i64, c_u32, c_float = ctypes.c_int, ctypes.c_int64, ctypes.c_uint32, ctypes.c_float
c_void_p, c_char_p = ctypes.c_void_p, ctypes.c_char_p
c_int_p = ctypes.POINTER(ctypes.c_int)

TM_OK = 0
TM_ERR_NULL_POINTER = 1
TM_ERR_SHAPE = 2
TM_ERR_ALIGNMENT = 3
TM_ERR_DTYPE = 4
TM_ERR_UNSUPPORTED = 5
TM_ERR_CUDA = 6
TM_ERR_DEVICE_TIMEOUT = 7
TM_ERR_TOO_LARGE = 8

TM_DTYPE_BF16 = 0
TM_DTYPE_FP16 = 1
TM_DTYPE_FP32 = 2

TM_EPI_GELU_TANH = 0x1
TM_EPI_SWIGLU = 0x2
TM_SPLITK_NOALLOC_MAX_BYTES = 16 << 20

_GEMM = [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p,
         c_i64, c_i64, c_i64, c_i64, c_i64, c_i64]

SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "tm_status_string": (c_char_p, [c_int]),
    "tm_version": (c_int, []),
    "tm_device_status": (c_int, [c_int, c_int_p, c_int]),
    "tm_dynamic_scaled_int8_quant": (
        c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_void_p]),
    "tm_static_scaled_int8_quant": (
        c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_void_p]),
    "tm_cutlass_scaled_mm": (c_int, [*_GEMM, c_void_p]),
    "tm_scaled_mm_i8_ex": (c_int, [*_GEMM, c_u32, c_void_p, c_void_p]),
    "tm_scaled_mm_i8_tile": (c_int, [*_GEMM, c_u32, c_void_p, c_int, c_void_p]),
    "tm_quantize_weight_int8": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_i64, c_i64, c_void_p]),
    "tm_scaled_mm_i8_all_reduce": (
        c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p,
                c_i64, c_i64, c_i64, c_i64, c_i64, c_void_p, c_void_p, c_void_p, c_int, c_int,
                c_u32, c_int, c_void_p]),
    "tm_scaled_mm_i8_reduce_scatter": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p,
                c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_void_p, c_void_p, c_int, c_int,
                c_u32, c_int, c_void_p]),
    "tm_scaled_mm_i8_workspace_size": (c_int, [c_i64, c_i64, c_i64, ctypes.POINTER(ctypes.c_uint64)]),
    "tm_scaled_mm_i8_ws": (c_int, [*_GEMM, c_u32, c_void_p, c_void_p, ctypes.c_uint64, c_void_p]),
    "tm_scaled_mm_i8_splitk": (
        c_int, [*_GEMM, c_u32, c_void_p, c_int, c_int, c_void_p, ctypes.c_uint64, c_void_p]),
    "tm_scaled_mm_i8_splitk_workspace_size": (
        c_int, [c_i64, c_i64, c_i64, c_int, c_int, ctypes.POINTER(ctypes.c_uint64)]),
    "tm_scaled_mm_i8_lora_reduce_scatter": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p,
                c_void_p, c_i64, c_void_p, c_i64, c_int, c_i64, c_i64, c_i64, c_i64, c_i64,
                c_i64, c_void_p, c_void_p, c_int, c_int, c_u32, c_void_p]),
    "tm_scaled_mm_i8_lora_all_reduce": (
        c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p,
                c_void_p, c_i64, c_void_p, c_i64, c_int, c_i64, c_i64, c_i64, c_i64, c_i64,
                c_void_p, c_void_p, c_void_p, c_int, c_int, c_u32, c_void_p]),
    "tm_scaled_mm_i8_ulysses_exchange": (
        c_int, [c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p, c_i64, c_i64,
                c_i64, c_i64, c_i64, c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_u32,
                c_void_p]),
    "tm_lora_down_proj": (
        c_int, [c_void_p, c_i64, c_void_p, c_i64, c_void_p, c_i64, c_int, c_i64, c_i64, c_void_p]),
    "tm_scaled_mm_i8_lora": (
        c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p,
                c_void_p, c_i64, c_void_p, c_i64, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                c_u32, c_void_p]),
    "tm_scaled_mm_i8_ulysses_send": (
        c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_i64, c_void_p, c_i64, c_void_p,
                c_i64, c_i64, c_i64, c_i64, c_i64, c_int, c_int, c_int, c_void_p]),
    "tm_scaled_mm_i8_splitk_noalloc": (c_int, [*_GEMM, c_u32, c_int, c_int, c_void_p]),
    "tm_peer_handle_size": (c_int, []),
    "tm_peer_alloc": (c_int, [ctypes.c_uint64, ctypes.POINTER(c_void_p), c_void_p]),
    "tm_peer_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "tm_peer_close": (c_int, [c_void_p]),
    "tm_peer_free": (c_int, [c_void_p]),
    "tm_modulate_int8_quant": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64,
                c_i64, c_i64, c_void_p]),
    "tm_rms_norm_modulate_int8_quant": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                c_void_p, c_i64, c_i64, c_i64, c_void_p]),
    "tm_residual_gate_rms_norm_modulate_int8_quant": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                c_float, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_void_p]),
}


def header_symbols(header: Path = HEADER) -> list[str]:
    """Names of every function declared in the public header."""
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(tm_[a-z0-9_]+)\s*\(", text)))


def declare(lib: ctypes.CDLL) -> ctypes.CDLL:
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def status_string(lib: ctypes.CDLL, status: int) -> str:
    return lib.tm_status_string(status).decode()
