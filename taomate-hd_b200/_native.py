"""Load the native libraries built by :mod:`taomate_hd_b200.build`.

There is no fallback: if the libraries are missing or older than the sources,
loading raises, so nothing in this package can silently run a CPU or stale
implementation.
"""
from __future__ import annotations

import ctypes
import threading

from . import build as _build

_lock = threading.Lock()
_torch_ops_loaded = False
_capi: ctypes.CDLL | None = None


class NativeLibraryError(RuntimeError):
    """The CUDA extension of taomate_hd_b200 is missing or stale."""


def _require_current() -> None:
    if not _build.is_current():
        raise NativeLibraryError(
            "taomate_hd_b200 native libraries are missing or stale; build them with "
            "`python -m taomate_hd_b200.build` (sm_100a, in-tree)"
        )


def load_torch_ops() -> None:
    """Register torch.ops.taomate_w8a8.* (idempotent)."""
    global _torch_ops_loaded
    with _lock:
        if _torch_ops_loaded:
            return
        _require_current()
        import torch

        torch.ops.load_library(str(_build.TORCH_SO))
        _torch_ops_loaded = True


def capi() -> ctypes.CDLL:
    """The C-ABI library (ctypes handle with declared signatures)."""
    global _capi
    with _lock:
        if _capi is None:
            _require_current()
            from .capi import declare

            _capi = declare(ctypes.CDLL(str(_build.CAPI_SO)))
        return _capi
