"""Shared pytest configuration.

``-m gpu`` tests need a CUDA device (a B200) and the built in-tree native
libraries; everything else runs on CPU.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built extension")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"kernels are built for sm_100a only (device is sm_{major}{minor})")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def tm_ops(cuda):
    from taomate_hd_b200 import ops

    return ops


@pytest.fixture(scope="session")
def capi(cuda):
    from taomate_hd_b200 import _native

    return _native.capi()


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test, the library's device status word must read 0."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch

    if not torch.cuda.is_available():
        return
    import ctypes

    from taomate_hd_b200 import _native

    code = ctypes.c_int(-1)
    status = _native.capi().tm_device_status(0, ctypes.byref(code), 1)
    assert status == 0 and code.value == 0, f"device status {code.value} (call status {status})"
