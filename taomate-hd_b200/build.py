"""Build the native libraries of the package in-tree.

* ``lib/libtaomate_w8a8.so``: every CUDA kernel plus the C ABI declared in
  ``include/taomate_w8a8.h``, compiled by nvcc for sm_100a only.
* ``lib/libtaomate_w8a8_torch.so``: the ``torch.ops.taomate_w8a8`` custom
  operators (C++, no CUDA code), linked against the C-ABI library.

A stamp file records a digest of every source and flag; ``is_current()``
compares it so that a stale binary is refused at import instead of being run.

Usage: ``python -m taomate_hd_b200.build [--force]``.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
HEADER = PKG.parent / "include" / "taomate_w8a8.h"
CAPI_SO = LIB / "libtaomate_w8a8.so"
TORCH_SO = LIB / "libtaomate_w8a8_torch.so"
STAMP = LIB / "build.stamp"

CUDA_SOURCES = ("runtime.cu", "quant.cu", "gemm_i8.cu", "peer_memory.cu", "lora_down.cu")
TORCH_SOURCES = ("torch_ops.cpp",)
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
NVCC_FLAGS = (*ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared")


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    if default.exists():
        return str(default)
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build taomate_hd_b200")


def _cuda_home() -> Path:
    return Path(_nvcc()).resolve().parent.parent


def source_digest() -> str:
    h = hashlib.sha256()
    for path in sorted(CSRC.iterdir()):
        if path.is_file():
            h.update(path.name.encode())
            h.update(path.read_bytes())
    h.update(HEADER.read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    h.update(Path(__file__).read_bytes())
    return h.hexdigest()


def is_current() -> bool:
    return (
        CAPI_SO.exists()
        and TORCH_SO.exists()
        and STAMP.exists()
        and STAMP.read_text().strip() == source_digest()
    )


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build command failed ({proc.returncode}):\n{' '.join(cmd)}\n"
                           f"{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout + proc.stderr, flush=True)


def build_capi(verbose: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    tmp = CAPI_SO.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", str(tmp), *(str(CSRC / s) for s in CUDA_SOURCES)]
    _run(cmd, verbose)
    os.replace(tmp, CAPI_SO)
    return CAPI_SO


def _cxx() -> str:
    """The host C++ compiler for the torch op library: the system ``g++`` on
    PATH (torch's own toolchain), not ``$CXX``.  A compiler that links
    libstdc++ statically would give the library a private copy of the iostream
    and locale machinery, and the first error message formatted inside an op
    (TORCH_CHECK with a number) would crash instead of raising."""
    cxx = shutil.which("g++")
    if cxx is None:
        raise RuntimeError("g++ not found on PATH")
    return cxx


def build_torch_ops(verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    LIB.mkdir(exist_ok=True)
    includes = [f"-I{p}" for p in cpp_extension.include_paths(device_type="cuda")]
    includes.append(f"-I{_cuda_home() / 'include'}")
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_SO.with_suffix(".so.tmp")
    cmd = [
        _cxx(), "-O2", "-std=c++17", "-fPIC", "-shared",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *includes,
        *(str(CSRC / s) for s in TORCH_SOURCES),
        "-o", str(tmp),
        f"-L{LIB}", "-ltaomate_w8a8",
        f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
        "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}",
    ]
    _run(cmd, verbose)
    _require_shared_libstdcxx(tmp)
    os.replace(tmp, TORCH_SO)
    return TORCH_SO


def _require_shared_libstdcxx(path: Path) -> None:
    """Refuse a torch op library that does not load the shared libstdc++."""
    needed = subprocess.run(["readelf", "-d", str(path)], capture_output=True, text=True)
    if needed.returncode == 0 and "libstdc++.so" not in needed.stdout:
        raise RuntimeError(f"{path.name} does not link libstdc++ dynamically; check the C++ compiler")


def build(force: bool = False, verbose: bool = False) -> None:
    """Build both libraries unless the stamp says they match the sources."""
    if not force and is_current():
        return
    digest = source_digest()
    build_capi(verbose)
    build_torch_ops(verbose)
    STAMP.write_text(digest + "\n")


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args(argv)
    build(force=args.force, verbose=args.verbose)
    print(f"built {CAPI_SO}\nbuilt {TORCH_SO}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
