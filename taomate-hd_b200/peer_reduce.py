"""Fused row-parallel reduce-scatter / all-reduce over NVLink peer memory.

The row-parallel linears of the reference sum their partial outputs with an
NCCL all-reduce after the GEMM (src/taomate_hd/distributed/linear.py:279-289,
collectives.py:19-40).  These classes run the reduction inside the
scaled-GEMM kernel instead:

* ``PeerReduceScatter`` (``tm_scaled_mm_i8_reduce_scatter``): the epilogue
  pushes each bf16 partial block to the rank that owns those rows over
  NVLink while the GEMM keeps running; each CTA then drains its stores once
  and bumps per-source counters on the owners; CTAs out of GEMM tiles wait
  for the counters and reduce their own rows from local memory.
* ``PeerAllReduce`` (``tm_scaled_mm_i8_all_reduce``): the same, after which
  every owner pushes its reduced rows into every rank's full output and the
  kernel returns once all owners' rows have arrived.

Each rank allocates one buffer holding two sets (alternate calls) of
``world`` receive slots (``rows x cols`` bf16 in total), the counters and,
for the all-reduce, a ``rows x cols`` output; shares it by CUDA IPC handle
over the TP process group, and maps every peer's buffer once.  All ranks must
call in the same order with the same shapes and tile configuration; the
per-set use counts are kept identically on every rank.

Failure reporting: every wait inside the kernel is bounded (1 s).  A wait
that runs out (a peer that never contributes) records a device status word
and overwrites the rows the kernel could not produce with NaN in this rank's
own output; it never hangs.  The launch itself still returns success, because
the host does not wait for the kernel: call :meth:`check` at a point where a
device synchronisation is acceptable (or pass ``check_every=N`` to have every
Nth call do it), which raises ``RuntimeError`` when the status word is set.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native
from .parallel import ParallelContext


def _align(value: int, to: int = 256) -> int:
    return (value + to - 1) // to * to


class _DeviceArray:
    """``__cuda_array_interface__`` over memory this module allocated."""

    def __init__(self, ptr: int, shape: tuple[int, ...]):
        self.__cuda_array_interface__ = {
            "shape": shape, "typestr": "<i2", "data": (ptr, False), "version": 3, "strides": None}


def _wrap_bf16(ptr: int, rows: int, cols: int, device: torch.device) -> torch.Tensor:
    """A bf16 ``[rows, cols]`` tensor aliasing device memory at ``ptr`` (no copy)."""
    with torch.cuda.device(device):
        t = torch.as_tensor(_DeviceArray(ptr, (rows, cols)), device=device)
    return t.view(torch.bfloat16)


def _require_cuda(t, name: str) -> None:
    if getattr(t, "device", None) is None or t.device.type != "cuda":
        raise RuntimeError(f"{name} must be a CUDA tensor")


def _check_operands(q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
                    w_scale: torch.Tensor, bias: torch.Tensor | None, rows: int,
                    cols: int) -> tuple[int, int]:
    """The GEMM operands of the fused calls, checked before anything reaches
    the device (the kernels read ``rows`` token scales or one, ``cols``
    channel scales or one, and ``cols`` bias values): ``q`` int8
    ``[rows, k]`` and ``w_q`` int8 ``[cols, k]`` with contiguous rows, fp32
    contiguous scales, bf16 contiguous bias, all on CUDA.  Returns (rows, k)."""
    for t, name in ((q, "q"), (w_q, "w_q")):
        if getattr(t, "dtype", None) != torch.int8 or t.dim() != 2:
            raise ValueError(f"{name} must be a 2-D int8 tensor")
        _require_cuda(t, name)
        if t.stride(1) != 1:
            raise ValueError(f"{name} rows must be contiguous")
    m, k = q.shape
    if m != rows or w_q.shape[0] != cols or w_q.shape[1] != k:
        raise ValueError("shape differs from the one the buffers were built for")
    for t, name, n in ((q_scale, "q_scale", rows), (w_scale, "w_scale", cols)):
        if (getattr(t, "dtype", None) != torch.float32 or not t.is_contiguous()
                or t.numel() not in (1, n)):
            raise ValueError(f"{name} must be contiguous float32 with 1 or {n} values")
        _require_cuda(t, name)
    if bias is not None:
        if (getattr(bias, "dtype", None) != torch.bfloat16 or not bias.is_contiguous()
                or bias.numel() != cols):
            raise ValueError(f"bias must be contiguous bfloat16 with {cols} values")
        _require_cuda(bias, "bias")
    return m, k


def _check_lora(lora_t: torch.Tensor, lora_b: torch.Tensor, rows: int, cols: int) -> int:
    """The LoRA operands of the fused row-parallel linears: ``lora_t`` bf16
    ``[rows, r]`` and ``lora_b`` bf16 ``[cols, r]`` on CUDA, rows contiguous,
    r in {8, 16, ..., 64}.  The kernel's tensor maps assume these extents,
    so they are checked here before any launch.  Returns r."""
    for name, t in (("lora_t", lora_t), ("lora_b", lora_b)):
        if getattr(t, "dtype", None) != torch.bfloat16 or t.dim() != 2:
            raise ValueError(f"{name} must be a 2-D bfloat16 tensor")
        _require_cuda(t, name)
        if t.stride(1) != 1:
            raise ValueError(f"{name} rows must be contiguous")
    r = lora_t.shape[1]
    if lora_t.shape[0] != rows or tuple(lora_b.shape) != (cols, r):
        raise ValueError(f"lora_t must be [{rows}, r] and lora_b [{cols}, r]")
    if r < 8 or r > 64 or r % 8:
        raise ValueError("the LoRA rank must be a multiple of 8 up to 64")
    return r


class _PeerBuffers:
    """Two buffer sets per rank, shared across the TP group by CUDA IPC."""

    _gather = False

    def __init__(self, ctx: ParallelContext, rows: int, cols: int, device: torch.device,
                 *, check_every: int = 0):
        world, rank = ctx.tp_world_size, ctx.tp_rank
        if check_every < 0:
            raise ValueError("check_every must be >= 0")
        self.check_every = check_every
        if world < 1 or world > 8:
            raise ValueError("the fused reduction supports 1..8 ranks")
        self._check_shape(rows, cols, world)
        self.ctx, self.rows, self.cols, self.device = ctx, rows, cols, device
        self.world, self.rank = world, rank
        self.rows_per_owner = rows // world
        self._lib = _native.capi()
        self._own = None
        part_bytes = _align(rows * cols * 2)
        count_bytes = _align(world * 8 * (2 if self._gather else 1))
        out_bytes = part_bytes if self._gather else 0
        self._half = part_bytes + count_bytes + out_bytes
        handle_size = self._lib.tm_peer_handle_size()
        handle = (ctypes.c_char * handle_size)()
        base = ctypes.c_void_p()
        with torch.cuda.device(device):
            rc = self._lib.tm_peer_alloc(2 * self._half, ctypes.byref(base), handle)
            if rc != 0:
                raise RuntimeError(f"tm_peer_alloc failed: {self._lib.tm_status_string(rc).decode()}")
            torch.cuda.synchronize(device)
        self._own = base.value
        self._opened: list[int] = []
        bases = [0] * world
        bases[rank] = self._own
        if world > 1:
            gathered: list[bytes | None] = [None] * world
            torch.distributed.all_gather_object(gathered, bytes(handle), group=ctx.tp_group)
            with torch.cuda.device(device):
                for j, h in enumerate(gathered):
                    if j == rank:
                        continue
                    ptr = ctypes.c_void_p()
                    buf = (ctypes.c_char * handle_size).from_buffer_copy(h)
                    rc = self._lib.tm_peer_open(buf, ctypes.byref(ptr))
                    if rc != 0:
                        self.close()
                        raise RuntimeError(
                            f"tm_peer_open(rank {j}) failed: {self._lib.tm_status_string(rc).decode()}")
                    bases[j] = ptr.value
                    self._opened.append(ptr.value)
            torch.distributed.barrier(group=ctx.tp_group)
        arr = ctypes.c_void_p * world
        self._part = [arr(*[b + h * self._half for b in bases]) for h in (0, 1)]
        self._counts = [arr(*[b + h * self._half + part_bytes for b in bases]) for h in (0, 1)]
        self._outs = [arr(*[b + h * self._half + part_bytes + count_bytes for b in bases])
                      for h in (0, 1)] if self._gather else None
        self.calls = 0
        self._uses = [0, 0]
        self._failed = False

    @staticmethod
    def _check_shape(rows: int, cols: int, world: int) -> None:
        if rows % (256 * world):
            raise ValueError(f"rows ({rows}) must be a multiple of 256 * world ({256 * world})")
        if cols % 16:
            raise ValueError("cols must be a multiple of 16")

    def _check(self, q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
               w_scale: torch.Tensor, bias: torch.Tensor | None) -> tuple[int, int]:
        return _check_operands(q, q_scale, w_q, w_scale, bias, self.rows, self.cols)

    def _next_set(self) -> tuple[int, ctypes.c_void_p]:
        if self._failed:
            raise RuntimeError("an earlier call on these buffers failed on this rank, so its "
                               "call count no longer matches the other ranks'; build new buffers")
        self.calls += 1
        half = self.calls & 1
        self._uses[half] += 1
        return half, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _raise(self, name: str, rc: int) -> None:
        self._failed = True
        raise RuntimeError(f"{name} failed: {self._lib.tm_status_string(rc).decode()}")

    def _after_call(self) -> None:
        if self.check_every and self.calls % self.check_every == 0:
            self.check()

    def check(self) -> None:
        """Synchronise this rank's device and raise ``RuntimeError`` if a wait
        inside one of this library's kernels ran out since the status word was
        last cleared (a peer that never contributed: the rows it should have
        produced hold NaN).  The word is left as it is."""
        # the status word is read by a blocking copy on the legacy stream, which
        # does not wait for work on non-blocking streams: synchronise first
        torch.cuda.synchronize(self.device)
        code = ctypes.c_int(0)
        index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        rc = self._lib.tm_device_status(index, ctypes.byref(code), 0)
        if rc != 0:
            self._raise("tm_device_status", rc)
        if code.value != 0:
            raise RuntimeError(
                f"fused row-parallel reduction on rank {self.rank}: a bounded device wait ran "
                f"out (device status {code.value}); rows without all contributions hold NaN")

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after a device sync)."""
        if getattr(self, "_own", None) is None:
            return
        torch.cuda.synchronize(self.device)
        for ptr in self._opened:
            self._lib.tm_peer_close(ctypes.c_void_p(ptr))
        self._opened = []
        self._lib.tm_peer_free(ctypes.c_void_p(self._own))
        self._own = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PeerReduceScatter(_PeerBuffers):
    """Symmetric receive buffers + the fused GEMM/reduce-scatter for one shape."""

    def _check_out(self, out: torch.Tensor) -> None:
        if (tuple(out.shape) != (self.rows_per_owner, self.cols)
                or getattr(out, "dtype", None) != torch.bfloat16 or out.stride(1) != 1):
            raise ValueError(f"out must be bf16 [{self.rows_per_owner}, {self.cols}] "
                             "with contiguous rows")
        _require_cuda(out, "out")

    def __call__(self, q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
                 w_scale: torch.Tensor, bias: torch.Tensor | None, out: torch.Tensor,
                 tile_n: int = 0) -> torch.Tensor:
        """``out[rows/world, cols] = (sum over ranks of this row block of q @ w_q^T) + bias``.

        ``q``: int8 ``[rows, k]`` local activations; ``q_scale``: fp32 per-token
        (or one) scales; ``w_q``: int8 ``[cols, k]`` local weight shard;
        ``w_scale``: fp32 ``[cols]``; ``bias``: bf16 ``[cols]`` or None.
        """
        m, k = self._check(q, q_scale, w_q, w_scale, bias)
        self._check_out(out)
        half, stream = self._next_set()
        rc = self._lib.tm_scaled_mm_i8_reduce_scatter(
            out.data_ptr(), q.data_ptr(), w_q.data_ptr(), q_scale.data_ptr(), q_scale.numel(),
            w_scale.data_ptr(), w_scale.numel(), None if bias is None else bias.data_ptr(),
            m, self.cols, k, q.stride(0), w_q.stride(0), out.stride(0),
            self._part[half], self._counts[half], self.world, self.rank, self._uses[half],
            tile_n, stream)
        if rc != 0:
            self._raise("tm_scaled_mm_i8_reduce_scatter", rc)
        self._after_call()
        return out

    def lora(self, q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
             w_scale: torch.Tensor, bias: torch.Tensor | None, lora_t: torch.Tensor,
             lora_b: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """The row-parallel LoRA linear with its reduce-scatter fused
        (lora_checkpoint.py:127-143, fused-row-reduce branch): each rank's
        ``round(round(q @ w_q^T) + lora_t @ lora_b^T)`` partial goes to the row
        owners, which sum in rank order and add ``bias`` once.  ``lora_t`` bf16
        ``[rows, r]`` (this rank's ``x_local A_local^T``), ``lora_b`` bf16
        ``[cols, r]`` carrying the adapter scale."""
        m, k = self._check(q, q_scale, w_q, w_scale, bias)
        self._check_out(out)
        r = _check_lora(lora_t, lora_b, m, self.cols)
        half, stream = self._next_set()
        rc = self._lib.tm_scaled_mm_i8_lora_reduce_scatter(
            out.data_ptr(), q.data_ptr(), w_q.data_ptr(), q_scale.data_ptr(), q_scale.numel(),
            w_scale.data_ptr(), w_scale.numel(), None if bias is None else bias.data_ptr(),
            lora_t.data_ptr(), lora_t.stride(0), lora_b.data_ptr(), lora_b.stride(0), r,
            m, self.cols, k, q.stride(0), w_q.stride(0), out.stride(0),
            self._part[half], self._counts[half], self.world, self.rank, self._uses[half], stream)
        if rc != 0:
            self._raise("tm_scaled_mm_i8_lora_reduce_scatter", rc)
        self._after_call()
        return out


class PeerAllReduce(_PeerBuffers):
    """Symmetric buffers + the fused GEMM/all-reduce for one shape.

    The result lives in this object's output buffers (two, alternating by
    call): a call's output stays valid until the second call after it.
    """

    _gather = True

    def __init__(self, ctx: ParallelContext, rows: int, cols: int, device: torch.device,
                 *, check_every: int = 0):
        super().__init__(ctx, rows, cols, device, check_every=check_every)
        # tensor views over this rank's own output of each set (the memory
        # belongs to this object and is freed by close())
        self._views = [_wrap_bf16(self._outs[h][self.rank], self.rows, self.cols, device)
                       for h in (0, 1)]

    def __call__(self, q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
                 w_scale: torch.Tensor, bias: torch.Tensor | None,
                 tile_n: int = 0) -> torch.Tensor:
        """``[rows, cols] = (sum over ranks of q @ w_q^T) + bias`` on every rank."""
        m, k = self._check(q, q_scale, w_q, w_scale, bias)
        half, stream = self._next_set()
        rc = self._lib.tm_scaled_mm_i8_all_reduce(
            q.data_ptr(), w_q.data_ptr(), q_scale.data_ptr(), q_scale.numel(),
            w_scale.data_ptr(), w_scale.numel(), None if bias is None else bias.data_ptr(),
            m, self.cols, k, q.stride(0), w_q.stride(0), self._part[half], self._counts[half],
            self._outs[half], self.world, self.rank, self._uses[half], tile_n, stream)
        if rc != 0:
            self._raise("tm_scaled_mm_i8_all_reduce", rc)
        self._after_call()
        return self._views[half]

    def lora(self, q: torch.Tensor, q_scale: torch.Tensor, w_q: torch.Tensor,
             w_scale: torch.Tensor, bias: torch.Tensor | None, lora_t: torch.Tensor,
             lora_b: torch.Tensor) -> torch.Tensor:
        """The row-parallel LoRA linear with its all-reduce fused: as
        :meth:`PeerReduceScatter.lora`, then every owner's reduced rows reach
        every rank; returns ``[rows, cols]`` (valid until the second call
        after this one)."""
        m, k = self._check(q, q_scale, w_q, w_scale, bias)
        r = _check_lora(lora_t, lora_b, m, self.cols)
        half, stream = self._next_set()
        rc = self._lib.tm_scaled_mm_i8_lora_all_reduce(
            q.data_ptr(), w_q.data_ptr(), q_scale.data_ptr(), q_scale.numel(),
            w_scale.data_ptr(), w_scale.numel(), None if bias is None else bias.data_ptr(),
            lora_t.data_ptr(), lora_t.stride(0), lora_b.data_ptr(), lora_b.stride(0), r,
            m, self.cols, k, q.stride(0), w_q.stride(0), self._part[half], self._counts[half],
            self._outs[half], self.world, self.rank, self._uses[half], stream)
        if rc != 0:
            self._raise("tm_scaled_mm_i8_lora_all_reduce", rc)
        self._after_call()
        return self._views[half]
