"""GPU, 2 / 4 / 8 ranks on as many GPUs: the fused row-parallel reduce-scatter
and all-reduce (plain and with the LoRA delta), plus the failure path of
their bounded waits on one GPU.

Each rank holds a K-shard of a row-parallel W8A8 linear (linear.py:259-289
semantics: per-token activation scales and per-channel weight scales over the
local K slice).  ``PeerReduceScatter`` must leave on every rank the sum over
ranks of the bf16 partials for its row block plus the bias;
``PeerAllReduce`` the full sum plus bias on every rank, with a call's output
surviving the next call (alternating output sets).  Both are checked over
several consecutive calls (alternating buffer sets, advancing epochs) at a
small shape and at the BASELINE shapes (480p fc2: 8192 x 3072 x 12288 / t;
768p out-projection: 20480 x 3072 x 3072 / t):

* against the oracle on sampled rows: each rank's bf16 partial of the sampled
  rows comes from the oracle's exact int32 GEMM and fp32 epilogue, the
  partials are summed in fp32 in rank order and the bias is added, the order
  the kernel uses, so the fused result must match bit for bit;
* against NCCL's reduce-scatter / all-reduce of the same partials.  NCCL
  sums bf16 partials with a bf16 rounding after every step, so where terms
  cancel its result can be far from the exact sum in relative terms; the
  check is the rounding bound itself: at most world + 2 roundings, each off
  by at most 2^-8 (bf16's unit roundoff) of the magnitudes involved, i.e.
  |fused - nccl| <= (world + 2) * 2^-8 * (sum of |partial| + |bias| + |fused|).
  |bias| is there because the fused path rounds rank 0's partial before the
  bias is added and NCCL's input after, and the two can nearly cancel.

The ranks run as child processes with NCCL's NVLS off; each world size is
skipped on a box with fewer GPUs.
"""
from __future__ import annotations

import ctypes
import datetime
import multiprocessing as mp
import os
import pickle
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sample_rows(lo: int, hi: int, count: int, seed: int) -> np.ndarray:
    """Rows at the block's edges plus a random sample, sorted."""
    g = torch.Generator().manual_seed(seed)
    edges = [lo, lo + 1, lo + 127, lo + 128, hi - 129, hi - 128, hi - 1]
    rand = (lo + torch.randperm(hi - lo, generator=g)[:count]).numpy()
    return np.unique(np.clip(np.concatenate([np.array(edges), rand]), lo, hi - 1))


def _oracle_rows(orc, x_full: torch.Tensor, w_full: torch.Tensor, bias: torch.Tensor,
                 world: int, rows: np.ndarray) -> torch.Tensor:
    """Reduced bf16 rows of the row-parallel linear: per-rank partials of the
    local K slices, fp32 sum in rank order, then the bias."""
    k = x_full.shape[1]
    kl = k // world
    acc = torch.zeros(len(rows), w_full.shape[0], dtype=torch.float32)
    xs = x_full[torch.from_numpy(rows)]
    for r in range(world):
        wq, ws = orc.quantize_weight(w_full[:, r * kl:(r + 1) * kl])
        acc += orc.w8a8_linear(xs[:, r * kl:(r + 1) * kl].contiguous(), wq, ws).float()
    return (acc + bias.float()).to(torch.bfloat16)


def _rs_cases(world: int) -> list[tuple[int, int, int, int]]:
    # (m, n, k over all ranks, calls)
    return [(512 * world, 768, 256 * world, 4), (8192, 3072, 12288, 3)]


def _ar_cases(world: int) -> list[tuple[int, int, int, int]]:
    return [(512 * world, 768, 256 * world, 4), (20480, 3072, 3072, 3)]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    result = {"rank": rank, "ok": False}
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        torch.distributed.init_process_group(
            "nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=90),
            device_id=device)
        from oracle import w8a8_oracle as orc
        from taomate_hd_b200 import _native, ops
        from taomate_hd_b200.collectives import all_reduce_sum, reduce_scatter_rows
        from taomate_hd_b200.parallel import ParallelContext
        from taomate_hd_b200.peer_reduce import PeerAllReduce, PeerReduceScatter

        group = torch.distributed.group.WORLD
        ctx = ParallelContext(tp_world_size=world, tp_rank=rank, tp_group=group)
        checks = []
        for mode, cases in (("rs", _rs_cases(world)), ("ar", _ar_cases(world))):
            for (m, n, k, calls) in cases:
                kl = k // world
                rows = m // world
                peer = (PeerReduceScatter if mode == "rs" else PeerAllReduce)(ctx, m, n, device)
                out = torch.empty(rows, n, dtype=torch.bfloat16, device=device)
                g = torch.Generator().manual_seed(1000 + m + n)
                bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
                w_full = orc.weight(n, k, seed=m + n + 1)
                wq, ws = ops.quantize_weight_int8(w_full[:, rank * kl:(rank + 1) * kl]
                                                  .contiguous().to(device))
                prev = None
                for call in range(calls):
                    x_full = orc.activation(m, k, seed=call * 7 + m + k)
                    x_local = x_full[:, rank * kl:(rank + 1) * kl].contiguous().to(device)
                    q, s, _ = ops.scaled_int8_quant(x_local)
                    if mode == "rs":
                        y = peer(q, s, wq, ws.reshape(-1), bias.to(device), out)
                    else:
                        y = peer(q, s, wq, ws.reshape(-1), bias.to(device))
                    # NCCL on the same partials (the bias once, from rank 0)
                    partial = ops.scaled_mm(q, wq.t(), s, ws.reshape(1, -1), torch.bfloat16,
                                            bias.to(device) if rank == 0 else None)
                    mag = partial.abs().float()
                    if mode == "rs":
                        nccl = reduce_scatter_rows(partial, group=group, world_size=world)
                        mag_sum = torch.empty(rows, n, dtype=torch.float32, device=device)
                        torch.distributed.reduce_scatter_tensor(mag_sum, mag, group=group)
                    else:
                        nccl = all_reduce_sum(partial, group=group, world_size=world)
                        mag_sum = mag
                        torch.distributed.all_reduce(mag_sum, group=group)
                    torch.cuda.synchronize()
                    lo, hi = (rank * rows, (rank + 1) * rows) if mode == "rs" else (0, m)
                    idx = _sample_rows(lo, hi, 96, seed=call + m)
                    ref = _oracle_rows(orc, x_full, w_full, bias, world, idx)
                    got = y.cpu()[torch.from_numpy(idx - (lo if mode == "rs" else 0))]
                    exact = bool(torch.equal(got.view(torch.int16), ref.view(torch.int16)))
                    err = float((got.float() - ref.float()).abs().max())
                    yf = y.float()
                    bound = (world + 2) * 2.0 ** -8 * (mag_sum + bias.to(device).float().abs()
                                                       + yf.abs())
                    excess = (yf - nccl.float()).abs() / bound.clamp_min(1e-30)
                    nccl_close = bool((excess <= 1.0).all())
                    nccl_excess = float(excess.max())
                    kept = True
                    if mode == "ar" and prev is not None:
                        kept = bool(torch.equal(prev[0].cpu(), prev[1]))
                    if mode == "ar":
                        prev = (y, y.cpu().clone())
                    checks.append((mode, m, n, k, call, exact, err, nccl_close, nccl_excess, kept))
                peer.check()
                peer.close()
        # Row-parallel LoRA linears with the fused reduction
        # (lora_checkpoint.py:127-143): every rank's partial is the LoRA GEMM's
        # own epilogue output (no bias); the owners sum them in rank order in
        # fp32 and add the bias once, so the result equals the gathered
        # partials summed that way, bit for bit.
        m, n, kl, r_lora = 512 * world, 768, 256, 64
        g = torch.Generator(device=device).manual_seed(70 + rank)
        q = torch.randint(-127, 128, (m, kl), generator=g, device=device, dtype=torch.int8)
        wq = torch.randint(-127, 128, (n, kl), generator=g, device=device, dtype=torch.int8)
        sq = torch.rand(m, 1, generator=g, device=device) * 1e-2
        sw = torch.rand(n, generator=g, device=device) * 1e-3
        t_l = torch.randn(m, r_lora, generator=g, device=device).to(torch.bfloat16)
        b_l = (torch.randn(n, r_lora, generator=g, device=device) * 0.02).to(torch.bfloat16)
        bias = (torch.randn(n, generator=torch.Generator(device=device).manual_seed(71),
                            device=device) * 0.01).to(torch.bfloat16)
        partial = ops.scaled_mm_lora(q, wq.t(), sq, sw.reshape(1, -1), t_l, b_l)
        parts = [torch.empty_like(partial) for _ in range(world)]
        torch.distributed.all_gather(parts, partial, group=group)
        acc = torch.zeros(m, n, dtype=torch.float32, device=device)
        for part in parts:
            acc += part.float()
        want = (acc + bias.float()).to(torch.bfloat16)
        rows = m // world
        for mode in ("lora_ar", "lora_rs"):
            peer = (PeerAllReduce if mode == "lora_ar" else PeerReduceScatter)(ctx, m, n, device)
            out = torch.empty(rows, n, dtype=torch.bfloat16, device=device)
            for call in range(2):
                if mode == "lora_ar":
                    y = peer.lora(q, sq, wq, sw, bias, t_l, b_l)
                    ref = want
                else:
                    y = peer.lora(q, sq, wq, sw, bias, t_l, b_l, out)
                    ref = want[rank * rows:(rank + 1) * rows]
                torch.cuda.synchronize()
                exact = bool(torch.equal(y.view(torch.int16), ref.view(torch.int16)))
                err = float((y.float() - ref.float()).abs().max())
                checks.append((mode, m, n, kl * world, call, exact, err, True, 0.0, True))
            peer.check()
            peer.close()
        # Ulysses exchange of a merged QKV projection: the fused send layout
        # through NCCL's all-to-all equals the reference path (permute the
        # ordinary output, then the same all-to-all)
        from taomate_hd_b200.ulysses import merged_qkv_sequence_to_heads_w8a8

        heads, hd, tokens, d = 8, 128, 256, 512
        g = torch.Generator(device=device).manual_seed(50 + rank)
        qx = torch.randint(-127, 128, (tokens, d), generator=g, device=device, dtype=torch.int8)
        gw = torch.Generator(device=device).manual_seed(60)
        wx = torch.randint(-127, 128, (3 * heads * hd, d), generator=gw, device=device,
                           dtype=torch.int8)
        sx = torch.rand(tokens, 1, generator=g, device=device) * 1e-2
        swx = torch.rand(3 * heads * hd, generator=gw, device=device) * 1e-3
        got = merged_qkv_sequence_to_heads_w8a8(qx, sx, wx, swx, None, num_heads=heads,
                                               head_dim=hd, group=group, world=world)
        plain = ops.scaled_mm(qx, wx.t(), sx, swx.reshape(1, -1), torch.bfloat16)
        send = orc.merged_qkv_send_layout(plain, heads, hd, world)
        recv = torch.empty_like(send)
        torch.distributed.all_to_all_single(recv, send, group=group)
        ref = recv.movedim(0, 1).contiguous().view(3, tokens * world, heads // world, hd)
        torch.cuda.synchronize()
        ulysses_ok = all(torch.equal(a, b) for a, b in zip(got, ref.unbind(0)))
        # the exchange done by the QKV epilogue over NVLink: the same (q, k, v)
        # bit for bit as the NCCL path, over three calls, with 8 heads and with
        # 9 (the last shard padded with a zero head)
        from taomate_hd_b200.ulysses import PeerUlyssesExchange

        for heads_x in (8, 9):
            ex = PeerUlyssesExchange(tokens, heads_x, hd, device, group=group, world=world,
                                     rank=rank)
            for call in range(3):
                gx = torch.Generator(device=device).manual_seed(80 + 10 * call + rank)
                qx2 = torch.randint(-127, 128, (tokens, d), generator=gx, device=device,
                                    dtype=torch.int8)
                gw2 = torch.Generator(device=device).manual_seed(90 + call)
                wx2 = torch.randint(-127, 128, (3 * heads_x * hd, d), generator=gw2,
                                    device=device, dtype=torch.int8)
                sx2 = torch.rand(tokens, 1, generator=gx, device=device) * 1e-2
                swx2 = torch.rand(3 * heads_x * hd, generator=gw2, device=device) * 1e-3
                want = merged_qkv_sequence_to_heads_w8a8(qx2, sx2, wx2, swx2, None,
                                                         num_heads=heads_x, head_dim=hd,
                                                         group=group, world=world)
                got2 = ex(qx2, sx2, wx2, swx2, None)
                torch.cuda.synchronize()
                ulysses_ok = ulysses_ok and all(
                    torch.equal(a.view(torch.int16), b.view(torch.int16))
                    for a, b in zip(got2, want))
            ex.check()
            torch.distributed.barrier()
            ex.close()
        code = ctypes.c_int(-1)
        _native.capi().tm_device_status(rank, ctypes.byref(code), 1)
        result.update(ok=True, checks=checks, device_status=code.value, ulysses_ok=ulysses_ok)
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    except Exception:
        result["error"] = traceback.format_exc()
    Path(out_dir, f"rank{rank}.pkl").write_bytes(pickle.dumps(result))


def _run_world(world: int, tmp_path: Path) -> list[dict]:
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    out = []
    for r in range(world):
        f = tmp_path / f"rank{r}.pkl"
        assert f.exists(), f"rank {r} produced no result"
        out.append(pickle.loads(f.read_bytes()))
    return out


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_row_parallel_reductions(tmp_path, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    for res in _run_world(world, tmp_path):
        r = res["rank"]
        assert res["ok"], res.get("error")
        assert res["device_status"] == 0
        assert res["ulysses_ok"], f"rank {r}: Ulysses exchange differs from the reference path"
        for (mode, m, n, k, call, exact, err, nccl_close, excess, kept) in res["checks"]:
            where = f"{mode} world {world} rank {r} {m}x{n}x{k} call {call}"
            assert exact, f"{where}: differs from the oracle (max abs {err})"
            assert nccl_close, f"{where}: differs from the NCCL path ({excess:.2f} x the bound)"
            assert kept, f"{where}: the previous call's output changed"


def test_bounded_wait_poisons_unreduced_rows(capi, cuda):
    """One GPU, a two-rank buffer set whose second rank never runs: the
    kernel's wait for that source runs out after its limit (about a second),
    the call's own rows come back as NaN instead of a partial sum, the device
    status word reports the timeout, and the context stays usable.  The same
    for the all-reduce, whose gather wait then also poisons the missing
    owner's rows."""
    m, n, k, world = 512, 256, 256, 2
    rows = m // world
    g = torch.Generator(device=cuda).manual_seed(3)
    a = torch.randint(-127, 128, (m, k), generator=g, device=cuda, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, device=cuda, dtype=torch.int8)
    sa = torch.rand(m, generator=g, device=cuda) * 1e-2
    sb = torch.rand(n, generator=g, device=cuda) * 1e-3
    parts = [torch.zeros(world * rows * n, dtype=torch.bfloat16, device=cuda) for _ in range(world)]
    flags = [torch.zeros(2 * world, dtype=torch.int64, device=cuda) for _ in range(world)]
    outs = [torch.zeros(m, n, dtype=torch.bfloat16, device=cuda) for _ in range(world)]
    arr = ctypes.c_void_p * world
    part_p = arr(*[t.data_ptr() for t in parts])
    flag_p = arr(*[t.data_ptr() for t in flags])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = torch.zeros(rows, n, dtype=torch.bfloat16, device=cuda)
    rc = capi.tm_scaled_mm_i8_reduce_scatter(
        out.data_ptr(), a.data_ptr(), b.data_ptr(), sa.data_ptr(), m, sb.data_ptr(), n, None,
        m, n, k, k, k, n, part_p, flag_p, world, 0, 1, 0, stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.isnan(out.float()).all()
    code = ctypes.c_int(-1)
    assert capi.tm_device_status(0, ctypes.byref(code), 1) == 0
    assert code.value == 1  # wait timeout, now cleared
    for t in flags:
        t.zero_()
    rc = capi.tm_scaled_mm_i8_all_reduce(
        a.data_ptr(), b.data_ptr(), sa.data_ptr(), m, sb.data_ptr(), n, None, m, n, k, k, k,
        part_p, flag_p, arr(*[t.data_ptr() for t in outs]), world, 0, 1, 0, stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.isnan(outs[0].float()).all()  # own rows and the missing owner's rows
    assert capi.tm_device_status(0, ctypes.byref(code), 1) == 0
    assert code.value == 1
    # the context is intact: an ordinary GEMM still runs and matches cuBLAS
    acc = torch.empty(m, n, dtype=torch.int32, device=cuda)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    assert capi.tm_scaled_mm_i8_ex(y.data_ptr(), 0, a.data_ptr(), b.data_ptr(), sa.data_ptr(), m,
                                   sb.data_ptr(), n, None, m, n, k, k, k, n, 0, acc.data_ptr(),
                                   stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(acc, torch._int_mm(a, b.t()))
