"""GPU, 2 ranks on 2 GPUs: the fused row-parallel reduce-scatter and all-reduce.

Each rank holds a K-shard of a row-parallel W8A8 linear (linear.py:259-289
semantics: per-token activation scales and per-channel weight scales over the
local K slice).  ``PeerReduceScatter`` must produce, on every rank, the sum
over ranks of the bf16 partials for its row block plus the bias: checked
against the CPU oracle and against the NCCL reduce-scatter path, over several
consecutive calls (alternating buffer sets, advancing epochs).  ``PeerAllReduce``
must leave the full sum (plus bias) on every rank, checked the same way against
the oracle and NCCL's all-reduce; the output of a call must survive the next
call (alternating output sets).  Runs as child
processes with NCCL's NVLS disabled; skipped with fewer than 2 GPUs.
"""
from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import pickle
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    result = {"rank": rank, "ok": False}
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        device = torch.device("cuda", rank)
        torch.distributed.init_process_group(
            "nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
            device_id=device)
        from oracle import w8a8_oracle as orc
        from taomate_hd_b200 import _native, ops
        from taomate_hd_b200.collectives import all_reduce_sum, reduce_scatter_rows
        from taomate_hd_b200.parallel import ParallelContext
        from taomate_hd_b200.peer_reduce import PeerAllReduce, PeerReduceScatter

        group = torch.distributed.group.WORLD
        ctx = ParallelContext(tp_world_size=world, tp_rank=rank, tp_group=group)
        errors = []
        for (m, n, k) in [(512, 768, 1024), (2048, 3072, 2048)]:
            peer = PeerReduceScatter(ctx, m, n, device)
            rows = m // world
            out = torch.empty(rows, n, dtype=torch.bfloat16, device=device)
            g = torch.Generator().manual_seed(1000 + m)
            bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
            w_full = orc.weight(n, k, seed=m + 1)
            for call in range(5):
                x_full = orc.activation(m, k, seed=call * 7 + m)
                kl = k // world
                x_local = x_full[:, rank * kl:(rank + 1) * kl].contiguous()
                w_local = w_full[:, rank * kl:(rank + 1) * kl].contiguous()
                q, s, _ = ops.scaled_int8_quant(x_local.to(device))
                wq, ws = ops.quantize_weight_int8(w_local.to(device))
                peer(q, s, wq, ws.reshape(-1), bias.to(device), out)
                # NCCL path on the same operands
                partial = ops.scaled_mm(q, wq.t(), s, ws.reshape(1, -1), torch.bfloat16)
                nccl = reduce_scatter_rows(partial, group=group, world_size=world)
                torch.cuda.synchronize()
                # oracle: rank-ordered fp32 sum of the bf16 partials, then the bias
                ref = torch.zeros(m, n, dtype=torch.float32)
                for r in range(world):
                    xr = x_full[:, r * kl:(r + 1) * kl]
                    wr_q, wr_s = orc.quantize_weight(w_full[:, r * kl:(r + 1) * kl])
                    ref += orc.w8a8_linear(xr, wr_q, wr_s).float()
                ref = (ref + bias.float()).to(torch.bfloat16)[rank * rows:(rank + 1) * rows]
                got = out.cpu().float()
                err = float((got - ref.float()).abs().max())
                tol = float((1e-2 + 1e-2 * ref.float().abs()).min())
                close = bool(torch.allclose(got, ref.float(), atol=1e-2, rtol=1e-2))
                nccl_close = bool(torch.allclose(got, nccl.cpu().float() + bias.float(), atol=2e-2,
                                                 rtol=2e-2))
                errors.append((m, n, k, call, err, close, nccl_close, tol))
            peer.close()
        ar_errors = []
        for (m, n, k) in [(512, 768, 1024), (2048, 3072, 1536)]:
            peer = PeerAllReduce(ctx, m, n, device)
            g = torch.Generator().manual_seed(2000 + m)
            bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
            w_full = orc.weight(n, k, seed=m + 3)
            kl = k // world
            w_local = w_full[:, rank * kl:(rank + 1) * kl].contiguous()
            wq, ws = ops.quantize_weight_int8(w_local.to(device))
            prev = None
            for call in range(5):
                x_full = orc.activation(m, k, seed=call * 11 + m + 1)
                x_local = x_full[:, rank * kl:(rank + 1) * kl].contiguous()
                q, s, _ = ops.scaled_int8_quant(x_local.to(device))
                y = peer(q, s, wq, ws.reshape(-1), bias.to(device))
                partial = ops.scaled_mm(q, wq.t(), s, ws.reshape(1, -1), torch.bfloat16)
                nccl = all_reduce_sum(partial, group=group, world_size=world)
                torch.cuda.synchronize()
                ref = torch.zeros(m, n, dtype=torch.float32)
                for r in range(world):
                    xr = x_full[:, r * kl:(r + 1) * kl]
                    wr_q, wr_s = orc.quantize_weight(w_full[:, r * kl:(r + 1) * kl])
                    ref += orc.w8a8_linear(xr, wr_q, wr_s).float()
                ref = (ref + bias.float()).to(torch.bfloat16).float()
                got = y.cpu().float()
                err = float((got - ref).abs().max())
                close = bool(torch.allclose(got, ref, atol=1e-2, rtol=1e-2))
                nccl_close = bool(torch.allclose(got, nccl.cpu().float() + bias.float(),
                                                 atol=2e-2, rtol=2e-2))
                # the previous call's output is still intact (alternating sets)
                kept = True if prev is None else bool(torch.equal(prev[0].cpu(), prev[1]))
                prev = (y, y.cpu().clone())
                ar_errors.append((m, n, k, call, err, close, nccl_close, kept))
            peer.close()
        # Ulysses exchange of a merged QKV projection: the fused send layout
        # through NCCL's all-to-all equals the reference path (permute the
        # ordinary output, then the same all-to-all)
        from oracle.w8a8_oracle import merged_qkv_send_layout
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
        send = merged_qkv_send_layout(plain, heads, hd, world)
        recv = torch.empty_like(send)
        torch.distributed.all_to_all_single(recv, send, group=group)
        ref = recv.movedim(0, 1).contiguous().view(3, tokens * world, heads // world, hd)
        torch.cuda.synchronize()
        ulysses_ok = all(torch.equal(a, b) for a, b in zip(got, ref.unbind(0)))
        code = ctypes_status(_native)
        result.update(ok=True, errors=errors, ar_errors=ar_errors, device_status=code,
                      ulysses_ok=ulysses_ok)
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    except Exception:
        result["error"] = traceback.format_exc()
    Path(out_dir, f"rank{rank}.pkl").write_bytes(pickle.dumps(result))


def ctypes_status(native) -> int:
    import ctypes

    code = ctypes.c_int(-1)
    native.capi().tm_device_status(torch.cuda.current_device(), ctypes.byref(code), 1)
    return code.value


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_fused_reduce_scatter_two_ranks(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    for r in range(world):
        f = tmp_path / f"rank{r}.pkl"
        assert f.exists(), f"rank {r} produced no result"
        res = pickle.loads(f.read_bytes())
        assert res["ok"], res.get("error")
        assert res["device_status"] == 0
        for (m, n, k, call, err, close, nccl_close, tol) in res["errors"]:
            assert close, f"rank {r} {m}x{n}x{k} call {call}: max err {err}"
            assert nccl_close, f"rank {r} {m}x{n}x{k} call {call}: differs from the NCCL path"
        assert res["ulysses_ok"], f"rank {r}: Ulysses exchange differs from the reference path"
        for (m, n, k, call, err, close, nccl_close, kept) in res["ar_errors"]:
            assert close, f"all-reduce rank {r} {m}x{n}x{k} call {call}: max err {err}"
            assert nccl_close, f"all-reduce rank {r} {m}x{n}x{k} call {call}: differs from NCCL"
            assert kept, f"all-reduce rank {r} {m}x{n}x{k} call {call}: previous output changed"
