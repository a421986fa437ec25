"""CPU, world_size 2 over gloo: tensor-parallel semantics of the path.

* Column-parallel W8A8 (QKV / fc1): per-token scales cover the full K and
  weight scales are per output row, so the concatenated rank shards equal the
  unsharded W8A8 linear bit-exactly (linear.py:145-159, w8a8.py:117-145).
* Row-parallel W8A8 (out-proj / fc2): each rank quantises its local K slice
  (activation and weight), and the bf16 partials are summed over the group
  (linear.py:259-289).
* The package's sharding helpers and reductions (all-reduce, reduce-scatter,
  gathered merged-column output, fused LoRA row reduction) on gloo.
* Failure detection on the host: a rank that dies before a collective makes
  the surviving rank's collective fail within the process-group timeout.
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

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 60.0) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group(
        "gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _semantics_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    result = {"rank": rank, "ok": False}
    try:
        _init(rank, world, port)
        from oracle import w8a8_oracle as orc
        from taomate_hd_b200 import collectives, dit

        group = torch.distributed.group.WORLD
        M, K, N = 24, 256, 96
        x = orc.activation(M, K, seed=5)
        w = orc.weight(N, K, seed=6)

        # column-parallel W8A8 == unsharded W8A8 (bit-exact)
        wq_full, ws_full = orc.quantize_weight(w)
        full = orc.w8a8_linear(x, wq_full, ws_full)
        w_local = dit.column_slice(w, world, rank)
        wq, ws = orc.quantize_weight(w_local)
        y_local = orc.w8a8_linear(x, wq, ws)
        gathered = collectives.all_gather_concat(y_local, dim=-1, group=group, world_size=world)
        result["column_exact"] = bool(torch.equal(gathered, full))

        # row-parallel W8A8: local-K quantisation, bf16 partial sum
        w_row = dit.row_slice(w, world, rank)
        x_row = dit.row_slice(x, world, rank)
        wq_r, ws_r = orc.quantize_weight(w_row)
        partial = orc.w8a8_linear(x_row, wq_r, ws_r)
        summed = collectives.all_reduce_sum(partial, group=group, world_size=world)
        expect = None
        for r in range(world):
            qr, sr = orc.quantize_weight(orc.row_shard(w, world, r))
            p = orc.w8a8_linear(orc.row_shard(x, world, r), qr, sr).float()
            expect = p if expect is None else expect + p
        result["row_exact"] = bool(torch.equal(summed, expect.to(torch.bfloat16)))
        # local-K quantisation differs from full-K quantisation (TP-dependent)
        result["row_close_to_full"] = float((summed.float() - full.float()).abs().max())

        # reduce-scatter of rows == slice of the all-reduced sum
        rs = collectives.reduce_scatter_rows(partial, group=group, world_size=world)
        rows = M // world
        result["reduce_scatter_exact"] = bool(torch.equal(rs, summed[rank * rows:(rank + 1) * rows]))

        # gathered merged-column (Q, K, V sharded separately) output equals the
        # per-rank projections of the oracle's shards, in rank order
        torch.manual_seed(0)
        w_full = torch.randn(N, K).to(torch.bfloat16)
        b_full = torch.randn(N).to(torch.bfloat16)
        sizes = (32, 32, 32)
        y_m = collectives.all_gather_concat(
            torch.nn.functional.linear(x, dit.column_slice(w_full, world, rank, sizes)),
            dim=-1, group=group, world_size=world)
        ref_parts = [torch.nn.functional.linear(x, orc.merged_column_shard(w_full, sizes, world, r))
                     for r in range(world)]
        result["merged_gather_exact"] = bool(torch.equal(y_m, torch.cat(ref_parts, dim=-1)))

        # fused LoRA row reduction (lora_checkpoint.py:127-143): one reduce of
        # (base partial + update * scale) on the local K slices, then the bias
        a_full = (torch.randn(4, K) * 0.02).to(torch.bfloat16)
        b_lora = (torch.randn(N, 4) * 0.02).to(torch.bfloat16)
        x_local = dit.row_slice(x, world, rank)
        base_partial = torch.nn.functional.linear(x_local, dit.row_slice(w_full, world, rank))
        lora_partial = orc.lora_column(base_partial, x_local, dit.row_slice(a_full, world, rank),
                                       b_lora, 2.0)
        y_fused = collectives.all_reduce_sum(lora_partial, group=group, world_size=world) + b_full
        y_ref = torch.nn.functional.linear(x.float(), w_full.float(), b_full.float())
        y_lora_ref = y_ref + 2.0 * (x.float() @ a_full.float().t() @ b_lora.float().t())
        scale = y_lora_ref.abs().max()
        result["lora_fused_err"] = float((y_fused.float() - y_lora_ref).abs().max() / scale)
        result["ok"] = True
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    except Exception:
        result["error"] = traceback.format_exc()
    Path(out_dir, f"rank{rank}.pkl").write_bytes(pickle.dumps(result))


def _run(target, world: int, tmp_path: Path, *extra, timeout: float = 180.0) -> list[dict]:
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, str(tmp_path), *extra))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    out = []
    for r in range(world):
        f = tmp_path / f"rank{r}.pkl"
        out.append(pickle.loads(f.read_bytes()) if f.exists() else {"rank": r, "ok": False, "error": "no result"})
    return out


def test_tp_semantics_world2(tmp_path):
    results = _run(_semantics_worker, 2, tmp_path)
    for res in results:
        assert res["ok"], res.get("error")
        assert res["column_exact"]
        assert res["row_exact"]
        assert res["reduce_scatter_exact"]
        assert res["merged_gather_exact"]
        assert res["lora_fused_err"] < 2e-2
        assert 0 < res["row_close_to_full"] < 0.1


def _ulysses_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    """Ulysses exchange of merged QKV send buffers (the oracle's layout, with
    zero-head padding: 3 heads over 2 ranks) through exchange_qkv: rank r
    must receive heads [r L, (r + 1) L) of every rank's tokens, in rank order
    (distributed/ulysses.py:166-212)."""
    result = {"rank": rank, "ok": False}
    try:
        _init(rank, world, port)
        from oracle import w8a8_oracle as orc
        from taomate_hd_b200.ulysses import exchange_qkv

        tokens, heads, head_dim = 5, 3, 4
        local = -(-heads // world)

        def value_of(r):
            g = torch.Generator().manual_seed(90 + r)
            return torch.randn(tokens, 3 * heads * head_dim, generator=g).to(torch.bfloat16)

        send = orc.merged_qkv_send_layout(value_of(rank), heads, head_dim, world)
        got = exchange_qkv(send, group=torch.distributed.group.WORLD)
        padded = [torch.nn.functional.pad(value_of(r).view(tokens, 3, heads, head_dim),
                                          (0, 0, 0, world * local - heads)) for r in range(world)]
        ok = True
        for qkv in range(3):
            want = torch.cat([p[:, qkv, rank * local:(rank + 1) * local] for p in padded])
            ok &= got[qkv].shape == (tokens * world, local, head_dim)
            ok &= torch.equal(got[qkv].view(torch.int16), want.view(torch.int16))
        result.update(ok=True, exchange_exact=bool(ok))
        torch.distributed.destroy_process_group()
    except Exception:
        result["error"] = traceback.format_exc()
    Path(out_dir, f"rank{rank}.pkl").write_bytes(pickle.dumps(result))


def test_ulysses_exchange_world2(tmp_path):
    for res in _run(_ulysses_worker, 2, tmp_path):
        assert res["ok"], res.get("error")
        assert res["exchange_exact"]


def _failure_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    result = {"rank": rank}
    try:
        _init(rank, world, port, timeout_s=10.0)
        if rank == 1:
            # this rank fails on the host before joining the next collective
            result["raised"] = True
            Path(out_dir, f"rank{rank}.pkl").write_bytes(pickle.dumps(result))
            os._exit(3)
        from taomate_hd_b200 import collectives

        value = torch.ones(8)
        try:
            collectives.all_reduce_sum(value, group=torch.distributed.group.WORLD, world_size=world)
            result["collective_error"] = None
        except Exception as exc:  # the dead peer surfaces as an error, not a hang
            result["collective_error"] = type(exc).__name__
    except Exception:
        result["error"] = traceback.format_exc()
    Path(out_dir, f"rank{rank}.pkl").write_bytes(pickle.dumps(result))
    os._exit(0)


def test_dead_rank_fails_collective_instead_of_hanging(tmp_path):
    results = _run(_failure_worker, 2, tmp_path, timeout=90.0)
    assert results[1].get("raised")
    assert results[0].get("collective_error") is not None, results[0]


def test_collectives_require_initialised_group():
    from taomate_hd_b200 import collectives

    x = torch.ones(4)
    assert collectives.all_reduce_sum(x, group=None, world_size=1) is x
    with pytest.raises(RuntimeError):
        collectives.all_reduce_sum(x, group=None, world_size=2)
    with pytest.raises(RuntimeError):
        collectives.reduce_scatter_rows(torch.ones(4, 2), group=None, world_size=2)
    assert np.array_equal(collectives.reduce_scatter_rows(x, group=None, world_size=1).numpy(), x.numpy())
