#!/usr/bin/env python
"""Benchmark of the W8A8 tensor-parallel DiT linear path on B200.

Workload (the 480p LOW-stage DiT MLP): M = 8192
tokens, d = 3072, ffn = 12288; X bf16 ~N(0,1) with 0.1% outlier channels x20;
weights N(0,0.02) quantised per output channel; one step =
quant(X) -> fc1 (column-parallel, +bias, GELU-tanh fused) -> quant ->
fc2 (row-parallel, +bias) -> reduce-scatter of the fc2 partials over the TP
group.  The TP degree equals the GPU count (strong scaling: the total work
is fixed).  Metric: whole-job int8 TOPS = 2 * (2 M d ffn) / step time.

Timing: W untimed warm-up steps; K timed steps, each bracketed by CUDA events
on the launching stream, with L2 flushed between steps outside the events (a
256 MiB buffer written, then another 256 MiB read, so that no dirty flush
lines are written back inside the next step); barrier + synchronize around the timed region;
the max over ranks is reported.  ``e2e`` repeats the step through the same
public API with the input copied from pinned host memory and the output read
back each step.

``--impl reference`` times the reference algorithm on the host cores (the
CPU oracle: per-token quant, exact int32 GEMM, fp32 epilogue), rank 0 only.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {ours,reference}]
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "W8A8 TP-linear TOPS & % INT8 peak at 1/2/4/8 B200; ms per 768p DiT block"
TOKENS, D, FFN = 8192, 3072, 12288
BLOCK_TOKENS, HEADS, HEAD_DIM = 20480, 24, 128
FLUSH_BYTES = 256 * 1024 * 1024
WORKLOAD = "480p LOW-stage DiT MLP (BASELINE configs[1]): fc1 column-parallel +bias+GELU-tanh, fc2 row-parallel + reduce-scatter"


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true")
    p.add_argument("--reduce", choices=["fused", "nccl"], default="fused",
                   help="fc2 reduce-scatter: fused into the GEMM epilogue over NVLink, or NCCL")
    args = p.parse_args(argv)
    if args.warmup < 3:
        p.error("--warmup must be at least 3")
    if args.steps < 1:
        p.error("--steps must be positive")
    return args


# ----------------------------------------------------------------- peaks
def load_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def ncu_traffic_per_launch(profile: str) -> float | None:
    """DRAM bytes per launch recorded in a committed ncu summary, if present."""
    path = ROOT / "profiles" / profile
    if not path.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", path.read_text())
    return float(m.group(1)) if m else None


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling (200 ms) of SM clocks and throttle reasons."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        time.sleep(0.25)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                try:
                    rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
                except ValueError:
                    continue
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags)
                          if f.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------- distributed
def setup_distributed(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world == 1 and args.gpus > 1:
        raise SystemExit("--gpus N > 1 must be launched with torch.distributed.run (one rank per GPU)")
    return world, rank, local


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        torch.distributed.barrier()


class L2Flush:
    """Empties L2 (126 MB) of anything a timed launch could reuse: writes one
    256 MiB buffer, then reads another.  After the write alone L2 may hold the
    flush's dirty lines, whose write-back to HBM could land inside the next
    timed launch; after the read it holds only clean lines of a buffer no
    timed kernel touches.  ``write_only`` is the write alone (the end-to-end
    loop, whose region holds the flush itself)."""

    def __init__(self, device: torch.device):
        self.dirty = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
        self.clean = torch.ones(FLUSH_BYTES // 4, dtype=torch.float32, device=device)
        self.sink = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self) -> None:
        self.dirty.zero_()
        torch.sum(self.clean, dim=0, out=self.sink)

    def write_only(self) -> None:
        self.dirty.zero_()


# ----------------------------------------------------------------- CPU reference
def cpu_reference_setup(rows: int, seed: int = 0):
    """Oracle operands for ``rows`` tokens of the workload at TP=1."""
    from oracle import w8a8_oracle as orc

    x = orc.activation(rows, D, seed)
    w1q, w1s = orc.quantize_weight(orc.weight(FFN, D, seed + 10))
    w2q, w2s = orc.quantize_weight(orc.weight(D, FFN, seed + 20))
    g = torch.Generator().manual_seed(seed + 1)
    b1 = (torch.randn(FFN, generator=g) * 0.01).to(torch.bfloat16)
    b2 = (torch.randn(D, generator=g) * 0.01).to(torch.bfloat16)
    return x, (w1q, w1s, b1), (w2q, w2s, b2)


def cpu_reference_step(x, fc1, fc2):
    from oracle import w8a8_oracle as orc

    q1, s1 = orc.dynamic_scaled_int8_quant(x)
    h, _ = orc.scaled_mm(q1, fc1[0], s1, fc1[1], fc1[2], torch.bfloat16, gelu=True)
    q2, s2 = orc.dynamic_scaled_int8_quant(h)
    y, _ = orc.scaled_mm(q2, fc2[0], s2, fc2[1], fc2[2], torch.bfloat16)
    return y


def time_cpu_reference(rows: int, min_seconds: float, max_passes: int) -> dict:
    torch.set_num_threads(os.cpu_count() or 1)
    x, fc1, fc2 = cpu_reference_setup(rows)
    cpu_reference_step(x, fc1, fc2)  # warm-up
    times = []
    t_end = time.perf_counter() + min_seconds
    while len(times) < max_passes and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        cpu_reference_step(x, fc1, fc2)
        times.append(time.perf_counter() - t0)
    ops = 2 * 2 * rows * D * FFN
    per = statistics.mean(times)
    return {"value": ops / per / 1e12, "unit": "TOPS", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{rows} of {TOKENS} tokens at TP=1, {len(times)} passes of {per * 1e3:.1f} ms "
                      "(oracle quant + torch._int_mm + fp32 epilogue), TOPS of the sample"}


def time_cpu_bf16_linear(rows: int, min_seconds: float, max_passes: int) -> dict:
    """The repo-side BF16 baseline: ``nn.Linear`` (``F.linear``) for fc1 (+bias,
    GELU-tanh) and fc2 (+bias) of ``rows`` tokens on the host cores."""
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(rows, D, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(FFN, D, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(D, FFN, generator=g) * 0.02).to(torch.bfloat16)
    b1 = (torch.randn(FFN, generator=g) * 0.01).to(torch.bfloat16)
    b2 = (torch.randn(D, generator=g) * 0.01).to(torch.bfloat16)
    F = torch.nn.functional

    def step():
        return F.linear(F.gelu(F.linear(x, w1, b1), approximate="tanh"), w2, b2)

    step()
    times = []
    t_end = time.perf_counter() + min_seconds
    while len(times) < max_passes and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    per = statistics.mean(times)
    flops = 2 * 2 * rows * D * FFN
    return {"value": flops / per / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "bf16 nn.Linear",
            "sample": f"{rows} of {TOKENS} tokens, {len(times)} passes of {per * 1e3:.1f} ms "
                      "(F.linear fc1 + GELU-tanh + F.linear fc2 in bf16)"}


def run_reference(args) -> int:
    """The reference's arithmetic for the path on the host cores, on the same
    workload as our arm: every step quantises all 8192 tokens and runs fc1
    (+bias, GELU) and fc2 (+bias) through the exact int32 GEMM and the fp32
    epilogue.  Should K + W full steps not fit in about four minutes, each
    step takes an equal token sample instead (``config.sample_tokens``)."""
    world, rank, _ = setup_distributed(args)
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    rows = TOKENS
    x, fc1, fc2 = cpu_reference_setup(rows)
    t0 = time.perf_counter()
    cpu_reference_step(x, fc1, fc2)
    first = time.perf_counter() - t0
    budget_s = 240.0
    if first * (args.steps + args.warmup) > budget_s:
        rows = max(128, int(TOKENS * budget_s / (first * (args.steps + args.warmup))) // 128 * 128)
        x, fc1, fc2 = cpu_reference_setup(rows)
    for _ in range(args.warmup - 1):
        cpu_reference_step(x, fc1, fc2)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_reference_step(x, fc1, fc2)
    per = (time.perf_counter() - t0) / args.steps
    ops = 2 * 2 * rows * D * FFN
    value = ops / per / 1e12
    sample = (f"all {TOKENS} tokens per step" if rows == TOKENS else
              f"{rows} of {TOKENS} tokens per step (time bound)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens": TOKENS, "d": D, "ffn": FFN,
                   "parallelism": "tp1 (host cores)", "sample_tokens": rows,
                   "same_config": rows == TOKENS},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{sample} at TP=1 on the host cores (the reference's "
                                   "arithmetic restated in oracle/: per-token quant, exact int32 "
                                   "GEMM, fp32 epilogue; the reference's own int8 GEMM, vLLM "
                                   "cutlass_scaled_mm, has no CPU path and refuses int8 on "
                                   "sm_100)"},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------- our arm
STACK_BLOCKS = 40


def lora_block_stack(ctx, device: torch.device, g: torch.Generator, world: int,
                     flush: L2Flush) -> dict:
    """40 chained 768p blocks (QKV, out-proj, fc1, fc2) with
    the BF16 LoRA (rank 64, alpha 64) in the W8A8 epilogue and adaLN modulate
    fused into the activation quant; each block has its own weights, so every
    block streams its weights from HBM.  One forward of the 40 blocks per
    timed repetition (L2 flushed before it).  At N > 1 the row-parallel
    out-projection and fc2 reductions run both ways, NCCL all-reduce and fused
    into the LoRA GEMM over NVLink; the line's ms_per_block is the faster."""
    from taomate_hd_b200.dit import TPW8A8LoRABlockStack

    x = torch.randn(BLOCK_TOKENS, D, generator=g, device=device).to(torch.bfloat16)
    per_mode = {}
    for fused in ((False, True) if world > 1 else (False,)):
        stack = TPW8A8LoRABlockStack(STACK_BLOCKS, BLOCK_TOKENS, D, HEADS, HEAD_DIM, FFN, ctx,
                                     device, seed=11, fused=fused)
        stack.forward(x)
        torch.cuda.synchronize()
        barrier(world)
        reps = 3
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(reps)]
        for e0, e1 in ev:
            flush()
            e0.record()
            stack.forward(x)
            e1.record()
        torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(sum(e0.elapsed_time(e1) for e0, e1 in ev) / reps, world, device)
        per_mode["fused" if fused else "nccl"] = ms / STACK_BLOCKS
        if fused:
            stack.close()
            barrier(world)
        ops_per_block, lora_flops, launches = (stack.int8_ops_per_block,
                                               stack.lora_flops_per_block,
                                               stack.launches_per_block)
        del stack
        torch.cuda.empty_cache()
    per_block = min(per_mode.values())
    out = {"blocks": STACK_BLOCKS, "ms_per_forward": per_block * STACK_BLOCKS,
           "ms_per_block": per_block, "ms_per_block_by_reduce": per_mode,
           "int8_tops": ops_per_block / (per_block * 1e-3) / 1e12,
           "lora_bf16_tflops": lora_flops / (per_block * 1e-3) / 1e12,
           "config": f"M={BLOCK_TOKENS}, d={D}, heads {HEADS}x{HEAD_DIM}, ffn {FFN}, LoRA rank "
                     "64 alpha 64 in every W8A8 epilogue (down-projection on this package's "
                     "tcgen05 kernel), per-token adaLN modulate fused into the quant, GELU-tanh "
                     "after fc1; row-parallel reduce: "
                     + ("none (TP=1)" if world == 1
                        else "NCCL all-reduce or fused into the LoRA GEMM (the faster)"),
           "gpu_launches_per_block": launches}
    return out


SWEEP_M = (64, 256, 1024, 4096, 16384, 32768)
SWEEP_NK = ((3072, 3072), (12288, 3072))  # (N, K)


def skinny_sweep(world: int, device: torch.device, flush: L2Flush) -> list[dict]:
    """the scaled GEMM over M at two weight shapes.

    Each rank runs the column-parallel shard (N / TP) of its own weight; no
    collective.  Every shape is launched before any is timed.  Two
    measurements per shape:

    * ``us``: each launch timed alone with CUDA events (median of 10).
      Before each, L2 is flushed (``L2Flush``), so the weights come from HBM
      and no dirty flush lines are left for the timed kernel to write back
      (at small M that would dominate).
    * ``stream_us``: 64 launches back to back on one stream, each on its own
      copy of the weight (the copies together exceed twice the L2), timed as
      one region and divided by the launch count: the per-layer time of a
      chain of linears, where one launch's set-up overlaps the previous one.

    ``hbm_gbs`` / ``stream_hbm_gbs`` count the minimum bytes MK + NK + 2MN +
    4M + 4N once per launch.
    """
    from taomate_hd_b200 import ops

    g = torch.Generator(device=device).manual_seed(77)
    rows = []
    reps, chain = 10, 64
    for n_full, k in SWEEP_NK:
        n = n_full // world
        copies = max(2, -(-(2 * 126 * 2 ** 20) // (n * k)))  # > 2 x L2 of weights
        ws = [torch.randint(-127, 128, (n, k), generator=g, device=device, dtype=torch.int8)
              for _ in range(copies)]
        sb = torch.rand(1, n, generator=g, device=device) * 1e-3 + 1e-5
        inputs = {}
        for m in SWEEP_M:
            a = torch.randint(-127, 128, (m, k), generator=g, device=device, dtype=torch.int8)
            sa = torch.rand(m, 1, generator=g, device=device) * 1e-2 + 1e-4
            inputs[m] = (a, sa, torch.empty(m, n, dtype=torch.bfloat16, device=device))
            for _ in range(3):
                ops.scaled_mm(a, ws[0].t(), sa, sb, torch.bfloat16, out=inputs[m][2])
        torch.cuda.synchronize()
        for m in SWEEP_M:
            a, sa, y = inputs[m]
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(reps)]
            for e0, e1 in ev:
                flush()
                e0.record()
                ops.scaled_mm(a, ws[0].t(), sa, sb, torch.bfloat16, out=y)
                e1.record()
            torch.cuda.synchronize()
            us = 1e3 * max_over_ranks(statistics.median(e0.elapsed_time(e1) for e0, e1 in ev),
                                      world, device)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            flush()
            s0.record()
            for i in range(chain):
                ops.scaled_mm(a, ws[i % copies].t(), sa, sb, torch.bfloat16, out=y)
            s1.record()
            torch.cuda.synchronize()
            stream_us = 1e3 * max_over_ranks(s0.elapsed_time(s1) / chain, world, device)
            nbytes = m * k + n * k + 2 * m * n + 4 * m + 4 * n
            rows.append({"m": m, "n": n, "k": k, "tp": world, "us": round(us, 2),
                         "tops_per_gpu": round(2 * m * n * k / (us * 1e-6) / 1e12, 1),
                         "hbm_gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
                         "stream_us": round(stream_us, 2),
                         "stream_hbm_gbs": round(nbytes / (stream_us * 1e-6) / 1e9, 1)})
        del ws, sb, inputs
    return rows


def ulysses_send(device: torch.device, flush: L2Flush) -> list[dict]:
    """768p merged QKV projection per Ulysses rank (tokens / degree rows,
    all heads), written in the all-to-all send layout.

    ``fused_us``: the GEMM whose epilogue stores the send layout directly;
    ``permute_us``: the reference order, the token-major GEMM output then
    the permute copy into ``[degree, 3, tokens, heads / degree, head_dim]``
    (ulysses.py:153-163 of the reference).  Layout only: the exchange itself
    is NCCL's all-to-all in both cases and is not timed here.
    """
    from taomate_hd_b200 import ops
    from taomate_hd_b200.ulysses import qkv_send_buffer

    g = torch.Generator(device=device).manual_seed(78)
    n = 3 * HEADS * HEAD_DIM
    w = torch.randint(-127, 128, (n, D), generator=g, device=device, dtype=torch.int8)
    sw = torch.rand(n, generator=g, device=device) * 1e-3 + 1e-5
    bias = (torch.randn(n, generator=g, device=device) * 0.01).to(torch.bfloat16)
    rows, reps = [], 10
    for degree in (2, 8):
        m = BLOCK_TOKENS // degree
        a = torch.randint(-127, 128, (m, D), generator=g, device=device, dtype=torch.int8)
        sa = torch.rand(m, 1, generator=g, device=device) * 1e-2 + 1e-4

        def fused():
            return qkv_send_buffer(a, sa, w, sw, bias, num_heads=HEADS, head_dim=HEAD_DIM,
                                   world=degree)

        def permuted():
            y = ops.scaled_mm(a, w.t(), sa, sw.reshape(1, -1), torch.bfloat16, bias)
            return y.view(m, 3, degree, HEADS // degree, HEAD_DIM).permute(2, 1, 0, 3, 4) \
                    .contiguous()

        result = {"degree": degree, "tokens": m, "n": n, "k": D}
        for name, fn in (("fused_us", fused), ("permute_us", permuted)):
            for _ in range(3):
                fn()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(reps)]
            for e0, e1 in ev:
                flush()
                e0.record()
                fn()
                e1.record()
            torch.cuda.synchronize()
            result[name] = round(1e3 * sum(e0.elapsed_time(e1) for e0, e1 in ev) / reps, 2)
        rows.append(result)
        del a, sa
    return rows


def ulysses_exchange(ctx, world: int, device: torch.device, flush: L2Flush) -> dict:
    """768p merged QKV projection and its Ulysses all-to-all at degree = N
    (tokens / N rows per rank, all heads): the exchange done by the GEMM's
    epilogue over NVLink (``PeerUlyssesExchange``) against the send-layout
    GEMM followed by NCCL's ``all_to_all_single`` (both return the
    reference's (q, k, v)); median us, L2 flushed, max over ranks."""
    from taomate_hd_b200.ulysses import PeerUlyssesExchange, merged_qkv_sequence_to_heads_w8a8

    g = torch.Generator(device=device).manual_seed(79)
    n, m = 3 * HEADS * HEAD_DIM, BLOCK_TOKENS // world
    w = torch.randint(-127, 128, (n, D), generator=g, device=device, dtype=torch.int8)
    sw = torch.rand(n, generator=g, device=device) * 1e-3 + 1e-5
    bias = (torch.randn(n, generator=g, device=device) * 0.01).to(torch.bfloat16)
    a = torch.randint(-127, 128, (m, D), generator=g, device=device, dtype=torch.int8)
    sa = torch.rand(m, 1, generator=g, device=device) * 1e-2 + 1e-4
    group = ctx.tp_group  # the bench's Ulysses degree is its GPU count
    ex = PeerUlyssesExchange(m, HEADS, HEAD_DIM, device, group=group, world=world,
                             rank=ctx.tp_rank)
    fused = _timed(lambda: ex(a, sa, w, sw, bias), 10, flush, world, device)
    nccl = _timed(lambda: merged_qkv_sequence_to_heads_w8a8(
        a, sa, w, sw, bias, num_heads=HEADS, head_dim=HEAD_DIM, group=group, world=world),
        10, flush, world, device)
    same = all(torch.equal(x.view(torch.int16), y.view(torch.int16)) for x, y in zip(
        ex(a, sa, w, sw, bias), merged_qkv_sequence_to_heads_w8a8(
            a, sa, w, sw, bias, num_heads=HEADS, head_dim=HEAD_DIM, group=group, world=world)))
    ex.check()
    barrier(world)
    ex.close()
    moved = (world - 1) / world * m * n * 2  # bytes each rank sends to its peers
    return {"degree": world, "tokens_per_rank": m, "n": n, "k": D,
            "fused_us": round(1e3 * fused, 1), "send_gemm_plus_nccl_us": round(1e3 * nccl, 1),
            "bytes_leaving_rank": moved, "nvlink_gbs_fused": round(moved / (fused * 1e-3) / 1e9, 1),
            "bit_identical": same}


def _timed(fn, reps: int, flush: L2Flush, world: int, device) -> float:
    """Median device time (ms) of ``fn`` over ``reps`` calls, L2 flushed before
    each, barrier-separated, max over ranks."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        flush()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return max_over_ranks(statistics.median(times), world, device)


def multi_gpu_parity(mlp, world: int, rank: int, device, samples: int = 48) -> dict:
    """One untimed fc2 of the timed step's operands through the reduce-scatter
    path the bench ran (fused or NCCL) and through GEMM + NCCL, both compared
    with the oracle on sampled rows of every owner block.

    Oracle rows: each rank computes its bf16 partial of the sampled rows from
    its own int8 activations and weight shard (exact int32 GEMM, fp32
    epilogue), the ranks all-gather them, and each rank sums its owner rows in
    rank order in fp32 and adds the bias -- the fused kernel's reduction order
    (its bit-exactness is reported).  NCCL's ring rounds the running bf16 sum
    at each hop, so where terms cancel it can be far off in relative terms;
    its bar is the rounding bound: at most world + 2 roundings of 2^-8 (bf16's
    unit roundoff) of the magnitudes involved,
    |y - ref| <= (world + 2) 2^-8 (sum |partial| + |bias| + |ref|).
    """
    from oracle import w8a8_oracle as orc
    from taomate_hd_b200 import ops
    from taomate_hd_b200.collectives import reduce_scatter_rows

    rows = TOKENS // world
    g = torch.Generator().manual_seed(4321)
    idx = torch.cat([j * rows + torch.randperm(rows, generator=g)[:samples].sort().values
                     for j in range(world)])
    q = mlp.q2.q[idx.to(device)].cpu().numpy()
    sa = mlp.q2.s[idx.to(device)].cpu().numpy().reshape(-1)
    partial = orc.scaled_mm(q, mlp.fc2.q.cpu().numpy(), sa, mlp.fc2.scale.cpu().numpy(), None,
                            torch.bfloat16)[0].to(device)
    gathered = [torch.empty_like(partial) for _ in range(world)]
    torch.distributed.all_gather(gathered, partial)
    mine = slice(rank * samples, (rank + 1) * samples)
    ref = torch.zeros(samples, D, dtype=torch.float32, device=device)
    for r in range(world):
        ref += gathered[r][mine].float()
    ref = (ref + mlp.fc2.bias.float()).to(torch.bfloat16)
    mag = torch.zeros(samples, D, dtype=torch.float32, device=device)
    for r in range(world):
        mag += gathered[r][mine].float().abs()
    ring_bound = (world + 2) * 2.0 ** -8 * (mag + mlp.fc2.bias.float().abs() + ref.float().abs())
    local = (idx[mine] - rank * rows).to(device)

    out = torch.empty(rows, D, dtype=torch.bfloat16, device=device)
    if mlp.peer is not None:
        mlp.peer(mlp.q2.q, mlp.q2.s, mlp.fc2.q, mlp.fc2.scale, mlp.fc2.bias, out)
        mlp.peer.check()
        path = "fused"
    else:
        path = "nccl"
    part = ops.scaled_mm(mlp.q2.q, mlp.fc2.q.t(), mlp.q2.s, mlp.fc2.scale.reshape(1, -1),
                         torch.bfloat16, mlp.fc2.bias if rank == 0 else None)
    nccl = reduce_scatter_rows(part, group=torch.distributed.group.WORLD, world_size=world)
    if path == "nccl":
        out = nccl
    torch.cuda.synchronize()

    def compare(y: torch.Tensor, ring: bool) -> dict:
        got = y[local].float()
        d = (got - ref.float()).abs()
        ok = (bool((d <= ring_bound).all()) if ring
              else bool(torch.allclose(got, ref.float(), atol=1e-2, rtol=1e-2)))
        return {"max_abs": float(d.max()),
                "max_rel": float((d / ref.float().abs().clamp_min(1e-2)).max()),
                "bit_exact": bool(torch.equal(y[local].view(torch.int16), ref.view(torch.int16))),
                "within_tol": ok}

    res_path = compare(out, ring=path == "nccl")
    res_nccl = compare(nccl, ring=True)
    flag = torch.tensor([1 if res_path["within_tol"] else 0], dtype=torch.int32, device=device)
    torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN)
    exact = torch.tensor([1 if res_path["bit_exact"] else 0], dtype=torch.int32, device=device)
    torch.distributed.all_reduce(exact, op=torch.distributed.ReduceOp.MIN)
    return {"path": path, "rows_checked_per_rank": samples, "rank0": res_path,
            "nccl_rank0": res_nccl, "ok": bool(flag.item()),
            "bit_exact_all_ranks": bool(exact.item()),
            "tolerance": "fused: atol 1e-2 + rtol 1e-2 vs oracle rows (bit-exactness reported); "
                         "NCCL bf16 ring: (world + 2) * 2^-8 * (sum |partial| + |bias| + |ref|)"}


def reduce_vs_nccl(ctx, world: int, rank: int, device, flush: L2Flush) -> list[dict]:
    """The row-parallel GEMM with its reduction, fused over NVLink against the
    GEMM followed by NCCL, at this GPU count: 480p fc2 with a reduce-scatter
    (8192 x 3072 x 12288 / t) and the 768p out-projection with an all-reduce
    (20480 x 3072 x 3072 / t).  ``local_us`` is the GEMM alone (no reduction);
    ``nvlink_gbs_fused`` counts the bytes that must leave each rank,
    (t - 1) / t x M x N x 2 for the reduce-scatter and twice that for the
    all-reduce."""
    from taomate_hd_b200 import ops
    from taomate_hd_b200.collectives import all_reduce_sum_inplace_, reduce_scatter_rows
    from taomate_hd_b200.dit import row_weight
    from taomate_hd_b200.peer_reduce import PeerAllReduce, PeerReduceScatter

    out_rows = []
    for name, m, n, k, mode in (("fc2_480p_reduce_scatter", TOKENS, D, FFN, "rs"),
                                ("out_proj_768p_all_reduce", BLOCK_TOKENS, D, HEADS * HEAD_DIM,
                                 "ar")):
        kl = k // world
        g = torch.Generator(device=device).manual_seed(99 + rank)
        q = torch.randint(-127, 128, (m, kl), generator=g, device=device, dtype=torch.int8)
        sa = torch.rand(m, 1, generator=g, device=device) * 1e-2 + 1e-4
        w = row_weight(n, k, ctx, 7, device, bias=True)
        partial = torch.empty(m, n, dtype=torch.bfloat16, device=device)
        bias0 = w.bias if rank == 0 else None

        def local():
            ops.scaled_mm(q, w.q_t, sa, w.scale.reshape(1, -1), torch.bfloat16, bias0, out=partial)

        row = {"name": name, "m": m, "n": n, "k_per_rank": kl, "tp": world,
               "local_us": round(1e3 * _timed(local, 10, flush, world, device), 1)}
        if world > 1:
            rs_out = torch.empty(m // world, n, dtype=torch.bfloat16, device=device)
            if mode == "rs":
                peer = PeerReduceScatter(ctx, m, n, device)

                def fused():
                    peer(q, sa, w.q, w.scale, w.bias, rs_out)

                def nccl():
                    local()
                    reduce_scatter_rows(partial, group=ctx.tp_group, world_size=world, out=rs_out)
            else:
                peer = PeerAllReduce(ctx, m, n, device)

                def fused():
                    peer(q, sa, w.q, w.scale, w.bias)

                def nccl():
                    local()
                    all_reduce_sum_inplace_(partial, group=ctx.tp_group, world_size=world)
            fused_ms = _timed(fused, 10, flush, world, device)
            nccl_ms = _timed(nccl, 10, flush, world, device)
            peer.check()
            leave = (world - 1) / world * m * n * 2 * (1 if mode == "rs" else 2)
            row.update(fused_us=round(1e3 * fused_ms, 1), gemm_nccl_us=round(1e3 * nccl_ms, 1),
                       nvlink_gbs_fused=round(leave / (fused_ms * 1e-3) / 1e9, 1),
                       bytes_leaving_rank=int(leave))
            torch.cuda.synchronize()
            barrier(world)
            peer.close()
        out_rows.append(row)
        del q, sa, w, partial
        torch.cuda.empty_cache()
    return out_rows


def library_baselines(device, flush: L2Flush) -> dict:
    """The library bars on this GPU, timed like our kernels: cuBLAS's int8 GEMM
    (``torch._int_mm``, int32 out) alone and followed by the same fp32
    dequant + bias (+ GELU) epilogue in torch, at the fc1 and fc2 shapes, next
    to our GEMM on the same operands; and vLLM's ``scaled_int8_quant`` (the
    reference's own quant op) next to ours at both activation shapes, when
    vLLM's compiled ops load here."""
    from taomate_hd_b200 import ops

    g = torch.Generator(device=device).manual_seed(5)
    out = {}
    for name, m, n, k, gelu in (("fc1_480p", TOKENS, FFN, D, True),
                                ("fc2_480p", TOKENS, D, FFN, False)):
        a = torch.randint(-127, 128, (m, k), generator=g, device=device, dtype=torch.int8)
        b = torch.randint(-127, 128, (n, k), generator=g, device=device, dtype=torch.int8)
        sa = torch.rand(m, 1, generator=g, device=device) * 1e-3
        sb = torch.rand(1, n, generator=g, device=device) * 1e-3
        bias = (torch.randn(n, generator=g, device=device) * 0.01).to(torch.bfloat16)
        y = torch.empty(m, n, dtype=torch.bfloat16, device=device)

        def cublas():
            z = (sa * (sb * torch._int_mm(a, b.t()).float()) + bias.float()).to(torch.bfloat16)
            if gelu:
                z = torch.nn.functional.gelu(z.float(), approximate="tanh").to(torch.bfloat16)
            return z

        def cublas_gemm_only():
            return torch._int_mm(a, b.t())

        def ours():
            ops.scaled_mm(a, b.t(), sa, sb, torch.bfloat16, bias, gelu_tanh=gelu, out=y)

        row = {}
        for label, fn in (("ours_us", ours), ("cublas_int8_plus_torch_epilogue_us", cublas),
                          ("cublas_int8_gemm_only_us", cublas_gemm_only)):
            row[label] = round(1e3 * _timed(fn, 10, flush, 1, device), 1)
        row["ours_tops"] = round(2 * m * n * k / (row["ours_us"] * 1e-6) / 1e12, 1)
        row["cublas_gemm_only_tops"] = round(
            2 * m * n * k / (row["cublas_int8_gemm_only_us"] * 1e-6) / 1e12, 1)
        out[name] = row
        del a, b, sa, sb, bias, y
    try:
        from vllm import _custom_ops as vllm_ops

        vllm_quant = vllm_ops.scaled_int8_quant
    except Exception as exc:  # vLLM's compiled ops may not load
        vllm_quant = None
        out["vllm_quant"] = f"unavailable: {type(exc).__name__}"
    for cols in (D, FFN):
        x = torch.randn(TOKENS, cols, generator=g, device=device).to(torch.bfloat16)
        row = {"rows": TOKENS, "cols": cols,
               "ours_us": round(1e3 * _timed(lambda: ops.scaled_int8_quant(x), 10, flush, 1,
                                             device), 1)}
        if vllm_quant is not None:
            try:
                row["vllm_us"] = round(1e3 * _timed(lambda: vllm_quant(x), 10, flush, 1, device), 1)
            except Exception as exc:
                row["vllm_us"] = f"failed: {type(exc).__name__}"
        nbytes = TOKENS * cols * 3 + TOKENS * 4
        row["ours_gbs"] = round(nbytes / (row["ours_us"] * 1e-6) / 1e9, 1)
        out[f"quant_{TOKENS}x{cols}"] = row
        del x
    return out


def run_ours(args) -> int:
    world, rank, local = setup_distributed(args)
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        torch.distributed.init_process_group(
            "nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    from taomate_hd_b200.dit import TPW8A8BlockChain, TPW8A8MLP
    from taomate_hd_b200.parallel import ParallelContext

    ctx = ParallelContext(tp_world_size=world, tp_rank=rank,
                          tp_group=torch.distributed.group.WORLD if world > 1 else None)
    reduce = "fused_reduce_scatter" if args.reduce == "fused" else "reduce_scatter"
    mlp = TPW8A8MLP(TOKENS, D, FFN, ctx, device, seed=0, reduce=reduce)
    launches = mlp.launches_per_step
    g = torch.Generator(device=device).manual_seed(1234)
    x = torch.randn(TOKENS, D, generator=g, device=device)
    outliers = torch.randperm(D, generator=g, device=device)[: max(1, D // 1000)]
    x[:, outliers] *= 20
    x = x.to(torch.bfloat16)
    flush = L2Flush(device)

    for _ in range(args.warmup):
        mlp.forward(x)
        flush()
    torch.cuda.synchronize()
    barrier(world)

    K = args.steps
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    gemm_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        wall0 = time.perf_counter()
        for i in range(K):
            flush()
            starts[i].record()
            mlp.forward(x, gemm_ev[i])
            ends[i].record()
        torch.cuda.synchronize()
        barrier(world)
        wall = time.perf_counter() - wall0
    clock = clocks.summary()
    step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / K
    fc1_ms = [ev[0].elapsed_time(ev[1]) for ev in gemm_ev]
    fc2_ms = [ev[2].elapsed_time(ev[3]) for ev in gemm_ev]
    gemm_avg = (sum(fc1_ms) + sum(fc2_ms)) / (2 * K)
    fc2_avg = sum(fc2_ms) / K
    step_ms = max_over_ranks(step_ms, world, device)
    gemm_avg = max_over_ranks(gemm_avg, world, device)
    fc2_avg = max_over_ranks(fc2_avg, world, device)
    # where the step's time goes: the events around the four launches (the
    # fused reduce-scatter runs inside fc2's launch; an NCCL reduction comes
    # after it), mean over the timed steps, max over ranks per phase
    phases = {"quant_x": [s.elapsed_time(ev[0]) for s, ev in zip(starts, gemm_ev)],
              "fc1_gelu": fc1_ms,
              "quant_h": [ev[1].elapsed_time(ev[2]) for ev in gemm_ev],
              "fc2": fc2_ms,
              "after_fc2": [ev[3].elapsed_time(e) for ev, e in zip(gemm_ev, ends)]}
    breakdown = {name: round(max_over_ranks(sum(v) / K, world, device), 4)
                 for name, v in phases.items()}
    total_ops = mlp.int8_ops
    value = total_ops / (step_ms * 1e-3) / 1e12

    # e2e: the same step through the public API with this step's input copied in
    # from pinned host memory and its output read back to pinned host memory,
    # every step, inside the timed region.  The copies run on their own streams
    # (host->device on one, device->host on another) into double-buffered device
    # staging, so step i's read-back and step i+1's upload overlap the kernels as
    # in a serving loop; the region spans all K steps and ends when the last
    # read-back has landed.  With N ranks each uploads its 1/N row slice of the
    # input and the ranks all-gather it over NVLink (NCCL) before the forward,
    # so the host link carries the input once per step in total.
    rows_in = TOKENS // world
    x_host = x[rank * rows_in:(rank + 1) * rows_in].cpu().pin_memory()
    out_rows = mlp.out.shape[0] if world > 1 else TOKENS
    x_dev = [torch.empty_like(x) for _ in range(2)]
    x_part = [torch.empty(rows_in, D, dtype=x.dtype, device=device) for _ in range(2)]
    y_dev = [torch.empty(out_rows, D, dtype=torch.bfloat16, device=device) for _ in range(2)]
    y_host = [torch.empty(out_rows, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    main = torch.cuda.current_stream(device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    x_ready = [torch.cuda.Event() for _ in range(2)]
    x_free = [torch.cuda.Event() for _ in range(2)]
    y_ready = [torch.cuda.Event() for _ in range(2)]
    y_free = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i: int) -> None:
        b = i % 2
        with torch.cuda.stream(up):
            up.wait_event(x_free[b])
            (x_part[b] if world > 1 else x_dev[b]).copy_(x_host, non_blocking=True)
            x_ready[b].record(up)
        flush.write_only()
        main.wait_event(x_ready[b])
        if world > 1:
            torch.distributed.all_gather_into_tensor(x_dev[b], x_part[b])
        y = mlp.forward(x_dev[b])
        x_free[b].record(main)
        main.wait_event(y_free[b])
        y_dev[b].copy_(y)
        y_ready[b].record(main)
        with torch.cuda.stream(down):
            down.wait_event(y_ready[b])
            y_host[b].copy_(y_dev[b], non_blocking=True)
            y_free[b].record(down)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(main)
    for i in range(K):
        e2e_step(i)
    main.wait_stream(down)
    e_end.record(main)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end) / K, world, device)

    parity = multi_gpu_parity(mlp, world, rank, device) if world > 1 else None
    mlp_peer = mlp.peer
    extras = {}
    if not args.no_extras:
        del mlp
        torch.cuda.empty_cache()
        # the library bars first, on a GPU in the same state as the timed step
        # (after the long LoRA stack the same GEMM read ~45 % slower)
        libs = library_baselines(device, flush) if world == 1 else None
        xb = torch.randn(BLOCK_TOKENS, D, generator=g, device=device).to(torch.bfloat16)
        chains = {}
        for fused in ((False, True) if world > 1 else (False,)):
            block = TPW8A8BlockChain(BLOCK_TOKENS, D, HEADS, HEAD_DIM, FFN, ctx, device, seed=7,
                                     fused=fused)
            chains["fused" if fused else "nccl"] = _timed(lambda: block.forward(xb),
                                                          max(5, K // 2), flush, world, device)
            block_ops = block.int8_ops
            if fused:
                block.attn.peer_ar.check()
                block.mlp.peer_ar.check()
                barrier(world)
                block.attn.peer_ar.close()
                block.mlp.peer_ar.close()
            del block
            torch.cuda.empty_cache()
        block_ms = min(chains.values())
        lora_stack = lora_block_stack(ctx, device, g, world, flush)
        torch.cuda.empty_cache()
        reductions = reduce_vs_nccl(ctx, world, rank, device, flush)
        sweep = skinny_sweep(world, device, flush)
        ulysses = ulysses_send(device, flush) if world == 1 else None
        ulysses_x = ulysses_exchange(ctx, world, device, flush) if world > 1 else None
        extras = {"ms_per_768p_block_linear_chain": block_ms,
                  "block_768p_tops": block_ops / (block_ms * 1e-3) / 1e12,
                  "block_768p_chain_ms": chains,
                  "block_768p_config": f"M={BLOCK_TOKENS}, d={D}, QKV N={3 * HEADS * HEAD_DIM}, "
                                       f"out-proj, fc1 N={FFN} (+GELU), fc2; all-reduce after "
                                       "each row-parallel linear (fused over NVLink or NCCL; "
                                       "the line's ms is the faster); no LoRA / modulate fusion",
                  "lora_block_stack_768p": lora_stack,
                  "reduce_vs_nccl": reductions,
                  "skinny_sweep": sweep,
                  "ulysses_send_768p": ulysses,
                  "ulysses_exchange_768p": ulysses_x,
                  "library_baselines": libs}

    if rank == 0:
        peaks = load_peaks()
        peak_int8 = 2.0 * peaks["bf16_tflops"]
        per_launch_ops = 2 * TOKENS * D * (FFN // world)
        achieved = per_launch_ops / (gemm_avg * 1e-3) / 1e12
        traffic = ncu_traffic_per_launch("gemm_i8_pair_mlp480p.md") if world == 1 else None
        cpu_base = cpu_bf16 = None
        if world == 1 and not args.no_cpu_baseline:
            cpu_base = time_cpu_reference(rows=512, min_seconds=10.0, max_passes=40)
            cpu_bf16 = time_cpu_bf16_linear(rows=512, min_seconds=5.0, max_passes=20)
        line = {
            "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens": TOKENS, "d": D, "ffn": FFN,
                       "parallelism": f"tp{world}",
                       "reduce": ("none (TP=1)" if world == 1 else
                                  "fused into the fc2 GEMM epilogue (NVLink peer stores)"
                                  if args.reduce == "fused" else "nccl reduce_scatter_tensor"),
                       "l2": "flushed between steps outside the step events (256 MiB written, "
                             "then another 256 MiB read: no dirty flush lines left)"},
            "pct_int8_peak": 100.0 * value / (world * peak_int8),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_int8,
                         "unit": "TOPS", "frac": achieved / peak_int8, "traffic": traffic,
                         "kernel": "gemm_i8_pair_kernel<256,6,bf16> (fc1 and fc2 launches)",
                         "traffic_source": "ncu dram__bytes_read + dram__bytes_write per launch, "
                                           "mean of fc1 and fc2, from the one-GPU capture "
                                           "summarised in profiles/gemm_i8_pair_mlp480p.md "
                                           "(taken at commit d353045)",
                         "peak_source": f"2 x {peaks['source']} bf16 dense "
                                        f"({peaks['bf16_tflops']:.0f} TFLOP/s, MEASURED_PEAKS.json): "
                                        "sm_100 int8 tensor rate is twice bf16",
                         "frac_of_sustained": achieved / (2.0 * peaks["bf16_tflops_sustained"])},
            "clocks": clock,
            "nvlink_roofline": None if world == 1 else {
                "bound": "nvlink", "unit": "GB/s", "peak": 770.0,
                "peak_source": "measured peer copy per direction on this pool",
                "bytes_per_rank": (world - 1) / world * TOKENS * D * 2,
                "achieved": (world - 1) / world * TOKENS * D * 2 / (fc2_avg * 1e-3) / 1e9,
                "frac": (world - 1) / world * TOKENS * D * 2 / (fc2_avg * 1e-3) / 1e9 / 770.0,
                "kernel": "fc2 scatter-mode GEMM + owner reduction (partials leaving each rank)"},
            "e2e": {"value": total_ops / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
                    "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": world * x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": world * y_host[0].numel() * y_host[0].element_size(),
                    "pipelining": "upload and read-back on their own streams, double-buffered; "
                                  "L2 flushed inside the region before each step (256 MiB "
                                  "write); N > 1: each "
                                  "rank uploads its row slice, NCCL all-gather of the input"},
            "gpu_launches": K * launches,
            "step_breakdown_ms": breakdown,
            "wall_s_timed_region": wall,
            "extras": extras,
        }
        if parity is not None:
            line["parity"] = parity
        if cpu_base is not None:
            line["cpu_baseline"] = cpu_base
            line["cpu_baseline_bf16_linear"] = cpu_bf16
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        if mlp_peer is not None:
            mlp_peer.close()
        torch.distributed.destroy_process_group()
    if parity is not None and not parity["ok"]:
        print("parity check failed: the reduced fc2 rows differ from the oracle", file=sys.stderr)
        return 1
    return 0


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
