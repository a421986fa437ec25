"""bench.py's host-side contract, on the CPU: argument rules, the reference
arm's JSON line (rank 0 only), the clock-record parsing that decides whether a
run is kept, and the committed ncu traffic figure the roofline line carries."""
import io
import json
import contextlib

import pytest
import torch

import bench


def test_parse_args_enforces_warmup_and_steps():
    args = bench.parse_args([])
    assert (args.gpus, args.impl, args.reduce) == (1, "ours", "fused")
    assert args.warmup >= 3 and args.steps >= 1
    with pytest.raises(SystemExit):
        bench.parse_args(["--warmup", "2"])
    with pytest.raises(SystemExit):
        bench.parse_args(["--steps", "0"])


def _run_reference(monkeypatch, argv, env=None):
    # A small workload of the same shape keeps the CPU run to a second or so;
    # the arm reads the sizes at call time.
    monkeypatch.setattr(bench, "TOKENS", 128)
    monkeypatch.setattr(bench, "D", 256)
    monkeypatch.setattr(bench, "FFN", 512)
    for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(key, raising=False)
    for key, value in (env or {}).items():
        monkeypatch.setenv(key, value)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        rc = bench.main(argv)
    return rc, out.getvalue()


def test_reference_arm_prints_one_json_line(monkeypatch):
    rc, text = _run_reference(monkeypatch, ["--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert rc == 0
    lines = [ln for ln in text.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC
    assert line["unit"] == "TOPS" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 1, 3)
    assert line["config"]["workload"] == bench.WORKLOAD
    assert line["config"]["same_config"] is True and line["config"]["sample_tokens"] == 128
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["value"] == line["value"] and cpu["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "TOPS",
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work(monkeypatch):
    rc, text = _run_reference(monkeypatch,
                              ["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3"],
                              env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert rc == 0 and text == ""


def test_reference_arm_refuses_mismatched_world(monkeypatch):
    with pytest.raises(SystemExit):
        _run_reference(monkeypatch, ["--impl", "reference", "--gpus", "4", "--warmup", "3"],
                       env={"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0"})
    with pytest.raises(SystemExit):
        _run_reference(monkeypatch, ["--impl", "reference", "--gpus", "2", "--warmup", "3"])


def _clock_summary(lines):
    sampler = bench.ClockSampler(0)
    sampler.file.write("".join(line + "\n" for line in lines))
    return sampler.summary()


def test_clock_summary_median_and_reasons():
    na = "Not Active"
    rows = [f"0, {mhz}, 1965, 650.1, 0x0, {na}, {na}, {na}, {cap}"
            for mhz, cap in ((1965, na), (1950, "Active"), (1965, na), (1800, "Active"), (1965, na))]
    rows.append("0, [N/A], 1965, 650.1, 0x0, na, na, na, na")  # unparsable sample: skipped
    s = _clock_summary(rows)
    assert s["samples"] == 5
    assert s["sm_mhz"] == 1965 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"]


def test_clock_summary_reports_slowdowns_and_empty_records():
    na = "Not Active"
    s = _clock_summary([f"0, 1200, 1965, 990.0, 0x8, Active, {na}, Active, {na}"])
    assert s["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    assert _clock_summary([]) == {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"],
                                  "samples": 0}


def test_committed_ncu_traffic_figure_is_read():
    traffic = bench.ncu_traffic_per_launch("gemm_i8_pair_mlp480p.md")
    assert traffic is not None and 1e8 < traffic < 1e9
    assert bench.ncu_traffic_per_launch("no_such_profile.md") is None


def test_peaks_have_the_roofline_denominators():
    peaks = bench.load_peaks()
    assert peaks["source"] in ("measured", "fallback")
    assert peaks["hbm_gbs"] > 1000 and peaks["bf16_tflops"] > 500
    assert peaks["bf16_tflops_sustained"] <= peaks["bf16_tflops"] * 1.05


def test_l2_flush_writes_then_reads(monkeypatch):
    monkeypatch.setattr(bench, "FLUSH_BYTES", 1 << 20)
    flush = bench.L2Flush(torch.device("cpu"))
    assert flush.dirty.numel() * flush.dirty.element_size() == 1 << 20
    assert flush.clean.numel() * flush.clean.element_size() == 1 << 20
    flush.dirty.fill_(7)
    flush()
    assert int(flush.dirty.max()) == 0 and float(flush.sink) == flush.clean.numel()
    flush.dirty.fill_(7)
    flush.sink.fill_(-1)
    flush.write_only()
    assert int(flush.dirty.max()) == 0 and float(flush.sink) == -1
