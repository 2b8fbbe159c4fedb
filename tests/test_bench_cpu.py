"""bench.py's output contract, on CPU.

The reference arm (the reference's own CPU GEMM on a row sample) runs here
without a GPU: its JSON line carries the metric, config, cpu_baseline and e2e
keys, only rank 0 prints, and warm-up below 3 steps is refused. The clocks
record is parsed from nvidia-smi lines (median SM clock under load, the
throttle reasons that void a run), and the roofline object's denominators and
traffic come from MEASURED_PEAKS.json (or the stated fallback) and the
committed per-kernel traffic summaries."""
import argparse
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402

LINE_KEYS = ["impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
             "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"]


def test_reference_arm_line():
    args = argparse.Namespace(size=512, dtype=None, warmup=1, steps=2)
    line = bench.reference_arm(args, 0, 1)
    assert all(k in line for k in LINE_KEYS), sorted(line)
    assert line["impl"] == "reference" and line["unit"] == "TFLOP/s" and line["value"] > 0
    assert line["higher_is_better"] is True and line["vs_baseline"] is None
    assert line["steps"] == 2 and line["warmup"] == 1 and line["ms_per_step"] > 0
    assert line["config"]["workload"] == "gemm_bf16_512^3_nshard"
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    assert "rows" in cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    json.dumps(line)  # serialisable as is


def test_reference_arm_only_on_rank_0():
    args = argparse.Namespace(size=512, dtype=None, warmup=1, steps=1)
    assert bench.reference_arm(args, 1, 2) is None


def _run(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, "bench.py"] + args, cwd=ROOT, capture_output=True, text=True,
                          timeout=600, env=e)


def test_reference_cli_prints_exactly_one_json_line():
    out = _run(["--impl", "reference", "--size", "512", "--steps", "1", "--warmup", "3"])
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["steps"] == 1 and d["warmup"] == 3


def test_other_ranks_print_nothing():
    out = _run(["--impl", "reference", "--size", "512", "--gpus", "2", "--steps", "1", "--warmup", "3"],
               env={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == ""


def test_warmup_below_three_is_refused():
    out = _run(["--impl", "reference", "--size", "512", "--steps", "1", "--warmup", "2"])
    assert out.returncode != 0 and "warmup" in out.stderr


class _FakeProc:
    def poll(self):
        return 0

    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def _sampler(lines):
    s = bench.ClockSampler(0)
    s.proc = _FakeProc()
    s.lines = list(lines)
    return s.stop()


def _smi(sm, mx=1965, watts=900.0, active="0x4", hw="Not Active", hwt="Not Active", swt="Not Active",
         cap="Active"):
    return f"0, {sm}, {mx}, {watts}, {active}, {hw}, {hwt}, {swt}, {cap}"


def test_clocks_median_under_load_and_power_cap():
    rec = _sampler([_smi(345, watts=120.0, cap="Not Active"), _smi(1320), _smi(1305), _smi(1335)])
    assert rec["sm_mhz"] == 1320 and rec["sm_max_mhz"] == 1965
    assert rec["reasons"] == ["sw_power_cap"] and rec["samples"] == 4
    assert rec["power_w"] == 900.0  # idle samples (below 30% of max clock) left out


def test_clocks_report_the_reasons_that_void_a_run():
    rec = _sampler([_smi(1900, hwt="Active", cap="Not Active"), _smi(1890, hw="Active", cap="Not Active")])
    assert rec["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]


def test_clocks_without_nvidia_smi():
    s = bench.ClockSampler(0)
    assert s.stop()["reasons"] == ["nvidia-smi unavailable"]


def test_clocks_ignore_malformed_lines():
    rec = _sampler(["garbage", "0, [N/A], 1965, 1, 2, 3, 4, 5, 6", _smi(1500, cap="Not Active")])
    assert rec["sm_mhz"] == 1500 and rec["samples"] == 1 and rec["reasons"] == []


def test_peaks_source(tmp_path, monkeypatch):
    peaks, src = bench.measured_peaks()
    assert set(peaks) == set(bench.FALLBACK_PEAKS) and all(v > 0 for v in peaks.values())
    assert src in ("measured", "fallback")
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench.measured_peaks() == (bench.FALLBACK_PEAKS, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6500, "bf16_tflops": 1650,
                                                              "bf16_tflops_sustained": 1390, "extra": 1}))
    assert bench.measured_peaks() == ({"hbm_gbs": 6500.0, "bf16_tflops": 1650.0,
                                       "bf16_tflops_sustained": 1390.0}, "measured")


def test_traffic_comes_from_committed_summaries():
    t = bench.load_traffic("umma_nshard_bf16_16384")
    assert t is not None and 5e9 < t < 5e10  # bytes per 16384^3 launch: between the compulsory 1.6 GB and far beyond
    assert bench.load_traffic("no_such_kernel") is None


@pytest.mark.parametrize("name", sorted(f[:-len(".traffic.json")] for f in os.listdir(os.path.join(ROOT, "profiles"))
                                        if f.endswith(".traffic.json")))
def test_every_traffic_summary_is_readable(name):
    assert bench.load_traffic(name) > 0


def test_cpu_cost_model_predicts_the_whole_problem():
    """cpu_reference_rate's extrapolation (fixed + rows x per-row cost, fitted
    on two row counts of a column block) against one direct call of the
    reference's CPU GEMM on the whole problem. Loose bounds: a shared CPU."""
    import time
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import aegis_capi as ac
    import oracle_py as op
    n = 1536
    cb = bench.cpu_reference_rate(n, samples=2, width=512)
    assert cb["fixed_s"] >= 0 and cb["per_row_s"] > 0 and "fixed" in cb["sample"] and "per row" in cb["sample"]
    g = ac.Generator(0)
    A, B = g.uniform(n * n, "f16"), g.uniform(n * n, "f16")
    d = op.make_desc(n, n, n, dtype="f16")
    t0 = time.perf_counter()
    (op.ref_cpu_reference if cb["kind"] == "reference" else op.gemm_ref)(d, A, B)
    direct = time.perf_counter() - t0
    assert 0.5 * direct < cb["seconds"] < 2.0 * direct, (cb["seconds"], direct)
