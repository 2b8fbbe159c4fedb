#!/usr/bin/env python
"""Key ncu metrics of profiled kernels, one column per report.

    ncu_summary.py REPORT.ncu-rep [...] [--kernel REGEX] [--flops F] [--bytes B]
                   [--peak-tflops P] [--peak-gbs G] [--traffic-json OUT]
    ncu_summary.py --csv RAW.csv [...]        # the output of `ncu -i R --page raw --csv`

The counterpart of the reference's tools/ncu_summary.sh for sm_100a kernels. Its
rows are the metrics that show a Blackwell kernel's bound:
- tcgen05 tensor-op throughput (per dtype);
- the TMA path (L2 -> SM bytes);
- DRAM bytes, L2 hit rate;
- launch shape and occupancy;
- warp stall reasons.

With --flops or --bytes (algorithmic work per launch) it adds the achieved rate and, with
--peak-tflops / --peak-gbs, its fraction of that peak. --traffic-json writes the per-launch
DRAM bytes in the form bench.py reads from profiles/<name>.traffic.json. The report's
last launch of the kernel (or of the --kernel match) is the one summarised.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import re
import shutil
import subprocess
import sys

METRICS = [
    "gpu__time_duration.sum",
    "sm__cycles_elapsed.avg.per_second",
    "launch__grid_size",
    "launch__block_size",
    "launch__cluster_dim_x",
    "launch__registers_per_thread",
    "launch__shared_mem_per_block_dynamic",
    "launch__occupancy_limit_registers",
    "launch__occupancy_limit_shared_mem",
    "launch__waves_per_multiprocessor",
    "sm__ops_path_tensor_op_utchmma_src_bf16_dst_fp32_sparsity_off.avg.pct_of_peak_sustained_elapsed",
    "sm__ops_path_tensor_op_utchmma_src_fp16_dst_fp32_sparsity_off.avg.pct_of_peak_sustained_elapsed",
    "sm__pipe_tensor_cycles_active_realtime.avg.pct_of_peak_sustained_elapsed",
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "lts__t_sector_hit_rate.pct",
    "l1tex__m_xbar2l1tex_read_bytes.sum",
    "l1tex__m_xbar2l1tex_read_bytes_mem_global_op_tma_ld.sum",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "sm__cycles_active.avg",
    "gpc__cycles_elapsed.max",
    "smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_barrier_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_wait_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_branch_resolving_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_math_pipe_throttle_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_mio_throttle_per_issue_active.ratio",
    "smsp__average_warps_issue_stalled_sleeping_per_issue_active.ratio",
]

_SCALE = {  # unit -> factor to the base unit (seconds, bytes, hertz)
    "ns": 1e-9, "nsecond": 1e-9, "us": 1e-6, "usecond": 1e-6, "ms": 1e-3, "msecond": 1e-3, "s": 1.0, "second": 1.0,
    "byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "Tbyte": 1e12,
    "hz": 1.0, "Khz": 1e3, "Mhz": 1e6, "Ghz": 1e9,
}


def raw_csv(report: str) -> str:
    ncu = shutil.which("ncu") or "/usr/local/cuda/bin/ncu"
    r = subprocess.run([ncu, "--import", report, "--page", "raw", "--csv"], capture_output=True, text=True)
    if r.returncode != 0:
        raise SystemExit(f"ncu --import {report} failed: {r.stderr.strip()[:300]}")
    return r.stdout


def parse(text: str, kernel: str | None = None) -> dict:
    """{metric: (value, unit)} of the last launch (matching `kernel`) in a
    raw-page CSV: row 0 names, row 1 units, then one row per launch."""
    rows = [r for r in csv.reader(io.StringIO(text)) if r]
    start = next((i for i, r in enumerate(rows) if "Kernel Name" in r or "ID" in r[:1]), None)
    if start is None or len(rows) < start + 3:
        raise SystemExit("no profiled launch in the report")
    names, units, launches = rows[start], rows[start + 1], rows[start + 2:]
    ki = names.index("Kernel Name") if "Kernel Name" in names else None
    if kernel and ki is not None:
        launches = [r for r in launches if re.search(kernel, r[ki])]
        if not launches:
            raise SystemExit(f"no launch matches --kernel {kernel}")
    row = launches[-1]
    out = {"Kernel Name": (row[ki] if ki is not None else "?", "")}
    for i, n in enumerate(names):
        if i < len(row):
            out[n] = (row[i], units[i] if i < len(units) else "")
    return out


def number(m: dict, name: str) -> float | None:
    """A metric in base units (s, bytes, Hz, or as given), or None."""
    if name not in m:
        return None
    v, u = m[name]
    try:
        x = float(v.replace(",", ""))
    except ValueError:
        return None
    return x * _SCALE.get(u, 1.0)


def derived(m: dict, flops: float | None, nbytes: float | None, peak_tflops: float | None,
            peak_gbs: float | None) -> list[tuple[str, str]]:
    t = number(m, "gpu__time_duration.sum")
    out = []
    rd, wr = number(m, "dram__bytes_read.sum"), number(m, "dram__bytes_write.sum")
    if rd is not None and wr is not None:
        out.append(("traffic (DRAM read + write per launch)", f"{(rd + wr) / 1e6:.2f} MB"))
        if nbytes:
            out.append(("traffic / algorithmic bytes", f"{(rd + wr) / nbytes:.2f}"))
    if t:
        if flops:
            ach = flops / t / 1e12
            out.append(("achieved TFLOP/s (algorithmic flops / duration)", f"{ach:.1f}"))
            if peak_tflops:
                out.append(("fraction of the TFLOP/s peak", f"{ach / peak_tflops:.3f}"))
        if nbytes:
            ach = nbytes / t / 1e9
            out.append(("achieved GB/s (algorithmic bytes / duration)", f"{ach:.0f}"))
            if peak_gbs:
                out.append(("fraction of the GB/s peak", f"{ach / peak_gbs:.3f}"))
    return out


def table(summaries: list[tuple[str, dict]], extra: list[list[tuple[str, str]]]) -> str:
    head = "| metric | " + " | ".join(name for name, _ in summaries) + " |"
    lines = [head, "|---|" + "---|" * len(summaries)]
    lines.append("| kernel | " + " | ".join(m["Kernel Name"][0][:60] for _, m in summaries) + " |")
    for metric in METRICS:
        cells = []
        for _, m in summaries:
            v, u = m.get(metric, ("-", ""))
            cells.append(f"{v} {u}".strip() if v not in ("", None) else "-")
        if any(c != "-" for c in cells):
            lines.append(f"| `{metric}` | " + " | ".join(cells) + " |")
    labels = []
    for ex in extra:
        for k, _ in ex:
            if k not in labels:
                labels.append(k)
    for k in labels:
        lines.append(f"| {k} | " + " | ".join(dict(ex).get(k, "-") for ex in extra) + " |")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="ncu_summary.py")
    ap.add_argument("reports", nargs="*", help=".ncu-rep files")
    ap.add_argument("--csv", nargs="*", default=[], help="raw-page CSV files instead of reports")
    ap.add_argument("--kernel", default=None, help="regex on the kernel name (default: the last launch)")
    ap.add_argument("--flops", type=float, default=None, help="algorithmic FLOPs per launch")
    ap.add_argument("--bytes", type=float, default=None, help="algorithmic bytes per launch")
    ap.add_argument("--peak-tflops", type=float, default=None)
    ap.add_argument("--peak-gbs", type=float, default=None)
    ap.add_argument("--traffic-json", default=None, help="write DRAM bytes per launch (first report)")
    ap.add_argument("--command", default="", help="the profiled command, recorded in --traffic-json")
    a = ap.parse_args(argv)
    sources = [(os.path.basename(r).removesuffix(".ncu-rep"), raw_csv(r)) for r in a.reports]
    sources += [(os.path.basename(c).removesuffix(".csv"), open(c).read()) for c in a.csv]
    if not sources:
        ap.error("give at least one report or --csv file")
    summaries = [(name, parse(text, a.kernel)) for name, text in sources]
    extra = [derived(m, a.flops, a.bytes, a.peak_tflops, a.peak_gbs) for _, m in summaries]
    sys.stdout.write(table(summaries, extra))
    if a.traffic_json:
        m = summaries[0][1]
        rd, wr = number(m, "dram__bytes_read.sum"), number(m, "dram__bytes_write.sum")
        if rd is None or wr is None:
            raise SystemExit("the report has no dram__bytes_read/write.sum")
        with open(a.traffic_json, "w") as f:
            json.dump({"kernel": m["Kernel Name"][0], "dram_bytes_read": rd, "dram_bytes_write": wr,
                       "dram_bytes_per_launch": rd + wr, "command": a.command}, f, indent=1)
    return 0


if __name__ == "__main__":
    sys.exit(main())
