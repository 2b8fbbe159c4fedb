#!/usr/bin/env python
"""aegis_perf: the perf DB and the winners header for sm_100a.

    aegis_perf.py ingest --db perf.db RUN.jsonl [...]     # aegis_tune output
    aegis_perf.py pick --db perf.db [--arch 100]           # winners per shape
    aegis_perf.py emit-header --db perf.db [--arch 100] [--out include/aegis/winners/sm_100a.h]
    aegis_perf.py table RUN.jsonl                          # one run as a text table

The subset of the reference's `aegis-perf` crate (rust/aegis-perf/src/
{db.rs,tune.rs,schema.sql}) that turns tuner runs into dispatch:
  - schema: the runs / kernels / measurements / paired / winners /
    schema_version tables of schema.sql:2-108, with the columns this library
    produces: the winners' percent of cuBLAS and of cublaslt_best and their
    paired CIs (schema.sql:63-68), but no cuBLASLt algorithm columns, since
    nothing here dispatches to a vendor library;
  - the baselines ("cublas", "cublaslt_best") are measured beside the
    kernels and never win;
  - kernel_id = sha1("op|impl|config"), as db.rs keys kernels;
  - winner per (arch, op, dtype, shape): the fastest cold median of the
    shape's latest run. The paired tie test decides ties (tune.rs): the
    runner-up is tied when the 95% CI of runner-up / fastest contains 1.0,
    and replaces the fastest when the whole CI lies below 1.0; with no paired
    row, the runner-up is tied when its median lies inside the fastest's
    p10-p90 band. On a tie the incumbent winner stays if it is in the tie set;
  - the header (tune.rs:295-405): generated, rows sorted by (N, K, M), one
    row per shape, with the paired figures in the comment.
Python's sqlite3 stands in for rusqlite (there is no Rust toolchain here).
"""
from __future__ import annotations

import argparse
import datetime as _dt
import hashlib
import json
import os
import sqlite3
import sys

SCHEMA_VERSION = 2

SCHEMA = """
CREATE TABLE IF NOT EXISTS runs (
  run_id TEXT PRIMARY KEY,
  device_id TEXT NOT NULL,
  sm_arch INTEGER NOT NULL,
  gpu_name TEXT,
  sms INTEGER,
  cuda_ver INTEGER,
  driver_ver INTEGER,
  seed TEXT,
  data_seed INTEGER,
  protocol_version INTEGER,
  started_at TEXT NOT NULL
);
CREATE TABLE IF NOT EXISTS kernels (
  kernel_id TEXT PRIMARY KEY,
  op TEXT NOT NULL,
  impl TEXT NOT NULL,
  config_json TEXT NOT NULL
);
CREATE TABLE IF NOT EXISTS measurements (
  run_id TEXT NOT NULL REFERENCES runs(run_id),
  kernel_id TEXT NOT NULL REFERENCES kernels(kernel_id),
  dtype TEXT NOT NULL,
  m INTEGER, n INTEGER, k INTEGER,
  median_us REAL, p10_us REAL, p90_us REAL,
  tflops REAL, gbps REAL,
  reps INTEGER,
  checked INTEGER, pass INTEGER,
  max_abs_err REAL,
  protocol_version INTEGER NOT NULL DEFAULT 2,
  batch_n INTEGER,
  cache_mode TEXT,
  buffer_sets INTEGER
);
CREATE INDEX IF NOT EXISTS idx_meas_shape ON measurements(m, n, k, dtype);
CREATE TABLE IF NOT EXISTS paired (
  run_id TEXT NOT NULL REFERENCES runs(run_id),
  op TEXT NOT NULL,
  dtype TEXT NOT NULL,
  m INTEGER, n INTEGER, k INTEGER,
  a_impl TEXT NOT NULL,
  b_impl TEXT NOT NULL,
  role TEXT,
  pairs INTEGER,
  ratio_median REAL,
  ratio_ci_lo REAL,
  ratio_ci_hi REAL,
  tied INTEGER,
  bootstrap_resamples INTEGER,
  bootstrap_seed TEXT,
  protocol_version INTEGER,
  cache_mode TEXT
);
CREATE INDEX IF NOT EXISTS idx_paired_shape ON paired(run_id, m, n, k);
CREATE TABLE IF NOT EXISTS winners (
  sm_arch INTEGER NOT NULL,
  op TEXT NOT NULL,
  dtype TEXT NOT NULL,
  shape_bucket TEXT NOT NULL,
  kernel_id TEXT NOT NULL REFERENCES kernels(kernel_id),
  run_id TEXT NOT NULL REFERENCES runs(run_id),
  median_us REAL,
  pct_of_cublas REAL,
  tied INTEGER NOT NULL DEFAULT 0,
  tie_set TEXT,
  pick_reason TEXT,
  protocol_version INTEGER NOT NULL DEFAULT 2,
  tie_method TEXT,
  ratio_ci_lo REAL,
  ratio_ci_hi REAL,
  cublas_ratio_ci_lo REAL,
  cublas_ratio_ci_hi REAL,
  pct_of_cublaslt_best REAL,
  lt_ratio_ci_lo REAL,
  lt_ratio_ci_hi REAL,
  PRIMARY KEY (sm_arch, op, dtype, shape_bucket)
);
CREATE TABLE IF NOT EXISTS schema_version (
  id INTEGER PRIMARY KEY CHECK (id = 1),
  version INTEGER NOT NULL
);
"""


def connect(path: str) -> sqlite3.Connection:
    con = sqlite3.connect(path)
    con.executescript(SCHEMA)
    row = con.execute("SELECT version FROM schema_version WHERE id = 1").fetchone()
    if row is None:
        con.execute("INSERT INTO schema_version (id, version) VALUES (1, ?)", (SCHEMA_VERSION,))
    elif row[0] != SCHEMA_VERSION:
        raise SystemExit(f"DB schema v{row[0]}, this tool expects v{SCHEMA_VERSION}")
    return con


def kernel_id(op: str, impl: str, config: str) -> str:
    return hashlib.sha1(f"{op}|{impl}|{config}".encode()).hexdigest()


def ingest(con: sqlite3.Connection, path: str) -> tuple[int, int]:
    """Add one aegis_tune output file. Returns (measurements, paired) rows."""
    nm = np_ = 0
    runs: dict[str, dict] = {}
    with open(path) as f:
        rows = [json.loads(ln) for ln in f if ln.strip().startswith("{")]
    for r in rows:
        if r.get("kind") == "run":
            runs[r["run_id"]] = r
            con.execute(
                "INSERT OR REPLACE INTO runs (run_id, device_id, sm_arch, gpu_name, sms, cuda_ver, driver_ver, seed, "
                "data_seed, protocol_version, started_at) VALUES (?,?,?,?,?,?,?,?,?,?,?)",
                (r["run_id"], r.get("device", "?"), int(r["sm_arch"]), r.get("device"), r.get("sms"),
                 r.get("cuda_ver"), r.get("driver_ver"), str(r.get("seed")), r.get("data_seed"),
                 r.get("protocol_version", 2), r["started_at"]))
    for r in rows:
        kind = r.get("kind")
        if kind == "measurement":
            if r["run_id"] not in runs and con.execute("SELECT 1 FROM runs WHERE run_id = ?",
                                                       (r["run_id"],)).fetchone() is None:
                raise SystemExit(f"{path}: measurement of unknown run {r['run_id']}")
            cfg = json.dumps(r.get("config", {}), sort_keys=True)
            kid = kernel_id(r["op"], r["impl"], cfg)
            con.execute("INSERT OR IGNORE INTO kernels (kernel_id, op, impl, config_json) VALUES (?,?,?,?)",
                        (kid, r["op"], r["impl"], cfg))
            con.execute(
                "INSERT INTO measurements (run_id, kernel_id, dtype, m, n, k, median_us, p10_us, p90_us, tflops, "
                "gbps, reps, checked, pass, max_abs_err, protocol_version, batch_n, cache_mode, buffer_sets) "
                "VALUES (?,?,?,?,?,?,?,?,?,?,?,?,?,?,?,?,?,?,?)",
                (r["run_id"], kid, r["dtype"], r["m"], r["n"], r["k"], r["median_us"], r["p10_us"], r["p90_us"],
                 r.get("tflops"), r.get("gbps"), r.get("reps"), int(bool(r.get("checked"))),
                 int(bool(r.get("pass", True))), r.get("max_abs_err"), r.get("protocol_version", 2),
                 r.get("batch_n"), r.get("cache_mode"), r.get("buffer_sets")))
            nm += 1
        elif kind == "paired":
            con.execute(
                "INSERT INTO paired (run_id, op, dtype, m, n, k, a_impl, b_impl, role, pairs, ratio_median, "
                "ratio_ci_lo, ratio_ci_hi, tied, bootstrap_resamples, bootstrap_seed, protocol_version, cache_mode) "
                "VALUES (?,?,?,?,?,?,?,?,?,?,?,?,?,?,?,?,?,?)",
                (r["run_id"], r["op"], r["dtype"], r["m"], r["n"], r["k"], r["a_impl"], r["b_impl"], r["role"],
                 r["pairs"], r["ratio_median"], r["ratio_ci_lo"], r["ratio_ci_hi"], int(bool(r["tied"])),
                 r.get("bootstrap_resamples"), str(r.get("bootstrap_seed")), r.get("protocol_version", 2),
                 r.get("cache_mode")))
            np_ += 1
    con.commit()
    return nm, np_


def _latest_runs(con: sqlite3.Connection, arch: int):
    """(op, dtype, m, n, k) -> the latest run_id with measurements of that shape."""
    q = ("SELECT k.op, m.dtype, m.m, m.n, m.k, m.run_id, r.started_at FROM measurements m "
         "JOIN kernels k USING (kernel_id) JOIN runs r USING (run_id) WHERE r.sm_arch = ? AND m.pass = 1")
    latest: dict[tuple, tuple[str, str]] = {}
    for op, dtype, mm, nn, kk, run, started in con.execute(q, (arch,)):
        key = (op, dtype, mm, nn, kk)
        if key not in latest or started > latest[key][1]:
            latest[key] = (run, started)
    return {k: v[0] for k, v in latest.items()}


def pick(con: sqlite3.Connection, arch: int) -> int:
    """Recompute the winners of every shape from its latest run. Returns rows written."""
    written = 0
    for (op, dtype, mm, nn, kk), run in sorted(_latest_runs(con, arch).items()):
        meas = con.execute(
            "SELECT k.impl, m.kernel_id, m.median_us, m.p10_us, m.p90_us FROM measurements m JOIN kernels k "
            "USING (kernel_id) WHERE m.run_id = ? AND k.op = ? AND m.dtype = ? AND m.m = ? AND m.n = ? AND m.k = ? "
            "AND m.pass = 1 ORDER BY m.median_us", (run, op, dtype, mm, nn, kk)).fetchall()
        ours = [x for x in meas if not x[0].startswith("cublas")]
        base = next((x for x in meas if x[0] == "cublas"), None)
        lt = next((x for x in meas if x[0] == "cublaslt_best"), None)
        if not ours:
            continue
        fastest, runner = ours[0], (ours[1] if len(ours) > 1 else None)
        bucket = f"{mm}x{nn}x{kk}"

        def paired_row(role, a_impl, b_impl=None):
            q = ("SELECT ratio_ci_lo, ratio_ci_hi FROM paired WHERE run_id = ? AND op = ? AND dtype = ? AND m = ? "
                 "AND n = ? AND k = ? AND role = ? AND a_impl = ?")
            args = [run, op, dtype, mm, nn, kk, role, a_impl]
            if b_impl:
                q += " AND b_impl = ?"
                args.append(b_impl)
            return con.execute(q, args).fetchone()

        choice, tied, tie_set, method, ci, reason = fastest, 0, [fastest[0]], None, (None, None), "fastest"
        if runner is not None:
            pr = paired_row("runner_up", fastest[0], runner[0])
            if pr is not None:
                method, ci = "paired", pr
                if pr[0] <= 1.0 <= pr[1]:
                    tied, tie_set = 1, [fastest[0], runner[0]]
                elif pr[1] < 1.0:  # the runner-up is CI-confirmed faster
                    method, choice, reason = "paired_swap", runner, "runner-up CI-confirmed faster"
            elif runner[2] <= fastest[4]:
                method, tied, tie_set = "band", 1, [fastest[0], runner[0]]
        if tied:
            inc = con.execute(
                "SELECT k.impl FROM winners w JOIN kernels k USING (kernel_id) WHERE w.sm_arch = ? AND w.op = ? "
                "AND w.dtype = ? AND w.shape_bucket = ?", (arch, op, dtype, bucket)).fetchone()
            if inc and inc[0] in tie_set and inc[0] != fastest[0]:
                choice = runner if runner[0] == inc[0] else fastest
                reason = f"tie: incumbent {inc[0]} kept"
            else:
                reason = "fastest (tie)"
        pct = base[2] / choice[2] * 100.0 if base else 0.0
        pct_lt = lt[2] / choice[2] * 100.0 if lt else None
        cb = paired_row("cublas", fastest[0])
        lb = paired_row("cublaslt_best", fastest[0])
        mine = choice is fastest
        con.execute(
            "INSERT OR REPLACE INTO winners (sm_arch, op, dtype, shape_bucket, kernel_id, run_id, median_us, "
            "pct_of_cublas, tied, tie_set, pick_reason, protocol_version, tie_method, ratio_ci_lo, ratio_ci_hi, "
            "cublas_ratio_ci_lo, cublas_ratio_ci_hi, pct_of_cublaslt_best, lt_ratio_ci_lo, lt_ratio_ci_hi) "
            "VALUES (?,?,?,?,?,?,?,?,?,?,?,2,?,?,?,?,?,?,?,?)",
            (arch, op, dtype, bucket, choice[1], run, choice[2], pct, tied, json.dumps(tie_set), reason, method,
             ci[0], ci[1], cb[0] if cb and mine else None, cb[1] if cb and mine else None, pct_lt,
             lb[0] if lb and mine else None, lb[1] if lb and mine else None))
        written += 1
    con.commit()
    return written


def header_text(con: sqlite3.Connection, arch: int, generated: str) -> tuple[str, int]:
    """The winners header: one row per (shape, operand type) tuned; dispatch
    prefers the rows of the call's type."""
    rows = con.execute(
        "SELECT w.shape_bucket, w.dtype, k.impl, w.pct_of_cublas, w.tied, w.tie_set, w.pick_reason, w.tie_method, "
        "w.ratio_ci_lo, w.ratio_ci_hi, w.cublas_ratio_ci_lo, w.cublas_ratio_ci_hi, w.median_us, "
        "w.pct_of_cublaslt_best FROM winners w "
        "JOIN kernels k USING (kernel_id) WHERE w.sm_arch = ? AND w.op = 'gemm'", (arch,)).fetchall()
    by_shape: dict[tuple[int, int, int, str], tuple] = {}
    for r in rows:
        m, n, k = (int(x) for x in r[0].split("x"))
        by_shape[(m, n, k, r[1])] = r
    name = f"sm{arch}a" if arch == 100 else f"sm{arch}"
    out = [
        f"// Generated by aegis_perf.py emit-header, {generated}.",
        "// Do not edit. Regenerate on the device after tuning (aegis_tune -> aegis_perf.py ingest, pick, emit-header).",
        f"// Tuned GEMM winners for {name}, read by aegis::matmul (csrc/matmul.cu).",
        "// Row: M, N, K, tuned impl, dispatch (always Aegis: no vendor-library dispatch), kernel % of cuBLAS",
        "// (median ratio of the tuning run), paired 95% CI of cuBLAS time / winner time (0, 0: none),",
        "// operand type the row was tuned on.",
        "// \"[tie test ...]\" in a comment: the paired CI of runner-up / winner time.",
        "#pragma once",
        '#include "aegis/matmul.h"',
        "",
    ]
    if not by_shape:
        out.append(f"// No winners recorded for {name} yet: aegis::matmul uses its built-in rule.")
        return "\n".join(out) + "\n", 0
    define = "AEGIS_WINNERS_SM100" if arch == 100 else f"AEGIS_WINNERS_SM{arch}"
    out += [f"#define {define} 1", f"inline constexpr aegis::detail::Winner kWinners_{name}[] = {{"]
    for (m, n, k, _), r in sorted(by_shape.items(), key=lambda kv: (kv[0][1], kv[0][2], kv[0][0], kv[0][3])):
        (_, dtype, impl, pct, tied, tie_set, reason, method, lo, hi, clo, chi, med, pct_lt) = r
        note = [f"{dtype}, {med:.2f} us"]
        if clo is not None:
            note.append(f"{pct:.1f}% of cuBLAS (paired CI {clo * 100:.1f}-{chi * 100:.1f}%)")
        else:
            note.append(f"{pct:.1f}% of cuBLAS (unpaired)")
        if pct_lt is not None:
            note.append(f"{pct_lt:.1f}% of cublaslt_best")
        if method in ("paired", "paired_swap") and lo is not None:
            note.append(f"[tie test runner-up / winner {lo:.3f}-{hi:.3f}]")
        if tied:
            others = [x for x in json.loads(tie_set or "[]") if x != impl]
            note.append(f"TIED with {', '.join(others)} ({reason})")
        elif reason and reason != "fastest":
            note.append(reason)
        out.append(f'    {{{m}, {n}, {k}, "{impl}", aegis::detail::Dispatch::Aegis, {pct:.1f}, {clo or 0:.4f}, '
                   f'{chi or 0:.4f}, aegis::gemm::DType::{"BF16" if dtype == "bf16" else "F16"}}},  // '
                   + "; ".join(note))
    out.append("};")
    return "\n".join(out) + "\n", len(by_shape)


def table(path: str) -> str:
    rows = [json.loads(ln) for ln in open(path) if ln.strip().startswith("{")]
    meas = [r for r in rows if r.get("kind") == "measurement"]
    shapes = sorted({(r["m"], r["n"], r["k"], r["dtype"]) for r in meas})
    lines = [f"{'shape':>22} {'dtype':>5} {'winner':>28} {'us':>9} {'TFLOP/s':>8} {'GB/s(w)':>8} {'% cuBLAS':>8} "
             f"{'% Lt best':>9}"]
    for m, n, k, d in shapes:
        rs = sorted((r for r in meas if (r["m"], r["n"], r["k"], r["dtype"]) == (m, n, k, d)),
                    key=lambda r: r["median_us"])
        ours = [r for r in rs if not r["impl"].startswith("cublas")]
        cb = next((r for r in rs if r["impl"] == "cublas"), None)
        lt = next((r for r in rs if r["impl"] == "cublaslt_best"), None)
        if not ours:
            continue
        w = ours[0]
        pct = cb["median_us"] / w["median_us"] * 100 if cb else 0.0
        pct_lt = f"{lt['median_us'] / w['median_us'] * 100:9.1f}" if lt else f"{'-':>9}"
        lines.append(f"{f'{m}x{n}x{k}':>22} {d:>5} {w['impl']:>28} {w['median_us']:9.2f} {w['tflops']:8.1f} "
                     f"{w.get('weights_gbps', 0):8.0f} {pct:8.1f} {pct_lt}")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="aegis_perf.py")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("ingest")
    p.add_argument("--db", required=True)
    p.add_argument("files", nargs="+")
    p = sub.add_parser("pick")
    p.add_argument("--db", required=True)
    p.add_argument("--arch", type=int, default=100)
    p = sub.add_parser("emit-header")
    p.add_argument("--db", required=True)
    p.add_argument("--arch", type=int, default=100)
    p.add_argument("--out", default=None)
    p = sub.add_parser("table")
    p.add_argument("file")
    a = ap.parse_args(argv)
    if a.cmd == "table":
        sys.stdout.write(table(a.file))
        return 0
    con = connect(a.db)
    if a.cmd == "ingest":
        for f in a.files:
            nm, np_ = ingest(con, f)
            print(f"{f}: {nm} measurements, {np_} paired tests")
    elif a.cmd == "pick":
        print(f"{pick(con, a.arch)} winners")
    elif a.cmd == "emit-header":
        when = _dt.datetime.now(_dt.timezone.utc).strftime("%Y-%m-%d %H:%M UTC")
        text, n = header_text(con, a.arch, when)
        if a.out:
            os.makedirs(os.path.dirname(os.path.abspath(a.out)), exist_ok=True)
            with open(a.out, "w") as f:
                f.write(text)
            print(f"{a.out}: {n} rows")
        else:
            sys.stdout.write(text)
    return 0


if __name__ == "__main__":
    sys.exit(main())
