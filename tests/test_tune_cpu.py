"""Tuner pipeline on CPU: aegis_tune's JSONL -> perf DB -> winners -> header.

Mirrors the reference's aegis-perf tests of the same steps
(rust/aegis-perf/src/tune.rs:430-495: the tie rule, the header's rows and
comments): a synthetic tuning run is ingested, winners are picked with the
paired tie rule, the header is emitted and compiled against
include/aegis/matmul.h. The tuner binary itself needs a GPU; here only its
argument handling runs.
"""
import json
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "aegis-core_b200", "tune"))
import aegis_perf as ap  # noqa: E402


def run_rows(run_id="tune-1", started="2026-12-01T10:00:00Z"):
    return [{"kind": "run", "run_id": run_id, "device": "NVIDIA B200", "sm_arch": 100, "sms": 148,
             "cuda_ver": 12090, "driver_ver": 13000, "started_at": started, "seed": 7, "data_seed": 42,
             "dtype": "bf16", "protocol_version": 2}]


def meas(run_id, impl, m, n, k, med, p10=None, p90=None, dtype="bf16"):
    return {"kind": "measurement", "run_id": run_id, "op": "gemm", "dtype": dtype, "m": m, "n": n, "k": k,
            "impl": impl, "config": {"family": impl.split("_")[0]}, "median_us": med,
            "p10_us": p10 if p10 is not None else med * 0.99, "p90_us": p90 if p90 is not None else med * 1.01,
            "tflops": 2.0 * m * n * k / (med * 1e6), "gbps": 1.0, "reps": 20, "batch_n": 4, "buffer_sets": 2,
            "cache_mode": "cold", "protocol_version": 2, "checked": impl != "cublas", "pass": True,
            "max_abs_err": 0.0}


def paired(run_id, a, b, role, m, n, k, lo, hi, dtype="bf16"):
    return {"kind": "paired", "run_id": run_id, "op": "gemm", "dtype": dtype, "m": m, "n": n, "k": k,
            "a_impl": a, "b_impl": b, "role": role, "pairs": 30, "ratio_median": (lo + hi) / 2,
            "ratio_ci_lo": lo, "ratio_ci_hi": hi, "tied": lo <= 1.0 <= hi, "bootstrap_resamples": 2000,
            "bootstrap_seed": 1, "protocol_version": 2, "cache_mode": "cold"}


def write(tmp_path, name, rows):
    p = tmp_path / name
    p.write_text("".join(json.dumps(r) + "\n" for r in rows))
    return str(p)


@pytest.fixture
def db(tmp_path):
    con = ap.connect(str(tmp_path / "perf.db"))
    yield con
    con.close()


def winner(con, bucket, dtype="bf16"):
    return con.execute("SELECT k.impl, w.tied, w.tie_method, w.pick_reason, w.pct_of_cublas FROM winners w JOIN "
                       "kernels k USING (kernel_id) WHERE w.shape_bucket = ? AND w.dtype = ?",
                       (bucket, dtype)).fetchone()


def test_ingest_pick_and_clear_winner(tmp_path, db):
    rows = run_rows() + [
        meas("tune-1", "cublas", 8192, 8192, 8192, 700.0),
        meas("tune-1", "umma_256x256x64_s7_c2", 8192, 8192, 8192, 760.0),
        meas("tune-1", "umma_128x256x64_s4", 8192, 8192, 8192, 830.0),
        paired("tune-1", "umma_256x256x64_s7_c2", "umma_128x256x64_s4", "runner_up", 8192, 8192, 8192, 1.08, 1.10),
        paired("tune-1", "umma_256x256x64_s7_c2", "cublas", "cublas", 8192, 8192, 8192, 0.91, 0.93),
    ]
    assert ap.ingest(db, write(tmp_path, "r.jsonl", rows)) == (3, 2)
    assert ap.pick(db, 100) == 1
    impl, tied, method, reason, pct = winner(db, "8192x8192x8192")
    assert (impl, tied, method, reason) == ("umma_256x256x64_s7_c2", 0, "paired", "fastest")
    assert pct == pytest.approx(700.0 / 760.0 * 100)


def test_cublaslt_best_is_a_baseline_not_a_winner(tmp_path, db):
    """A faster cublaslt_best row never becomes the winner; the winner records
    its percent of cublaslt_best and the paired CI (reference schema.sql:63-68)."""
    rows = run_rows() + [
        meas("tune-1", "cublas", 4096, 4096, 4096, 100.0),
        meas("tune-1", "cublaslt_best", 4096, 4096, 4096, 90.0),
        meas("tune-1", "umma_256x256x64_s7_c2", 4096, 4096, 4096, 95.0),
        paired("tune-1", "umma_256x256x64_s7_c2", "cublaslt#2", "cublaslt_best", 4096, 4096, 4096, 0.93, 0.96),
    ]
    ap.ingest(db, write(tmp_path, "r.jsonl", rows))
    assert ap.pick(db, 100) == 1
    impl, _, _, _, pct = winner(db, "4096x4096x4096")
    assert impl == "umma_256x256x64_s7_c2" and pct == pytest.approx(100.0 / 95.0 * 100)
    lt, lo, hi = db.execute("SELECT pct_of_cublaslt_best, lt_ratio_ci_lo, lt_ratio_ci_hi FROM winners").fetchone()
    assert lt == pytest.approx(90.0 / 95.0 * 100) and (lo, hi) == (0.93, 0.96)
    text, _ = ap.header_text(db, 100, "x")
    assert "94.7% of cublaslt_best" in text


def test_tie_keeps_the_incumbent_and_ci_swap(tmp_path, db):
    # Run 1: A wins clearly.
    r1 = run_rows("tune-1", "2026-12-01T10:00:00Z") + [
        meas("tune-1", "A", 1, 4096, 4096, 10.0), meas("tune-1", "B", 1, 4096, 4096, 12.0),
        paired("tune-1", "A", "B", "runner_up", 1, 4096, 4096, 1.15, 1.25)]
    ap.ingest(db, write(tmp_path, "r1.jsonl", r1))
    ap.pick(db, 100)
    assert winner(db, "1x4096x4096")[0] == "A"
    # Run 2 (later): B is fastest by median but the paired CI contains 1 -> tie, incumbent A stays.
    r2 = run_rows("tune-2", "2026-12-02T10:00:00Z") + [
        meas("tune-2", "B", 1, 4096, 4096, 9.9), meas("tune-2", "A", 1, 4096, 4096, 10.0),
        paired("tune-2", "B", "A", "runner_up", 1, 4096, 4096, 0.99, 1.03)]
    ap.ingest(db, write(tmp_path, "r2.jsonl", r2))
    ap.pick(db, 100)
    impl, tied, method, reason, _ = winner(db, "1x4096x4096")
    assert (impl, tied, method) == ("A", 1, "paired") and "incumbent A kept" in reason
    # Run 3: the runner-up's CI lies below 1 -> it is confirmed faster and takes the shape.
    r3 = run_rows("tune-3", "2026-12-03T10:00:00Z") + [
        meas("tune-3", "A", 1, 4096, 4096, 10.0), meas("tune-3", "B", 1, 4096, 4096, 10.05),
        paired("tune-3", "A", "B", "runner_up", 1, 4096, 4096, 0.95, 0.98)]
    ap.ingest(db, write(tmp_path, "r3.jsonl", r3))
    ap.pick(db, 100)
    impl, tied, method, _, _ = winner(db, "1x4096x4096")
    assert (impl, tied, method) == ("B", 0, "paired_swap")


def test_band_tie_without_a_paired_test(tmp_path, db):
    rows = run_rows() + [meas("tune-1", "A", 4, 4096, 4096, 10.0, 9.8, 10.4),
                         meas("tune-1", "B", 4, 4096, 4096, 10.3)]
    ap.ingest(db, write(tmp_path, "r.jsonl", rows))
    ap.pick(db, 100)
    impl, tied, method, reason, pct = winner(db, "4x4096x4096")
    assert (impl, tied, method, reason, pct) == ("A", 1, "band", "fastest (tie)", 0.0)


def test_failed_checks_never_win(tmp_path, db):
    bad = meas("tune-1", "A", 2, 64, 64, 1.0)
    bad["pass"] = False
    rows = run_rows() + [bad, meas("tune-1", "B", 2, 64, 64, 2.0)]
    ap.ingest(db, write(tmp_path, "r.jsonl", rows))
    ap.pick(db, 100)
    assert winner(db, "2x64x64")[0] == "B"


def test_header_rows_sorted_and_compile(tmp_path, db):
    rows = run_rows() + [
        meas("tune-1", "cublas", 4096, 4096, 4096, 100.0), meas("tune-1", "umma_256x256x64_s7_c2", 4096, 4096, 4096, 110.0),
        meas("tune-1", "cublas", 1, 4096, 4096, 13.0), meas("tune-1", "gemv_256x256_ksm", 1, 4096, 4096, 10.5),
        meas("tune-1", "cublas", 1, 14336, 4096, 20.0), meas("tune-1", "gemv_256x256_ksm", 1, 14336, 4096, 23.0),
        meas("tune-1", "umma_128x128x64_s6_ksm", 1, 14336, 4096, 40.0),
        paired("tune-1", "gemv_256x256_ksm", "cublas", "cublas", 1, 4096, 4096, 1.21, 1.26),
        # The same shape tuned in f16 too: one row per operand type.
        meas("tune-1", "umma_128x256x64_s4", 4096, 4096, 4096, 120.0, dtype="f16"),
    ]
    ap.ingest(db, write(tmp_path, "r.jsonl", rows))
    ap.pick(db, 100)
    text, n = ap.header_text(db, 100, "test")
    assert n == 4
    body = [ln for ln in text.splitlines() if ln.startswith("    {")]
    # Sorted by (N, K, M, type).
    assert [ln.split(",")[:3] for ln in body] == [["    {1", " 4096", " 4096"], ["    {4096", " 4096", " 4096"],
                                                  ["    {4096", " 4096", " 4096"], ["    {1", " 14336", " 4096"]]
    assert '"umma_256x256x64_s7_c2"' in body[1] and "DType::BF16}" in body[1]
    assert '"umma_128x256x64_s4"' in body[2] and "DType::F16}" in body[2]
    assert "123.8% of cuBLAS (paired CI 121.0-126.0%)" in body[0]  # 13.0 / 10.5 us
    assert "#define AEGIS_WINNERS_SM100 1" in text and "kWinners_sm100a[]" in text
    hdr = tmp_path / "inc" / "aegis" / "winners"
    hdr.mkdir(parents=True)
    (hdr / "sm_100a.h").write_text(text)
    tu = tmp_path / "tu.cpp"
    tu.write_text('#include "aegis/winners/sm_100a.h"\n'
                  "static_assert(sizeof(kWinners_sm100a) / sizeof(kWinners_sm100a[0]) == 4);\n"
                  "static_assert(kWinners_sm100a[0].M == 1 && kWinners_sm100a[3].N == 14336);\n"
                  "static_assert(kWinners_sm100a[2].dtype == aegis::gemm::DType::F16);\n"
                  "int main() { return 0; }\n")
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no g++")
    r = subprocess.run([cxx, "-std=c++20", "-fsyntax-only", f"-I{tmp_path / 'inc'}", f"-I{ROOT}/include",
                        "-I/usr/local/cuda/include", str(tu)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_empty_header_defines_nothing(db):
    text, n = ap.header_text(db, 100, "test")
    assert n == 0 and "AEGIS_WINNERS_SM100" not in text and "#pragma once" in text


def test_table_of_a_run(tmp_path):
    rows = run_rows() + [meas("tune-1", "cublas", 512, 512, 512, 8.0), meas("tune-1", "umma_128x128x64_s6", 512, 512, 512, 10.0)]
    out = ap.table(write(tmp_path, "r.jsonl", rows))
    assert "512x512x512" in out and "umma_128x128x64_s6" in out and "80.0" in out


def test_schema_version_is_checked(tmp_path):
    path = str(tmp_path / "v.db")
    con = ap.connect(path)
    con.execute("UPDATE schema_version SET version = 99")
    con.commit()
    con.close()
    with pytest.raises(SystemExit, match="schema v99"):
        ap.connect(path)


def test_tuner_binary_argument_errors():
    exe = os.path.join(ROOT, "aegis-core_b200", "build", "aegis_tune")
    if not os.path.exists(exe):
        pytest.skip("aegis_tune not built")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "--shapes is required" in r.stderr
    r = subprocess.run([exe, "--shapes", "x", "--dtype", "fp8"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "--dtype is f16 or bf16" in r.stderr


def test_committed_shapes_file_parses():
    path = os.path.join(ROOT, "aegis-core_b200", "tune", "shapes_b200.txt")
    shapes = []
    for line in open(path):
        line = line.split("#")[0].split()
        if line:
            shapes.append(tuple(int(x) for x in line))
    assert (8192, 8192, 8192) in shapes and (1, 4096, 14336) in shapes and (256, 256, 65536) in shapes
    assert all(len(s) == 3 and min(s) > 0 for s in shapes)


def test_committed_header_matches_the_committed_runs(tmp_path):
    """include/aegis/winners/sm_100a.h is what aegis_perf.py makes of the
    committed tuning runs (the rows, not the generation time)."""
    runs = os.path.join(ROOT, "aegis-core_b200", "tune", "runs")
    hdr = os.path.join(ROOT, "include", "aegis", "winners", "sm_100a.h")
    if not os.path.isdir(runs) or not os.path.exists(hdr):
        pytest.skip("no committed runs/header")
    con = ap.connect(str(tmp_path / "perf.db"))
    for f in sorted(os.listdir(runs)):
        if f.endswith(".jsonl"):
            ap.ingest(con, os.path.join(runs, f))
    ap.pick(con, 100)
    text, _ = ap.header_text(con, 100, "x")
    rows = lambda t: [ln for ln in t.splitlines() if ln.startswith("    {")]  # noqa: E731
    assert rows(text) == rows(open(hdr).read())
