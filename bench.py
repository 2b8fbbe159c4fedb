#!/usr/bin/env python
"""Benchmark of the aegis-b200 hot path; prints ONE JSON line (rank 0).

Default workload (every N): the 16384^3 bf16 GEMM C = A*B (FP32 accumulate,
bf16 out) with B N-sharded over the N GPUs (column shards) and C
all-gathered by the GEMM itself: aegis_gemm_bf16_nsharded stores every
finished tile into every rank's C (NVLink peer stores), then a one-element
NCCL all-reduce is the cross-rank barrier. At N = 1 it is the plain 16384^3
GEMM. Inputs uniform[-1, 1] from std::mt19937(0) (A then B), larger than L2
(A alone is 512 MiB), so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl aegis|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...

The line carries:
  - value: device-resident throughput (max over ranks of the event-timed K
    steps), roofline of the GEMM kernel against the measured burst bf16 peak
    (the timed region is ~0.1 s, not a power-capped seconds-long loop);
  - e2e: the same GEMM through the C ABI with the inputs copied in from
    pinned host memory and C read back every step, pipelined over two buffer
    sets (copies of step i+1 overlap the GEMM of step i);
  - cublas: torch.matmul (+ NCCL all-gather at N > 1) on the same shapes;
  - at N = 1: cpu_baseline (the reference's own CPU GEMM, throughput
    extrapolated from timed samples, see cpu_reference_rate), a check of
    sampled rows of C against the FP64 oracle, and `workloads`: the square
    8192^3 GEMM (bf16, f16), the decode GEMV (M = 1; K x N = 4096 x 14336 and
    4096 x 4096) and the tall-K split-K GEMM (256 x 256 x 65536), each with
    its roofline fraction and its ratio to cuBLAS and to cublaslt_best.

Single-GPU workloads on their own (`--workload square|gemv|splitk`) print a
line of the same form for one of those shapes.

`--impl reference` times the reference's own CPU GEMM
(aegis::bench::cpu_reference, FP64 accumulate, built from its source into
oracle/_ref; the C restatement oracle/liboracle.so when that is absent) on
samples of the same workload, on rank 0; other ranks exit at once.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "aegis-core_b200"))

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "GEMM TFLOP/s ({dtype} {n}^3, B N-sharded, C all-gathered in the epilogue)"


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["aegis", "reference"], default="aegis")
    p.add_argument("--workload", choices=["nshard", "square", "gemv", "splitk", "gemm"], default="nshard")
    p.add_argument("--size", type=int, default=None, help="square: M=N=K; nshard: M=N=K; splitk: M=N")
    p.add_argument("--k", type=int, default=None, help="gemv/splitk/gemm: K")
    p.add_argument("--n", type=int, default=None, help="gemv/gemm: N")
    p.add_argument("--m", type=int, default=None, help="gemv/gemm: M")
    p.add_argument("--dtype", choices=["bf16", "f16"], default=None)
    p.add_argument("--kernel", default=None, help="force a registry kernel (single-GPU workloads)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-workloads", action="store_true", help="skip the secondary single-GPU shapes at N = 1")
    p.add_argument("--no-lt", action="store_true", help="single-GPU workloads: skip the cublaslt_best sweep")
    a = p.parse_args(argv)
    if a.warmup < 3:
        p.error("--warmup must be >= 3")
    return a


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi samples every 50 ms while the timed region runs. start()
    returns once the first sample has arrived and stop() waits for one more,
    so even a region shorter than the interval is bracketed by samples."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        self._wait_for(1, 5.0)

    def _wait_for(self, n, limit_s):
        t0 = time.time()
        while len(self.lines) < n and time.time() - t0 < limit_s and self.proc.poll() is None:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self._wait_for(len(self.lines) + 1, 2.0)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons, pw = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            try:
                pw.append((float(parts[1]), float(parts[3])))
            except ValueError:
                pass
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        under_load = [s for s in sm if mx and s > 0.3 * mx] or sm
        watts = [w for s, w in pw if mx and s > 0.3 * mx] or [w for _, w in pw]
        return {"sm_mhz": statistics.median(under_load) if under_load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w": statistics.median(watts) if watts else None}


def load_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu summary
    (profiles/<name>.traffic.json), or None."""
    path = os.path.join(ROOT, "profiles", f"{name}.traffic.json")
    try:
        with open(path) as f:
            return float(json.load(f)["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


# ------------------------------------------------------------------ CPU side
CPU_WIDTH = 2048        # columns of B per reference call (a column block of the problem)
CPU_ROWS = (64, 512)    # the two row counts the cost model is fitted on


def cpu_reference_rate(n, samples, width=CPU_WIDTH, rows=CPU_ROWS):
    """Throughput of the reference's own CPU GEMM (aegis::bench::cpu_reference,
    reference src/bench/reference.cu:69-105, built into oracle/_ref; the C
    restatement when that is absent) on the n^3 problem, from timed samples.

    The reference transposes the B columns it is given into doubles on one
    thread (reference.cu:79-83), then splits the rows of C over min(16,
    cores) threads (:77, :99-102). A call on R rows and a block of W columns
    of B therefore costs f + R*r, with f and r both proportional to W (each
    column is transposed once and then dotted once per row; K is the full
    n). Each sample times P such calls at once on disjoint column blocks
    (P = usable cores // threads, so every core works), at R = rows[0] and
    rows[1]; f and r are fitted by least squares over all samples, and the
    full problem's time is the extrapolation
        t = ceil(n / (P * W)) * (f + n * r).
    The reference is f16-only, so the sample is f16 data from the same
    generator (its FP64 arithmetic does not depend on the input type).

    Returns a dict with value (TFLOP/s), seconds, fit, cores, kind, sample."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import aegis_capi as ac
    import oracle_py as op
    width = min(width, n)
    rows = tuple(min(r, n) for r in rows)
    g = ac.Generator(0)
    A = g.uniform(n * n, "f16")
    B = g.uniform(n * n, "f16")
    threads = min(16, os.cpu_count() or 1)
    usable = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    P = max(1, min(n // width, usable // threads))
    kind = "reference" if op.ref_available() else "port"
    span_b = (n - 1) * n + width

    def call(R, p):
        d = op.make_desc(R, width, n, ldb=n, dtype="f16")
        Bp = B[p * width:p * width + span_b]
        if kind == "reference":
            op.ref_cpu_reference(d, A[:R * n], Bp)
        else:
            op.gemm_ref(d, A[:R * n], Bp, nthreads=threads)

    def sample(R):
        ths = [threading.Thread(target=call, args=(R, p)) for p in range(P)]
        t0 = time.perf_counter()
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        return time.perf_counter() - t0

    pts = []
    for _ in range(samples):
        for R in rows:
            pts.append((R, sample(R)))
    xs = np.array([p[0] for p in pts], dtype=np.float64)
    ys = np.array([p[1] for p in pts], dtype=np.float64)
    if len(set(xs)) > 1:
        r, f = np.polyfit(xs, ys, 1)
    else:
        r, f = ys.mean() / xs[0], 0.0
    r, f = max(float(r), 1e-12), max(float(f), 0.0)
    rounds = math.ceil(n / (P * width))
    t_full = rounds * (f + n * r)
    value = 2.0 * n ** 3 / t_full / 1e12
    samp = (f"{P} concurrent reference calls, each on rows [0, R) x a {width}-column block of B (K = {n}), "
            f"R in {list(rows)}, {samples} sample(s) each, {threads} threads per call "
            f"(the reference's min(16, cores)); fitted per call: fixed {f:.3f} s (B transpose + copies) + "
            f"{r * 1e3:.3f} ms per row; full {n}^3 problem extrapolated as {rounds} rounds x "
            f"(fixed + {n} rows) = {t_full:.1f} s; f16 inputs (the reference's CPU GEMM is f16-only), "
            f"FP64 accumulate")
    return {"value": value, "seconds": t_full, "fixed_s": f, "per_row_s": r, "cores": threads * P,
            "kind": kind, "sample": samp, "points": pts}


def oracle_rows_check(A, B, C_rows, rows, n, dtype):
    """Sampled rows of the GPU's n^3 result against the FP64 oracle (the C
    restatement of reference src/bench/reference.cu:69-105 with the exact
    bf16/f16 decode), under the reference's bound c*sqrt(K)*eps and the
    north-star bound eps*K; the size switch of the reference's fuzzer
    (tools/aegis_fuzz.cu:448) checks sampled rows at this size too."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_py as op
    A_s = np.ascontiguousarray(A.reshape(n, n)[rows]).reshape(-1)
    d = op.make_desc(len(rows), n, n, dtype=dtype)
    ref = op.gemm_ref(d, A_s, B)
    tol_ref = op.tolerance(d, A_s, B)
    tol_ns = op.tolerance(d, A_s, B, kind="north_star")
    r = op.compare(d, C_rows.reshape(-1), ref, None, tol_ref)
    import aegis_capi as ac
    got = ac.to_f32(C_rows.reshape(-1), dtype).astype(np.float64).reshape(len(rows), n)
    err = float(np.max(np.abs(got - ref[0])))
    return {"rows": [int(x) for x in rows], "max_err_vs_oracle": err, "tol_reference": tol_ref,
            "tol_north_star": tol_ns, "pass": bool(r["pass"]) and err <= tol_ns}


# ------------------------------------------------------------------ helpers
def torch_view(torch, ptr, nelem, dtype):
    class _Dev:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (nelem,), "typestr": "<i2", "data": (ptr, False),
                                             "version": 3}
    t = torch.as_tensor(_Dev(), device="cuda")
    return t.view(dtype)


def tdtype(torch, name):
    return torch.bfloat16 if name == "bf16" else torch.float16


def emit(line):
    print(json.dumps(line), flush=True)


def max_over_ranks(torch, dist, world, v):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def ctypes_alloc(ctx, nbytes):
    import aegis_capi as ac
    out = ctypes.c_void_p()
    ac.check(ctx.lib.aegis_device_alloc(ctx.ptr, nbytes, ctypes.byref(out)), "aegis_device_alloc")
    return out.value


def ctypes_free(ctx, ptr):
    import aegis_capi as ac
    ac.check(ctx.lib.aegis_device_free(ctx.ptr, ctypes.c_void_p(ptr)), "aegis_device_free")


def graph_ms(torch, stream, fn, warmup, min_window_ms=2.0, windows=7):
    """Per-launch device time of fn(i) (i rotates the caller's buffer sets):
    `warmup` direct calls (any workspace is allocated here, outside capture),
    then windows of `batch` launches captured in one CUDA graph (>= min_window_ms
    each), replayed under CUDA events on `stream`; the median window. As the
    reference harness times graph-captured windows (src/bench/harness.cu:
    279-305), so host launch overhead does not starve the GPU."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(8):
        fn(i)
    e.record(stream)
    torch.cuda.synchronize()
    per = max(s.elapsed_time(e) / 8, 0.002)
    batch = int(min(4000, max(8, math.ceil(min_window_ms / per))))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(batch):
            fn(i)
    graph.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(windows):
        s.record(stream)
        graph.replay()
        e.record(stream)
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e) / batch)
    del graph
    return statistics.median(ts), batch


class LtBaseline:
    """cublaslt_best (tune/lt_baseline.cu): the cuBLASLt heuristic's top
    candidates for a row-major problem, split-K with reduced-precision
    partials dropped (reference src/bench/harness.cu:963-1031)."""
    WORKSPACE = 32 << 20  # the reference harness's cuBLAS workspace (harness.cu:157)

    def __init__(self, torch, bf16, M, N, K):
        path = os.path.join(ROOT, "aegis-core_b200", "build", "libaegis_ltbase.so")
        self.lib = ctypes.CDLL(path)
        self.lib.ltb_create.argtypes = [ctypes.c_int] * 4 + [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p),
                                                             ctypes.POINTER(ctypes.c_int),
                                                             ctypes.POINTER(ctypes.c_int)]
        self.lib.ltb_run.argtypes = [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 4 + [ctypes.c_size_t,
                                                                                            ctypes.c_void_p]
        self.lib.ltb_describe.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        self.lib.ltb_destroy.argtypes = [ctypes.c_void_p]
        self.h = ctypes.c_void_p()
        n, dropped = ctypes.c_int(0), ctypes.c_int(0)
        if self.lib.ltb_create(int(bf16), M, N, K, self.WORKSPACE, ctypes.byref(self.h), ctypes.byref(n),
                               ctypes.byref(dropped)) != 0:
            raise RuntimeError("cuBLASLt heuristic query failed")
        self.n, self.dropped = n.value, dropped.value
        self.ws = torch.empty(self.WORKSPACE, dtype=torch.uint8, device="cuda")

    def run(self, i, A, B, C, stream_ptr):
        rc = self.lib.ltb_run(self.h, i, A, B, C, self.ws.data_ptr(), self.WORKSPACE, stream_ptr)
        if rc != 0:
            raise RuntimeError(f"cublasLtMatmul candidate {i}: status {rc}")

    def describe(self, i):
        buf = ctypes.create_string_buffer(256)
        self.lib.ltb_describe(self.h, i, buf, 256)
        return json.loads(buf.value.decode())

    def close(self):
        if self.h:
            self.lib.ltb_destroy(self.h)
            self.h = ctypes.c_void_p()


# ------------------------------------------------------------------ single-GPU workloads
def measure_workload(torch, ctx, stream, wl, M, N, K, dtype, warmup, impl=None, lt=True):
    """One single-GPU shape through aegis::matmul (the C ABI's
    aegis_gemm_{f16,bf16}), against torch.matmul (cuBLAS) and cublaslt_best,
    each graph-timed with rotating buffer sets totalling >= 3 x L2 (cold L2,
    as the reference harness rotates sets, harness.cu:274-277). Returns the
    workload's record."""
    import aegis_capi as ac
    code = ac.DTYPE_BF16 if dtype == "bf16" else ac.DTYPE_F16
    tdt = tdtype(torch, dtype)
    g = ac.Generator(0)
    if wl == "gemv":  # activations ~N(0, 1), weights ~N(0, 0.02)
        A, B = g.normal(M * K, dtype, 0.0, 1.0), g.normal(K * N, dtype, 0.0, 0.02)
    else:
        A, B = g.uniform(M * K, dtype), g.uniform(K * N, dtype)
    footprint = 2 * (M * K + K * N + M * N)
    nsets = max(2, math.ceil(3 * L2_BYTES / footprint))
    hA = torch.from_numpy(A.view(np.int16))
    hB = torch.from_numpy(B.view(np.int16))
    sets = [(hA.cuda(), hB.cuda(), torch.zeros(M * N, dtype=torch.int16, device="cuda")) for _ in range(nsets)]
    plan = ctx.plan(M, N, K, impl, code)
    kernel = impl or plan["impl"]

    def ours(i):
        dA, dB, dC = sets[i % nsets]
        if impl:
            ctx.gemm_impl(impl, code, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, 0, dB.data_ptr(), N, 0, 0.0,
                          dC.data_ptr(), N, 0, 1)
        else:
            ctx.gemm(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), M, N, K, code)

    ms, batch = graph_ms(torch, stream, ours, warmup)
    outs = [torch.empty(M, N, dtype=tdt, device="cuda") for _ in range(nsets)]

    def cublas(i):
        dA, dB, _ = sets[i % nsets]
        torch.matmul(dA.view(tdt).view(M, K), dB.view(tdt).view(K, N), out=outs[i % nsets])

    cublas_ms, _ = graph_ms(torch, stream, cublas, warmup)
    dA, dB, dC = sets[0]
    a, b = dA.view(tdt).view(M, K), dB.view(tdt).view(K, N)
    ref = (a @ b).float()
    mine = dC.view(tdt).view(M, N).float()
    err = (mine - ref).abs().max().item()
    eps = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
    tol = eps * K * a.float().abs().max().item() * b.float().abs().max().item()
    lt_rec = None
    if lt:
        sweep = LtBaseline(torch, dtype == "bf16", M, N, K)
        best = None
        for c in range(sweep.n):
            def lt_fn(i, c=c):
                dA, dB, _ = sets[i % nsets]
                sweep.run(c, dA.data_ptr(), dB.data_ptr(), outs[i % nsets].data_ptr(), stream.cuda_stream)
            lt_fn(0)
            torch.cuda.synchronize()
            if (outs[0].float() - ref).abs().max().item() > tol:
                continue  # never a baseline that fails the check (harness.cu:1016)
            t, _ = graph_ms(torch, stream, lt_fn, warmup)
            if best is None or t < best[0]:
                best = (t, c)
        if best is not None:
            lt_rec = {"ms": best[0], "algo": sweep.describe(best[1]), "candidates": sweep.n,
                      "dropped_reduced_precision": sweep.dropped}
        sweep.close()
    peaks, src = measured_peaks()
    flops = 2.0 * M * N * K
    rec = {"workload": f"{wl}_{dtype}_{M}x{N}x{K}", "M": M, "N": N, "K": K, "dtype": dtype, "kernel": kernel,
           "plan": plan, "ms": ms, "launches_per_window": batch,
           "l2": f"cold: {nsets} rotating buffer sets (>= 3 x L2)"}
    if wl == "gemv":
        wbytes = 2.0 * K * N

        def rate(t):
            return wbytes / (t * 1e-3) / 1e9
        rec.update({"value": rate(ms), "unit": "GB/s (weights)"})
        rec["roofline"] = {"bound": "hbm", "achieved": rate(ms), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                           "frac": rate(ms) / peaks["hbm_gbs"], "peak_source": f"{src} hbm_gbs",
                           "algorithmic_bytes": "weights 2*K*N per launch",
                           "compulsory_gbs": 2.0 * (M * K + K * N + M * N) / (ms * 1e-3) / 1e9,
                           "traffic": load_traffic(f"gemv_m{M}_{K}x{N}")}
    else:
        def rate(t):
            return flops / (t * 1e-3) / 1e12
        rec.update({"value": rate(ms), "unit": "TFLOP/s"})
        if wl == "splitk" and 2.0 * M * N * K / (2.0 * (M * K + K * N)) < 281:
            # Below the ridge (~1.6 PFLOP/s / 6.5 TB/s): the input stream bounds it.
            hbm = 2.0 * (M * K + K * N + M * N) / (ms * 1e-3) / 1e9
            rec["roofline"] = {"bound": "hbm", "achieved": hbm, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                               "frac": hbm / peaks["hbm_gbs"], "peak_source": f"{src} hbm_gbs",
                               "algorithmic_bytes": "2*(M*K + K*N + M*N) per launch"}
        else:
            rec["roofline"] = {"bound": "tensor", "achieved": rate(ms), "peak": peaks["bf16_tflops"],
                               "unit": "TFLOP/s", "frac": rate(ms) / peaks["bf16_tflops"],
                               "peak_source": f"{src} bf16_tflops (burst)",
                               "traffic": load_traffic(f"{kernel}_{dtype}_{M}x{N}x{K}")}
    rec["cublas"] = {"value": rate(cublas_ms), "ratio_ours_over_cublas": cublas_ms / ms,
                     "what": "torch.matmul (cuBLAS), same buffers and timing"}
    if lt_rec:
        rec["cublaslt_best"] = {"value": rate(lt_rec["ms"]), "ratio_ours_over_cublaslt_best": lt_rec["ms"] / ms,
                                "algo": lt_rec["algo"], "candidates": lt_rec["candidates"],
                                "dropped_reduced_precision": lt_rec["dropped_reduced_precision"]}
    rec["check"] = {"max_abs_err_vs_cublas": err, "tol_north_star": tol, "pass": err <= tol}
    split = plan.get("splits", 1) > 1 and kernel.startswith("umma")
    rec["gpu_launches_per_call"] = 2 if split else 1
    del sets, outs
    return rec


SECONDARY = [  # (workload, M, N, K, dtype): the single-GPU targets and the tall-K case
    ("square", 8192, 8192, 8192, "bf16"),
    ("square", 8192, 8192, 8192, "f16"),
    ("gemv", 1, 14336, 4096, "f16"),
    ("gemv", 1, 4096, 4096, "f16"),
    ("splitk", 256, 256, 65536, "bf16"),
]


def secondary_workloads(torch, ctx, stream, warmup):
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    out = {}
    for wl, M, N, K, dt in SECONDARY:
        rec = measure_workload(torch, ctx, stream, wl, M, N, K, dt, warmup)
        out[rec["workload"]] = rec
        torch.cuda.empty_cache()
    out["clocks"] = clocks.stop()
    return out


def bench_single(args):
    import torch

    import aegis_capi as ac
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx = ac.Context(0)
    ctx.set_stream(stream.cuda_stream)
    wl = args.workload
    if wl == "square":
        M = N = K = args.size or 8192
        dtype = args.dtype or "bf16"
    elif wl == "splitk":
        M = N = args.size or 1024
        K = args.k or 65536
        dtype = args.dtype or "bf16"
    elif wl == "gemm":  # any M x N x K, uniform[-1, 1]
        M, N, K = args.m or 16384, args.n or 2048, args.k or 16384
        dtype = args.dtype or "bf16"
    else:
        M, K, N = args.m or 1, args.k or 4096, args.n or 4096
        dtype = args.dtype or "f16"
    clocks = ClockSampler(0)
    clocks.start()
    rec = measure_workload(torch, ctx, stream, wl, M, N, K, dtype, args.warmup, impl=args.kernel,
                           lt=not args.no_lt)
    clk = clocks.stop()
    line = {"metric": {"square": "GEMM TFLOP/s", "splitk": "GEMM TFLOP/s (tall-K split-K)", "gemm": "GEMM TFLOP/s",
                       "gemv": "GEMV HBM GB/s (weights)"}[wl],
            "value": rec["value"], "unit": rec["unit"], "n_gpus": 1, "steps": rec["launches_per_window"],
            "warmup": args.warmup, "ms_per_step": rec["ms"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic seeded (std::mt19937(0))",
            "config": {"workload": rec["workload"], "M": M, "N": N, "K": K, "kernel": rec["kernel"],
                       "plan": rec["plan"], "l2": rec["l2"],
                       "timing": "CUDA graph windows of the launches, median of 7 replays under events"},
            "roofline": rec["roofline"], "clocks": clk,
            "gpu_launches": rec["launches_per_window"] * rec["gpu_launches_per_call"],
            "cublas": rec["cublas"], "cublaslt_best": rec.get("cublaslt_best"), "check": rec["check"]}
    ctx.close()
    return line


# ------------------------------------------------------------------ nshard (default)
def bench_nshard(args, rank, local_rank, world):
    import torch
    import torch.distributed as dist

    import aegis_capi as ac
    import aegis_dist as ad

    n = args.size or 16384
    M = N = K = n
    dtype = args.dtype or "bf16"
    code = ac.DTYPE_BF16 if dtype == "bf16" else ac.DTYPE_F16
    tdt = tdtype(torch, dtype)
    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local_rank))
    stream = torch.cuda.Stream()  # the GEMM, its barriers and the baselines of this rank
    torch.cuda.set_stream(stream)
    ctx = ac.Context(local_rank)
    ctx.set_stream(stream.cuda_stream)
    c0, ns = ad.shard_columns(N, world, rank)

    # Host inputs: std::mt19937(0), uniform[-1, 1], A then B (the reference's order).
    g = ac.Generator(0)
    A = g.uniform(M * K, dtype)
    B = g.uniform(K * N, dtype)
    B_shard = np.ascontiguousarray(B.reshape(K, N)[:, c0:c0 + ns]).reshape(-1)
    dA = torch.from_numpy(A.view(np.int16)).cuda()
    dB = torch.from_numpy(B_shard.view(np.int16)).cuda()
    backend = ad.CudaIpcBackend(ctx)
    # Two C buffers, each visible to every rank (CUDA IPC): the pipelined e2e
    # loop alternates between them; the device-resident loop uses C[0].
    c_ptrs, pms, peers = [], [], []
    for _ in range(2):
        p = ctypes_alloc(ctx, M * N * 2)
        torch_view(torch, p, M * N, torch.int16).zero_()
        c_ptrs.append(p)
        if world > 1:
            pm = ad.exchange_handles(backend, p)
            pms.append(pm)
            peers.append(pm.addrs)
        else:
            peers.append([p])
    C = torch_view(torch, c_ptrs[0], M * N, torch.int16)
    flag = torch.zeros(1, dtype=torch.float32, device="cuda")

    def gemm(j, a_ptr=None, b_ptr=None):
        ctx.nsharded(M, N, K, a_ptr or dA.data_ptr(), K, b_ptr or dB.data_ptr(), ns, peers[j], N, world, rank, code)

    def barrier_on_stream():
        if world > 1:
            dist.all_reduce(flag)  # ordered after this rank's earlier work on the current stream

    def barrier():
        if world > 1:
            dist.barrier()

    k_ev = []

    def step(record=False):
        # Contract of the N-sharded call (include/aegis.h): every rank's C must
        # be free before the call (nobody still reading the previous result)
        # and complete only after the barrier that follows it. Nothing reads C
        # between steps here, so the barrier after the call is enough.
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        gemm(0)
        if record:
            e1.record(stream)
            k_ev.append((e0, e1))
        barrier_on_stream()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()

    # Correctness (outside timing): this rank's block against cuBLAS; every
    # rank's gathered C must hold identical per-block checksums.
    a = dA.view(tdt).view(M, K)
    b = dB.view(tdt).view(K, ns)
    cmine = C.view(tdt).view(M, N)
    ref = a @ b
    eps = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
    tol = 2 * (2.0 * math.sqrt(K) * eps)  # 2x the reference bound (both results rounded), max|A|,|B| <= 1
    err = (cmine[:, c0:c0 + ns].float() - ref.float()).abs().max().item()
    sums = torch.stack([cmine[:, r * ns:(r + 1) * ns].float().sum(dtype=torch.float64) for r in range(world)])
    if world > 1:
        allsums = [torch.zeros_like(sums) for _ in range(world)]
        dist.all_gather(allsums, sums)
        same = all(torch.equal(allsums[0], s) for s in allsums)
    else:
        same = True
    del ref
    if err > tol or not same:
        raise SystemExit(f"bench: result check failed on rank {rank}: max err {err} (tol {tol}), "
                         f"checksums identical: {same}")
    rng = np.random.RandomState(20261202)
    check_rows = sorted({0, M - 1} | set(int(x) for x in rng.choice(M, 14, replace=False)))
    C_rows = cmine[check_rows].contiguous().view(torch.int16).cpu().numpy().view(np.uint16) if rank == 0 else None

    # cuBLAS (+ NCCL all-gather at N > 1) on the same shapes: the library baseline.
    gathered = torch.empty(world * M * ns, dtype=tdt, device="cuda") if world > 1 else None
    out_cb = torch.empty(M, ns, dtype=tdt, device="cuda")

    def cublas_step():
        torch.matmul(a, b, out=out_cb)
        if world > 1:
            dist.all_gather_into_tensor(gathered, out_cb.view(-1))

    for _ in range(args.warmup):
        cublas_step()
    torch.cuda.synchronize()
    barrier()
    cs, ce = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cs.record(stream)
    for _ in range(args.steps):
        cublas_step()
    ce.record(stream)
    torch.cuda.synchronize()
    cublas_ms = max_over_ranks(torch, dist, world, cs.elapsed_time(ce) / args.steps)
    del gathered, out_cb
    barrier()

    # At N > 1: this rank's GEMM alone (same kernel and shard, no peer stores),
    # to show what the fused all-gather costs on top of the math.
    local_ms = None
    if world > 1:
        cptr_shard = c_ptrs[1] + 2 * c0

        def local():
            ctx.gemm_impl("umma_256x256x64_s7_c2", code, 0, 0, M, ns, K, 1.0, dA.data_ptr(), K, 0, dB.data_ptr(),
                          ns, 0, 0.0, cptr_shard, N, 0, 1)
        for _ in range(args.warmup):
            local()
        ls, le = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ls.record(stream)
        for _ in range(args.steps):
            local()
        le.record(stream)
        torch.cuda.synchronize()
        local_ms = ls.elapsed_time(le) / args.steps
        barrier()

    # Timed region: K steps, device-resident inputs.
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record(stream)
    for _ in range(args.steps):
        step(record=True)
    e_ev.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(torch, dist, world, s_ev.elapsed_time(e_ev) / args.steps)
    kernel_ms = statistics.mean(x.elapsed_time(y) for x, y in k_ev)

    e2e = None
    if not args.no_e2e:
        e2e = e2e_pipelined(torch, dist, ctx, args, world, rank, M, N, K, ns, c0, A, B_shard, c_ptrs, peers, code,
                            flag, stream)

    flops = 2.0 * M * N * K
    peaks, src = measured_peaks()
    achieved = 2.0 * M * ns * K / (kernel_ms * 1e-3) / 1e12
    traffic = load_traffic(f"umma_nshard_{dtype}_{n}") if world == 1 else None
    line = {
        "metric": METRIC.format(dtype=dtype, n=n),
        "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": dtype, "data": "synthetic: std::mt19937(0) uniform[-1,1], A then B",
        "config": {"workload": f"gemm_{dtype}_{n}^3_nshard", "M": M, "N": N, "K": K,
                   "parallelism": f"nshard{world}", "l2": "inputs larger than L2 (A = %d MiB)" % (M * K * 2 >> 20),
                   "kernel": "umma_256x256x64_s7_c2 (tcgen05 cta_group::2, peer-store epilogue)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"], "traffic": traffic,
                     "peak_source": f"{src} bf16_tflops (burst: the timed region is "
                                    f"{args.steps * ms / 1e3:.2f} s, not a seconds-long power-capped loop)",
                     "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"],
                     "algorithmic_flop_per_launch": 2.0 * M * ns * K},
        "clocks": clk,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "cublas": {"value": flops / (cublas_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                   "what": "torch.matmul per shard" + (" + NCCL all_gather_into_tensor" if world > 1 else ""),
                   "ratio_ours_over_cublas": cublas_ms / ms},
        "check": {"max_err_vs_cublas": err, "tol": tol, "gathered_checksums_identical": same},
    }
    if local_ms is not None:
        line["per_rank_kernel_ms"] = {"local_only": local_ms, "with_peer_push": kernel_ms, "npeers": world,
                                      "push_overhead": kernel_ms / local_ms - 1.0}
    if pms:
        torch.cuda.synchronize()
        barrier()
        for pm in pms:
            ad.close_peers(backend, pm)
    barrier()
    for p in c_ptrs:
        ctypes_free(ctx, p)
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and world == 1:
        if not args.no_cpu_baseline:
            cb = cpu_reference_rate(n, samples=2)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "cores", "kind", "sample")}
            line["cpu_baseline"]["unit"] = "TFLOP/s"
            line["check"]["oracle_rows"] = oracle_rows_check(A, B, C_rows, check_rows, n, dtype)
            line["check"]["max_err_vs_oracle"] = line["check"]["oracle_rows"]["max_err_vs_oracle"]
        if not args.no_workloads:
            line["workloads"] = secondary_workloads(torch, ctx, stream, args.warmup)
    ctx.close()
    return line if rank == 0 else None


def e2e_pipelined(torch, dist, ctx, args, world, rank, M, N, K, ns, c0, A, B_shard, c_ptrs, peers, code, flag,
                  stream):
    """End to end through the C ABI: every step copies its inputs in from
    pinned host memory, runs aegis_gemm_*_nsharded and reads C back, all
    inside the timed region. Two buffer sets alternate, so the copies of one
    step overlap the GEMM of the previous one:
      - copy-in stream: this rank's rows [r*M/P, (r+1)*M/P) of A and its B
        shard; at N > 1 the A slices are all-gathered over NVLink (NCCL), so
        each rank copies 1/P of A from the host instead of all of it;
      - compute stream: a barrier (no rank may store into a C that a peer is
        still reading back), the GEMM with its fused all-gather of C, the
        barrier after it;
      - copy-out stream: this rank reads back rows [r*M/P, (r+1)*M/P) of the
        gathered C, so the ranks together return all of C to the host.
    Bytes per step are whole-job totals."""
    h = M // world
    r0 = rank * h
    hA = torch.from_numpy(np.ascontiguousarray(A.reshape(M, K)[r0:r0 + h]).view(np.int16).reshape(-1)).pin_memory()
    hB = torch.from_numpy(B_shard.view(np.int16)).pin_memory()
    hC = torch.empty(h * N, dtype=torch.int16, pin_memory=True)
    dAs = [torch.empty(M * K, dtype=torch.int16, device="cuda") for _ in range(2)]
    dBs = [torch.empty(K * ns, dtype=torch.int16, device="cuda") for _ in range(2)]
    Cs = [torch_view(torch, p, M * N, torch.int16) for p in c_ptrs]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_gemm = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for j in range(2):  # all events start "done"
        ev_gemm[j].record(stream)
        ev_out[j].record(stream)

    def run_step(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_gemm[j])  # GEMM i-2 is done reading this set
            dAs[j][r0 * K:(r0 + h) * K].copy_(hA, non_blocking=True)
            dBs[j].copy_(hB, non_blocking=True)
            ev_in[j].record(s_in)
        stream.wait_event(ev_in[j])
        if world > 1:  # bytes only: any 16-bit type NCCL takes
            dist.all_gather_into_tensor(dAs[j].view(torch.bfloat16), dAs[j][r0 * K:(r0 + h) * K].view(torch.bfloat16))
        stream.wait_event(ev_out[j])  # this rank's read-back of C[j] (step i-2) is done
        if world > 1:
            dist.all_reduce(flag)  # ... and every other rank's: C[j] is free everywhere
        ctx.nsharded(M, N, K, dAs[j].data_ptr(), K, dBs[j].data_ptr(), ns, peers[j], N, world, rank, code)
        if world > 1:
            dist.all_reduce(flag)  # every rank's tiles have landed in C[j]
        ev_gemm[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_gemm[j])
            hC.copy_(Cs[j][r0 * N:(r0 + h) * N], non_blocking=True)
            ev_out[j].record(s_out)

    for i in range(max(2, args.warmup)):
        run_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    s_in.wait_event(es)
    for i in range(args.steps):
        run_step(i)
    stream.wait_event(ev_out[(args.steps - 1) % 2])
    ee.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(torch, dist, world, es.elapsed_time(ee) / args.steps)
    if world > 1:
        dist.barrier()
    return {"value": 2.0 * M * N * K / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": (M * K + K * N) * 2, "d2h_bytes_per_step": M * N * 2, "ms_per_step": e2e_ms,
            "api": "aegis_gemm_%s_nsharded (C ABI); pinned host buffers; two buffer sets, copy-in / compute / "
                   "copy-out streams; at N > 1 each rank copies 1/N of A in (NCCL all-gather of A) and reads "
                   "1/N of C's rows back" % ("bf16" if code == 1 else "f16")}


# ------------------------------------------------------------------ reference arm
def reference_arm(args, rank, world):
    """The reference's own CPU GEMM on the headline workload: each step is one
    pair of timed samples (cpu_reference_rate); the line's value is the
    full-problem throughput extrapolated from the steps after warm-up."""
    if rank != 0:
        return None
    n = args.size or 16384
    M = N = K = n
    dtype = args.dtype or "bf16"
    cpu_reference_rate(n, samples=args.warmup)  # warm-up steps
    cb = cpu_reference_rate(n, samples=args.steps)
    value = cb["value"]
    return {"impl": "reference", "metric": METRIC.format(dtype=dtype, n=n),
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cb["seconds"] * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic: std::mt19937(0) uniform[-1,1], A then B",
            "config": {"workload": f"gemm_{dtype}_{n}^3_nshard", "M": M, "N": N, "K": K,
                       "parallelism": "host cores"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cb["cores"], "kind": cb["kind"],
                             "sample": cb["sample"]},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    args = parse_args()
    rank, local_rank, world = dist_env()
    if args.gpus != world and not (args.gpus >= 1 and world == 1 and args.gpus == 1):
        if world == 1 and args.gpus > 1:
            raise SystemExit(f"--gpus {args.gpus} needs torchrun --nproc-per-node {args.gpus}")
    if args.impl == "reference":
        line = reference_arm(args, rank, world)
    elif args.workload == "nshard":
        line = bench_nshard(args, rank, local_rank, world)
    else:
        if world > 1:
            raise SystemExit("single-GPU workloads run with --gpus 1")
        line = bench_single(args)
    if line is not None and rank == 0:
        emit(line)


if __name__ == "__main__":
    main()
