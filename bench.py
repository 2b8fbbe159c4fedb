#!/usr/bin/env python
"""Benchmark of the aegis-b200 hot path; prints ONE JSON line (rank 0).

Default workload (every N): BASELINE config 5, C = A*B with M = N = K = 16384,
bf16 in, FP32 accumulate, bf16 out, B N-sharded over the N GPUs (column
shards), and C all-gathered by the GEMM itself: aegis_gemm_bf16_nsharded
stores every finished tile into every rank's C (NVLink peer stores), then a
one-element NCCL all-reduce is the cross-rank barrier. At N = 1 it is the
plain 16384^3 GEMM. Inputs uniform[-1, 1] from std::mt19937(0) (A then B),
larger than L2 (A alone is 512 MiB), so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl aegis|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...

Other single-GPU workloads for measurement (`--workload square|gemv|splitk`)
print the same line for BASELINE configs 2-4.

`--impl reference` times the reference's own CPU GEMM
(aegis::bench::cpu_reference, FP64 accumulate, built from its source into
oracle/_ref; the C restatement oracle/liboracle.so when that is absent) on a
row sample of the same workload, on rank 0; other ranks exit at once.
"""
from __future__ import annotations

import argparse
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


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["aegis", "reference"], default="aegis")
    p.add_argument("--workload", choices=["nshard", "square", "gemv", "splitk"], default="nshard")
    p.add_argument("--size", type=int, default=None, help="square: M=N=K; nshard: M=N=K; splitk: M=N")
    p.add_argument("--k", type=int, default=None, help="gemv/splitk: K")
    p.add_argument("--n", type=int, default=None, help="gemv: N")
    p.add_argument("--m", type=int, default=None, help="gemv: M")
    p.add_argument("--dtype", choices=["bf16", "f16"], default=None)
    p.add_argument("--kernel", default=None, help="force a registry kernel (single-GPU workloads)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    a = p.parse_args()
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
def cpu_leg(n, rows, repeats=1):
    """Time the reference's own CPU GEMM (aegis::bench::cpu_reference from
    oracle/_ref; the C restatement when that is absent) on `rows` rows of the
    n^3 problem. The reference is f16-only, so the sample is f16 data from the
    same generator (its FP64 arithmetic does not depend on the input type).
    Returns (mean seconds per repeat, kind, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import aegis_capi as ac
    import oracle_py as op
    g = ac.Generator(0)
    A_rows = g.uniform(rows * n, "f16")
    g.uniform((n - rows) * n, "f16")  # the rest of A: B comes after all of A in the stream
    B = g.uniform(n * n, "f16")
    d = op.make_desc(rows, n, n, dtype="f16")
    threads = min(16, os.cpu_count() or 1)
    kind = "reference" if op.ref_available() else "port"
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        if kind == "reference":
            op.ref_cpu_reference(d, A_rows, B)
        else:
            op.gemm_ref(d, A_rows, B, nthreads=threads)
        times.append(time.perf_counter() - t0)
    return times, kind, threads


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
    stream = torch.cuda.Stream()  # every launch, copy, event and collective of this rank on one stream
    torch.cuda.set_stream(stream)
    ctx = ac.Context(local_rank)
    ctx.set_stream(stream.cuda_stream)
    c0, ns = ad.shard_columns(N, world, rank)

    # Host inputs: std::mt19937(0), uniform[-1, 1], A then B (the reference's order).
    g = ac.Generator(0)
    A = g.uniform(M * K, dtype)
    B = g.uniform(K * N, dtype)
    B_shard = np.ascontiguousarray(B.reshape(K, N)[:, c0:c0 + ns])
    hA = torch.from_numpy(A.view(np.int16)).pin_memory()
    hB = torch.from_numpy(B_shard.view(np.int16).reshape(-1)).pin_memory()
    dA = torch.empty(M * K, dtype=torch.int16, device="cuda")
    dB = torch.empty(K * ns, dtype=torch.int16, device="cuda")
    dA.copy_(hA)
    dB.copy_(hB)
    c_ptr = ctypes_alloc(ctx, M * N * 2)
    C = torch_view(torch, c_ptr, M * N, torch.int16)
    C.zero_()
    backend = ad.CudaIpcBackend(ctx)
    if world > 1:
        pm = ad.exchange_handles(backend, c_ptr)
        peers = pm.addrs
    else:
        pm, peers = None, [c_ptr]
    flag = torch.zeros(1, dtype=torch.float32, device="cuda")

    k_ev = []

    def step(record=False):
        if record:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        ctx.nsharded(M, N, K, dA.data_ptr(), K, dB.data_ptr(), ns, peers, N, world, rank, code)
        if record:
            e1.record(stream)
            k_ev.append((e0, e1))
        if world > 1:
            dist.all_reduce(flag)  # barrier, ordered after the GEMM on the stream

    def barrier():
        if world > 1:
            dist.barrier()

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

    # End to end through the C ABI: pinned host inputs in, GEMM + gather, the
    # gathered C out on rank 0, all inside the timed region.
    e2e = None
    if not args.no_e2e:
        hC = torch.empty(M * N, dtype=torch.int16, pin_memory=True) if rank == 0 else None
        for _ in range(2):
            dA.copy_(hA, non_blocking=True)
            dB.copy_(hB, non_blocking=True)
            step()
            if rank == 0:
                hC.copy_(C, non_blocking=True)
        torch.cuda.synchronize()
        barrier()
        es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        es.record(stream)
        for _ in range(args.steps):
            dA.copy_(hA, non_blocking=True)
            dB.copy_(hB, non_blocking=True)
            step()
            if rank == 0:
                hC.copy_(C, non_blocking=True)
        ee.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(torch, dist, world, es.elapsed_time(ee) / args.steps)
        flops = 2.0 * M * N * K
        e2e = {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": (M * K + K * ns) * 2 * world, "d2h_bytes_per_step": M * N * 2,
               "ms_per_step": e2e_ms, "api": "aegis_gemm_%s_nsharded (C ABI), pinned host buffers" % dtype}

    flops = 2.0 * M * N * K
    peaks, src = measured_peaks()
    achieved = 2.0 * M * ns * K / (kernel_ms * 1e-3) / 1e12
    traffic = load_traffic(f"umma_nshard_{dtype}_{n}") if world == 1 else None
    line = {
        "metric": f"GEMM TFLOP/s ({dtype} {n}^3, B N-sharded, C all-gathered in the epilogue)",
        "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": dtype, "data": "synthetic: std::mt19937(0) uniform[-1,1], A then B",
        "config": {"workload": f"config5_gemm_{dtype}_{n}^3_nshard", "M": M, "N": N, "K": K,
                   "parallelism": f"nshard{world}", "l2": "inputs larger than L2 (A = %d MiB)" % (M * K * 2 >> 20),
                   "kernel": "umma_256x256x64_s7_c2 (tcgen05 cta_group::2, peer-store epilogue)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops_sustained"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops_sustained"],
                     "traffic": traffic, "peak_source": f"{src} bf16_tflops_sustained",
                     "frac_of_burst": achieved / peaks["bf16_tflops"]},
        "clocks": clk,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "cublas": {"value": flops / (cublas_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                   "what": "torch.matmul per shard" + (" + NCCL all_gather_into_tensor" if world > 1 else ""),
                   "ratio_ours_over_cublas": cublas_ms / ms},
        "check": {"max_err_vs_cublas": err, "tol": tol, "gathered_checksums_identical": same},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = 64
        times, kind, threads = cpu_leg(n, rows)
        line["cpu_baseline"] = {"value": 2.0 * rows * N * K / times[0] / 1e12, "unit": "TFLOP/s", "cores": threads,
                                "kind": kind, "sample": f"{rows} rows of the {n}^3 problem (A[0:{rows}] x B), f16 "
                                f"inputs (the reference's CPU GEMM is f16-only), FP64 accumulate, {times[0]:.2f} s"}
    if pm is not None:
        torch.cuda.synchronize()
        barrier()
        ad.close_peers(backend, pm)
    barrier()
    ctypes_free(ctx, c_ptr)
    if world > 1:
        dist.destroy_process_group()
    return line if rank == 0 else None


def max_over_ranks(torch, dist, world, v):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def ctypes_alloc(ctx, nbytes):
    import ctypes
    import aegis_capi as ac
    out = ctypes.c_void_p()
    ac.check(ctx.lib.aegis_device_alloc(ctx.ptr, nbytes, ctypes.byref(out)), "aegis_device_alloc")
    return out.value


def ctypes_free(ctx, ptr):
    import ctypes
    import aegis_capi as ac
    ac.check(ctx.lib.aegis_device_free(ctx.ptr, ctypes.c_void_p(ptr)), "aegis_device_free")


# ------------------------------------------------------------------ single-GPU workloads
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
        n = args.size or 8192
        M = N = K = n
        dtype = args.dtype or "bf16"
        gen = "uniform"
    elif wl == "splitk":
        M = N = args.size or 1024
        K = args.k or 65536
        dtype = args.dtype or "bf16"
        gen = "uniform"
    else:  # gemv
        M = args.m or 1
        K = args.k or 4096
        N = args.n or 4096
        dtype = args.dtype or "f16"
        gen = "normal"
    code = ac.DTYPE_BF16 if dtype == "bf16" else ac.DTYPE_F16
    tdt = tdtype(torch, dtype)
    g = ac.Generator(0)
    if gen == "uniform":
        A, B = g.uniform(M * K, dtype), g.uniform(K * N, dtype)
    else:
        A, B = g.normal(M * K, dtype, 0.0, 1.0), g.normal(K * N, dtype, 0.0, 0.02)
    footprint = 2 * (M * K + K * N + M * N)
    nsets = max(1, math.ceil(3 * L2_BYTES / footprint))  # cold L2: rotate buffer sets >= 3 x L2
    hA = torch.from_numpy(A.view(np.int16)).pin_memory()
    hB = torch.from_numpy(B.view(np.int16)).pin_memory()
    sets = []
    for _ in range(nsets):
        dA = hA.cuda()
        dB = hB.cuda()
        dC = torch.zeros(M * N, dtype=torch.int16, device="cuda")
        sets.append((dA, dB, dC))
    impl = args.kernel

    def launch(i):
        dA, dB, dC = sets[i % nsets]
        if impl:
            ctx.gemm_impl(impl, code, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, 0, dB.data_ptr(), N, 0, 0.0,
                          dC.data_ptr(), N, 0, 1)
        else:
            ctx.gemm(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), M, N, K, code)

    def timed(fn, steps):
        """Per-launch device time. Direct warm-up calls first (they allocate any
        workspace, outside capture); then the `steps` launches are captured in
        one CUDA graph and its replay is timed with events on the stream, as the
        reference harness times graph-captured windows (src/bench/harness.cu:
        279-305), so host launch overhead does not starve the GPU."""
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            ctx.set_stream(stream.cuda_stream)
            for i in range(steps):
                fn(i)
        ctx.set_stream(stream.cuda_stream)
        graph.replay()  # warm replay
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        graph.replay()
        e.record(stream)
        torch.cuda.synchronize()
        del graph
        return s.elapsed_time(e) / steps

    steps = args.steps
    if steps * 1.0 < 50 and M * N * K < 2 ** 36:
        steps = max(steps, 200)  # short kernels: enough launches for a stable mean
    clocks = ClockSampler(0)
    clocks.start()
    ms = timed(launch, steps)
    clk = clocks.stop()
    # correctness vs cuBLAS on set 0
    dA, dB, dC = sets[0]
    a, b = dA.view(tdt).view(M, K), dB.view(tdt).view(K, N)
    ref = (a @ b).float()
    err = (dC.view(tdt).view(M, N).float() - ref).abs().max().item()
    outs = [torch.empty(M, N, dtype=tdt, device="cuda") for _ in range(nsets)]

    def cublas(i):
        dA, dB, _ = sets[i % nsets]
        torch.matmul(dA.view(tdt).view(M, K), dB.view(tdt).view(K, N), out=outs[i % nsets])

    cub_clocks = ClockSampler(0)
    cub_clocks.start()
    cublas_ms = timed(cublas, steps)
    cub_clk = cub_clocks.stop()
    peaks, src = measured_peaks()
    flops = 2.0 * M * N * K
    choice = impl or ctx.choice(M, N, K)
    plan = ctx.plan(M, N, K, impl, code)
    if wl == "gemv":
        wbytes = 2.0 * K * N
        value = wbytes / (ms * 1e-3) / 1e9
        unit = "GB/s"
        roof = {"bound": "hbm", "achieved": value, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": value / peaks["hbm_gbs"], "traffic": load_traffic(f"gemv_m{M}_{K}x{N}"),
                "peak_source": f"{src} hbm_gbs", "algorithmic_bytes": "weights 2*K*N per launch",
                "compulsory_gbs": 2.0 * (M * K + K * N + M * N) / (ms * 1e-3) / 1e9}
        cub = {"value": wbytes / (cublas_ms * 1e-3) / 1e9, "unit": "GB/s"}
    else:
        value = flops / (ms * 1e-3) / 1e12
        unit = "TFLOP/s"
        roof = {"bound": "tensor", "achieved": value, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": value / peaks["bf16_tflops"], "traffic": load_traffic(f"{choice}_{dtype}_{M}x{N}x{K}"),
                "peak_source": f"{src} bf16_tflops (burst)",
                "frac_of_sustained": value / peaks["bf16_tflops_sustained"]}
        if wl == "splitk":
            hbm = 2.0 * (M * K + K * N) / (ms * 1e-3) / 1e9
            roof["hbm_gbs_of_inputs"] = hbm
            roof["hbm_frac"] = hbm / peaks["hbm_gbs"]
        cub = {"value": flops / (cublas_ms * 1e-3) / 1e12, "unit": "TFLOP/s"}
    cub["ratio_ours_over_cublas"] = cublas_ms / ms
    cub["clocks"] = {k: cub_clk.get(k) for k in ("sm_mhz", "power_w", "reasons")}
    line = {"metric": {"square": "GEMM TFLOP/s", "splitk": "GEMM TFLOP/s (tall-K split-K)",
                       "gemv": "GEMV HBM GB/s (weights)"}[wl],
            "value": value, "unit": unit, "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic seeded (std::mt19937(0))",
            "config": {"workload": f"{wl}_{dtype}_{M}x{N}x{K}", "M": M, "N": N, "K": K, "kernel": choice,
                       "plan": plan, "l2": f"cold: {nsets} rotating buffer sets (>= 3 x L2)",
                       "timing": "CUDA graph of the timed launches, replayed once under events"},
            "roofline": roof, "clocks": clk, "gpu_launches": steps * (2 if plan.get("splits", 1) > 1 and
                                                                      choice.startswith("umma") else 1),
            "cublas": cub, "check": {"max_abs_err_vs_cublas": err}}
    ctx.close()
    return line


# ------------------------------------------------------------------ reference arm
def reference_arm(args, rank, world):
    if rank != 0:
        return None
    n = args.size or 16384
    M = N = K = n
    dtype = args.dtype or "bf16"
    rows = 32
    times, kind, threads = cpu_leg(n, rows, repeats=args.warmup + args.steps)
    sec = statistics.mean(times[args.warmup:])
    value = 2.0 * rows * N * K / sec / 1e12
    sample = (f"{rows} rows of the {n}^3 GEMM per step (A[0:{rows}] x B), f16 inputs (the reference's CPU GEMM "
              f"is f16-only), FP64 accumulate")
    return {"impl": "reference", "metric": f"GEMM TFLOP/s ({dtype} {n}^3, B N-sharded, C all-gathered in the epilogue)",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic: std::mt19937(0) uniform[-1,1], A then B",
            "config": {"workload": f"config5_gemm_{dtype}_{n}^3_nshard", "M": M, "N": N, "K": K,
                       "parallelism": "host cores"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
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
