"""Randomized GEMM correctness against the FP64 oracle: the port of the
reference's tools/aegis_fuzz.cu (the production bar).

Each case comes from tests/fuzz_cases.py and runs through the C ABI: a named
registry kernel (aegis_gemm_impl) or the dispatcher (aegis_gemm_*_strided_batched).
A case passes when all four hold:
- every element is within the reference's bound c·√K·eps·max|A|·max|B|·|α| + eps·|β|·max|C0|
  (c = 2) and the north-star bound eps·K·…;
- NaN stays NaN and Inf stays the same Inf;
- C's padding columns are untouched;
- nothing is written outside C's span (NaN or sentinel guards around every allocation).

Modes: default, decode, large-K and poison (NaN everywhere outside the logical matrices).
The corrupt self-test pushes one element of a correct result past the bound, on the host
copy, and requires the checker to report it.

Case counts (AEGIS_FUZZ_CASES scales them; AEGIS_FUZZ_SEED picks the stream) keep the
default GPU suite to about a minute. A failing case replays alone:
AEGIS_FUZZ_SEED=s AEGIS_FUZZ_ONLY=i.
"""
import os

import numpy as np
import pytest

import aegis_capi as ac
import oracle_py as op
from fuzz_cases import GUARD, make_case
from gpu_util import context

SEED = int(os.environ.get("AEGIS_FUZZ_SEED", "1"))
SCALE = float(os.environ.get("AEGIS_FUZZ_CASES", "1"))
ONLY = os.environ.get("AEGIS_FUZZ_ONLY")
COUNTS = {"default": 160, "decode": 48, "large_k": 12, "poison": 64}
NAN16 = {"f16": 0x7E00, "bf16": 0x7FC0}
SENTINEL = 0x5A5A


def _impls(ctx):
    return [None] + [e["name"] for e in ctx.registry() if e["supported"]]


def _logical_mask(span, batch, stride, rows, cols, row_major, ld):
    mask = np.zeros(span, dtype=bool)
    r = np.arange(rows)[:, None]
    c = np.arange(cols)[None, :]
    idx = r * ld + c if row_major else c * ld + r
    for b in range(batch):
        mask[b * stride + idx.ravel()] = True
    return mask, idx


def build(case, poison, seed=SEED):
    """Host operands of a case (uint16 spans) and its oracle descriptor."""
    bf = case.dtype == "bf16"
    d = op.make_desc(case.M, case.N, case.K, case.layout_a, case.layout_b, case.lda, case.ldb, case.ldc, case.alpha,
                     case.beta, case.batch, case.stride_a, case.stride_b, case.stride_c, case.dtype)
    sa, sb, sc = op.spans(d)
    rng = np.random.default_rng([seed, case.index, 7])
    s = case.scale
    A = ac.f32_to_16(rng.uniform(-s, s, sa).astype(np.float32), bf)
    B = ac.f32_to_16(rng.uniform(-s, s, sb).astype(np.float32), bf)
    C0 = ac.f32_to_16(rng.uniform(-1, 1, sc).astype(np.float32), bf)
    ma, ia = _logical_mask(sa, case.batch, case.stride_a, case.M, case.K, case.layout_a == 0, case.lda)
    mb, ib = _logical_mask(sb, case.batch, case.stride_b, case.K, case.N, case.layout_b == 0, case.ldb)
    mc, _ = _logical_mask(sc, case.batch, case.stride_c, case.M, case.N, True, case.ldc)
    nan = NAN16[case.dtype]
    if poison:
        A[~ma] = nan
        B[~mb] = nan
        if case.beta != 0:
            C0[~mc] = nan
    if case.beta == 0:
        C0[:] = nan  # C must not be read
    for which, r, c, val in case.inject:
        enc = int(ac.f32_to_16(np.array([val], np.float32), bf)[0])
        if which == "A":
            A[ia[r, c]] = enc
        else:
            B[ib[r, c]] = enc
    return d, A, B, C0


def corrupt_first(out, ref, tol, bf16):
    """Push the first element past the bound (a NaN expectation becomes 0)."""
    want = ref[0, 0, 0]
    bad = 0.0 if not np.isfinite(want) else want + (4.0 * tol if tol > 0 else 1.0) + abs(want) * 0.5
    out[0] = int(ac.f32_to_16(np.array([bad], np.float32), bf16)[0])


def _to_device(torch, host_u16, off, guard_value):
    full = np.full(host_u16.size + off + 2 * GUARD, guard_value, dtype=np.uint16)
    full[GUARD + off:GUARD + off + host_u16.size] = host_u16
    return torch.from_numpy(full.view(np.int16)).cuda(), full


def run_case(torch, ctx, case, poison, seed, corrupt=False):
    d, A, B, C0 = build(case, poison, seed)
    guard = NAN16[case.dtype] if poison else SENTINEL
    tA, _ = _to_device(torch, A, case.off_a, guard)
    tB, _ = _to_device(torch, B, case.off_b, guard)
    tC, fullC = _to_device(torch, C0, case.off_c, guard)
    oa, ob, oc = GUARD + case.off_a, GUARD + case.off_b, GUARD + case.off_c
    dt = ac.DTYPE_BF16 if case.dtype == "bf16" else ac.DTYPE_F16
    pa, pb, pc = tA.data_ptr() + 2 * oa, tB.data_ptr() + 2 * ob, tC.data_ptr() + 2 * oc
    if case.impl:
        ctx.gemm_impl(case.impl, dt, d.layout_a, d.layout_b, d.M, d.N, d.K, d.alpha, pa, d.lda, d.stride_a, pb, d.ldb,
                      d.stride_b, d.beta, pc, d.ldc, d.stride_c, d.batch)
    else:
        ctx.gemm_strided_batched(d.layout_a, d.layout_b, d.M, d.N, d.K, d.alpha, pa, d.lda, d.stride_a, pb, d.ldb,
                                 d.stride_b, d.beta, pc, d.ldc, d.stride_c, d.batch, dt)
    ctx.synchronize()
    got_full = tC.cpu().numpy().view(np.uint16)
    outside = np.r_[0:oc, oc + C0.size:got_full.size]
    guards_ok = np.array_equal(got_full[outside], fullC[outside])
    out = got_full[oc:oc + C0.size].copy()
    c0 = C0 if d.beta != 0 else None
    ref = op.gemm_ref(d, A, B, c0)
    tol_ref = op.tolerance(d, A, B, c0, kind="reference")
    tol_ns = op.tolerance(d, A, B, c0, kind="north_star")
    if corrupt:
        corrupt_first(out, ref, tol_ref, case.dtype == "bf16")
    r_ref = op.compare(d, out, ref, C0, tol_ref)
    r_ns = op.compare(d, out, ref, C0, tol_ns)
    return r_ref["pass"] and r_ns["pass"] and guards_ok, (r_ref, r_ns), guards_ok


def _cases(mode):
    if ONLY is not None:
        return [int(ONLY)]
    return list(range(max(1, int(COUNTS[mode] * SCALE))))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["default", "decode", "large_k", "poison"])
def test_fuzz(cuda, mode):
    torch = cuda
    ctx = context(torch)
    impls = _impls(ctx)
    base_mode = "default" if mode == "poison" else mode
    seed = SEED + (1000 if mode == "poison" else 0)
    failures = []
    for i in _cases(mode):
        case = make_case(seed, i, impls, base_mode)
        ok, r, guards = run_case(torch, ctx, case, mode == "poison", seed)
        if not ok:
            failures.append(f"{case.describe()} -> guards_ok={guards} {r}")
    assert not failures, f"{len(failures)} failures (seed {seed}, mode {mode}):\n" + "\n".join(failures[:10])


@pytest.mark.gpu
def test_fuzz_corrupt_self_test(cuda):
    """--corrupt: every case, with one element pushed past the bound on the
    host copy, must be reported as a failure."""
    torch = cuda
    ctx = context(torch)
    impls = _impls(ctx)
    missed = []
    for i in range(max(1, int(24 * SCALE))):
        case = make_case(SEED + 2000, i, impls, "default")
        ok, _, _ = run_case(torch, ctx, case, False, SEED + 2000, corrupt=True)
        if ok:
            missed.append(case.describe())
    assert not missed, "corruption not caught:\n" + "\n".join(missed)
