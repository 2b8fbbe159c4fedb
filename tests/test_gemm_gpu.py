"""GEMM parity on the GPU through the C ABI, against the CPU oracle.

Covers the reference's correctness cases (tests/test_tma.cu, test_matmul.cu,
bench_gemm --check shapes in its CMakeLists.txt:202-212): every registry
kernel on the golden fixtures (outputs of the reference's own oracle), the
512^3 f16 workload (seed 0) and the square sweep (1024^3-8192^3, f16 and bf16,
sampled rows against the oracle plus the full matrix against cuBLAS), every
layout pair on the tcgen05 path, alpha/beta/batch, NaN/Inf, alpha == 0,
empty sizes, and misaligned operands (general kernel)."""
import os

import numpy as np
import pytest

import aegis_capi as ac
import oracle_py as op
from conftest import GOLDEN, golden_cases, load_golden
from gpu_util import check, context, dev, host, run

pytestmark = pytest.mark.gpu

IMPLS = ["umma_128x256x64_s4", "umma_128x128x64_s6", "umma_128x256x64_s4_ksm", "umma_128x128x64_s6_ksm",
         "umma_256x256x64_s7_c2", "umma_256x256x64_s7_c2_ksm", "umma_128x64x64_s8", "umma_128x64x64_s8_ksm",
         "umma_256x256x64_s7_c2_kw", "gemv_256x256_ksm", "gemv_128x256_ksm", "gemv_64x256_ksm", "gemv_32x256_ksm", "ummav_128x16x64_s11", "ummav_128x16x64_s6x2",
         "simt_64x64x16"]


def test_registry_all_supported(cuda):
    ctx = context(cuda)
    reg = ctx.registry()
    assert [e["name"] for e in reg] == IMPLS
    assert all(e["supported"] for e in reg), reg


@pytest.mark.parametrize("name", golden_cases())
@pytest.mark.parametrize("impl", [None] + IMPLS)
def test_golden(cuda, name, impl):
    d, A, B, C0, ref, _ = load_golden(name)
    ctx = context(cuda)
    dA, dB, dC = dev(cuda, A), dev(cuda, B), dev(cuda, C0)
    run(cuda, ctx, d, dA, dB, dC, impl)
    check(d, A, B, C0, host(dC), ref, f"{name} {impl}")


def test_config1_512_known_answers(cuda):
    d = op.make_desc(512, 512, 512)
    g = ac.Generator(0)
    A, B = g.uniform(512 * 512), g.uniform(512 * 512)
    z = np.load(os.path.join(GOLDEN, "config1_512.npz"))
    ctx = context(cuda)
    for impl in [None, "umma_128x256x64_s4", "umma_128x128x64_s6", "umma_256x256x64_s7_c2", "simt_64x64x16"]:
        dA, dB, dC = dev(cuda, A), dev(cuda, B), dev(cuda, np.zeros(512 * 512, np.uint16))
        run(cuda, ctx, d, dA, dB, dC, impl)
        out = host(dC)
        got = ac.to_f32(out, "f16").astype(np.float64)
        tol = float(z["ref_tol"])
        assert np.abs(got[z["sample_index"]] - z["sample"]).max() <= tol, impl
        check(d, A, B, None, out, op.gemm_ref(d, A, B), impl)


def _aligned_case(M, N, K, la, lb, alpha, beta, batch, dtype, seed):
    lda = (K if la == 0 else M) + 8
    ldb = (N if lb == 0 else K) + 16
    ldc = N + 3
    sa = lda * (M if la == 0 else K) + 64 if batch > 1 else 0
    sb = ldb * (K if lb == 0 else N) + 128 if batch > 1 else 0
    sc = ldc * M + 5 if batch > 1 else 0
    d = op.make_desc(M, N, K, la, lb, lda, ldb, ldc, alpha, beta, batch, sa, sb, sc, dtype)
    na, nb, nc = op.spans(d)
    g = ac.Generator(seed)
    return d, g.uniform(na, dtype), g.uniform(nb, dtype), g.uniform(nc, dtype)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("la,lb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("impl", ["umma_128x256x64_s4", "umma_128x128x64_s6", "umma_256x256x64_s7_c2",
                                  "umma_128x64x64_s8"])
def test_umma_layouts_alpha_beta_batch(cuda, dtype, la, lb, impl):
    """Operands the TMA path can address (16-byte aligned, ld % 8 == 0): the
    tcgen05 kernel with K-major and MN-major operands, edge tiles in M, N and K."""
    ctx = context(cuda)
    for (M, N, K, alpha, beta, batch) in [(300, 520, 200, 1.0, 0.0, 1), (129, 257, 1000, -0.5, 0.75, 2),
                                          (64, 64, 64, 2.0, 1.0, 1)]:
        d, A, B, C0 = _aligned_case(M, N, K, la, lb, alpha, beta, batch, dtype, seed=M + N + K)
        dA, dB, dC = dev(cuda, A), dev(cuda, B), dev(cuda, C0)
        run(cuda, ctx, d, dA, dB, dC, impl)
        check(d, A, B, C0, host(dC), op.gemm_ref(d, A, B, C0 if beta != 0 else None), f"{impl} {M}x{N}x{K}")


def _sample_rows(M):
    rows = sorted(set([0, 1, M // 2, M - 2, M - 1] + list(np.random.RandomState(M).choice(M, 11, replace=False))))
    return rows


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("n", [1024, 2048, 4096, 8192])
def test_square_sweep_config2(cuda, dtype, n):
    """Square sweep: C = A*B, M = N = K = n, uniform[-1, 1] from seed 0.
    Sampled rows against the FP64 oracle, the whole matrix against cuBLAS."""
    torch = cuda
    d = op.make_desc(n, n, n, dtype=dtype)
    g = ac.Generator(0)
    A, B = g.uniform(n * n, dtype), g.uniform(n * n, dtype)
    ctx = context(torch)
    dA, dB, dC = dev(torch, A), dev(torch, B), dev(torch, np.zeros(n * n, np.uint16))
    ctx.gemm(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), n, n, n, ac.DTYPE_BF16 if dtype == "bf16" else ac.DTYPE_F16)
    ctx.synchronize()
    assert ctx.choice(n, n, n).startswith("umma_")
    out = host(dC).reshape(n, n)
    tol = op.tolerance(d, A, B)
    rows = _sample_rows(n)
    sub = op.make_desc(len(rows), n, n, dtype=dtype)
    ref = op.gemm_ref(sub, A.reshape(n, n)[rows].ravel(), B)
    res = op.compare(sub, out[rows].ravel(), ref, None, tol)
    assert res["pass"], (rows, res)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    a = dA.view(tdt).view(n, n)
    b = dB.view(tdt).view(n, n)
    c_ref = (a @ b).float()
    c = dC.view(tdt).view(n, n).float()
    assert (c - c_ref).abs().max().item() <= 2 * tol


def test_nan_inf_alpha0_beta0_empty(cuda):
    torch = cuda
    ctx = context(torch)
    # beta == 0: C is not read (NaN in C stays out of the result).
    d = op.make_desc(130, 260, 70)
    g = ac.Generator(4)
    A, B = g.uniform(130 * 70), g.uniform(70 * 260)
    C0 = np.full(130 * 260, 0x7E00, np.uint16)
    for impl in [None, "umma_128x256x64_s4", "gemv_64x256_ksm", "simt_64x64x16"]:
        dA, dB, dC = dev(torch, A), dev(torch, B), dev(torch, C0)
        run(torch, ctx, d, dA, dB, dC, impl)
        out = host(dC)
        assert not np.isnan(ac.to_f32(out, "f16")).any(), impl
        check(d, A, B, None, out, op.gemm_ref(d, A, B), impl)
    # Empty sizes: nothing launched, C untouched.
    dC = dev(torch, C0)
    ctx.gemm(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), 0, 260, 70)
    ctx.gemm_ex(0, 0, 130, 260, 0, 1.0, dA.data_ptr(), 70, dB.data_ptr(), 260, 0.0, dC.data_ptr(), 260)
    ctx.synchronize()
    assert np.array_equal(host(dC), C0)


def test_misaligned_operands_take_the_general_kernel(cuda):
    torch = cuda
    ctx = context(torch)
    M, N, K = 77, 150, 99
    g = ac.Generator(8)
    A = g.uniform(M * K + 1)
    B = g.uniform(K * N + 1)
    dA, dB = dev(torch, A), dev(torch, B)
    dC = dev(torch, np.zeros(M * N + 1, np.uint16))
    # Offsets of one element: 2-byte aligned only.
    for impl in [None, "umma_128x256x64_s4_ksm"]:
        dt = ac.DTYPE_F16
        if impl:
            ctx.gemm_impl(impl, dt, 0, 0, M, N, K, 1.0, dA.data_ptr() + 2, K, 0, dB.data_ptr() + 2, N, 0, 0.0,
                          dC.data_ptr() + 2, N, 0, 1)
        else:
            ctx.gemm_ex(0, 0, M, N, K, 1.0, dA.data_ptr() + 2, K, dB.data_ptr() + 2, N, 0.0, dC.data_ptr() + 2, N)
        ctx.synchronize()
        d = op.make_desc(M, N, K)
        out = host(dC)[1:]
        check(d, A[1:], B[1:], None, out, op.gemm_ref(d, A[1:], B[1:]), str(impl))


def test_watchdog_selftest_and_context_reuse(cuda):
    torch = cuda
    ctx = context(torch)
    assert ctx.watchdog_selftest(20_000_000) == ac.AEGIS_OK
    ctx.synchronize()  # no pending watchdog bit from the self-test (it uses its own word)
    d = op.make_desc(256, 256, 256)
    g = ac.Generator(1)
    A, B = g.uniform(256 * 256), g.uniform(256 * 256)
    dA, dB, dC = dev(torch, A), dev(torch, B), dev(torch, np.zeros(256 * 256, np.uint16))
    run(torch, ctx, d, dA, dB, dC, "umma_128x256x64_s4")
    check(d, A, B, None, host(dC), op.gemm_ref(d, A, B))


def _winner_rows():
    """(M, N, K, impl) of every f16 row of the committed winners header (the
    type aegis_gemm_choice asks about)."""
    import re
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "aegis", "winners",
                        "sm_100a.h")
    if not os.path.exists(path):
        return []
    pat = re.compile(r'^\s*\{(\d+), (\d+), (\d+), "([^"]+)", aegis::detail::Dispatch::Aegis.*DType::F16\}')
    return [(int(m[1]), int(m[2]), int(m[3]), m[4]) for m in map(pat.match, open(path)) if m]


def test_dispatch_follows_the_tuned_winners(cuda):
    """aegis::matmul picks the tuned winner for every shape of the compiled
    header (exact match), and the nearest-M row for an untuned M of a tuned
    (N, K) (reference matmul.cu:432-467; ties go to the larger M)."""
    rows = _winner_rows()
    if not rows:
        pytest.skip("no winners header")
    ctx = context(cuda)
    for m, n, k, impl in rows:
        assert ctx.choice(m, n, k) == impl, (m, n, k)
    by_nk = {}
    for m, n, k, impl in rows:
        by_nk.setdefault((n, k), []).append((m, impl))
    import math
    for (n, k), ms in by_nk.items():
        for q in (2, 3, 8, 64, 3000):
            if any(m == q for m, _ in ms):
                continue
            best = min(ms, key=lambda r: (abs(math.log2(r[0]) - math.log2(q)), -r[0]))
            assert ctx.choice(q, n, k) == best[1], (q, n, k)
