"""Decode GEMV parity (the decode workload): M in {1, 4, 16}, activations
~N(0, 1), f16 weights ~N(0, 0.02) of K x N in {4096x4096, 4096x14336,
14336x4096}, std::mt19937 + std::normal_distribution<float> on the host;
every gemv configuration and the dispatcher, against the FP64 oracle with
both tolerance forms, bitwise identical across runs (deterministic split-K);
plus edge cases: N not a multiple of 8, K tails, column-major or misaligned
weights (element loads), batch, alpha/beta."""
import numpy as np
import pytest

import aegis_capi as ac
import oracle_py as op
from gpu_util import check, context, dev, host, run

pytestmark = pytest.mark.gpu

GEMV = ["gemv_256x256_ksm", "gemv_128x256_ksm", "gemv_64x256_ksm", "gemv_32x256_ksm", "ummav_128x16x64_s11", "ummav_128x16x64_s6x2"]
SHAPES = [(4096, 4096), (4096, 14336), (14336, 4096)]


def decode_inputs(M, K, N, seed=3):
    g = ac.Generator(seed)
    return g.normal(M * K, "f16", 0.0, 1.0), g.normal(K * N, "f16", 0.0, 0.02)


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("M", [1, 4, 16])
def test_config3(cuda, M, K, N):
    torch = cuda
    A, B = decode_inputs(M, K, N)
    d = op.make_desc(M, N, K)
    ref = op.gemm_ref(d, A, B)
    ctx = context(torch)
    # The dispatcher's pick: the tuned winner of this shape (a decode or a
    # split-K tensor-core kernel), checked like every other kernel below.
    assert ctx.choice(M, N, K) in {e["name"] for e in ctx.registry()}
    dA, dB = dev(torch, A), dev(torch, B)
    for impl in [None] + GEMV:
        outs = []
        for _ in range(3):
            dC = dev(torch, np.zeros(M * N, np.uint16))
            run(torch, ctx, d, dA, dB, dC, impl)
            outs.append(host(dC))
        assert all(np.array_equal(o, outs[0]) for o in outs), impl
        check(d, A, B, None, outs[0], ref, f"{impl} M={M} {K}x{N}")


@pytest.mark.parametrize("impl", GEMV)
def test_gemv_edges(cuda, impl):
    torch = cuda
    ctx = context(torch)
    for (M, N, K, la, lb, pad, alpha, beta, batch) in [(3, 1001, 777, 0, 0, 0, 1.0, 0.0, 1),
                                                       (16, 100, 4099, 1, 0, 8, -0.5, 0.75, 1),
                                                       (5, 333, 2053, 0, 1, 1, 2.0, 1.0, 2),
                                                       (9, 136, 7777, 1, 1, 0, 1.0, -1.0, 1),
                                                       (20, 64, 512, 0, 0, 3, 1.0, 0.5, 3)]:
        lda = (K if la == 0 else M) + pad
        ldb = (N if lb == 0 else K) + pad
        ldc = N + pad
        sa = lda * (M if la == 0 else K) if batch > 1 else 0
        sb = ldb * (K if lb == 0 else N) if batch > 1 else 0
        sc = ldc * M if batch > 1 else 0
        d = op.make_desc(M, N, K, la, lb, lda, ldb, ldc, alpha, beta, batch, sa, sb, sc)
        na, nb, nc = op.spans(d)
        g = ac.Generator(N + K)
        A, B, C0 = g.uniform(na), g.uniform(nb), g.uniform(nc)
        dA, dB, dC = dev(torch, A), dev(torch, B), dev(torch, C0)
        run(torch, ctx, d, dA, dB, dC, impl)
        check(d, A, B, C0, host(dC), op.gemm_ref(d, A, B, C0 if beta != 0 else None), f"{impl} {M}x{N}x{K}")


def test_gemv_bf16(cuda):
    torch = cuda
    ctx = context(torch)
    M, K, N = 4, 4096, 4096
    g = ac.Generator(11)
    A, B = g.normal(M * K, "bf16", 0, 1), g.normal(K * N, "bf16", 0, 0.02)
    d = op.make_desc(M, N, K, dtype="bf16")
    for impl in [None] + GEMV:
        dA, dB, dC = dev(torch, A), dev(torch, B), dev(torch, np.zeros(M * N, np.uint16))
        run(torch, ctx, d, dA, dB, dC, impl)
        check(d, A, B, None, host(dC), op.gemm_ref(d, A, B), str(impl))


# (impl, M, N, K, splits per tile): gemv plans of 2, 4 and 8 splits (the
# cluster split-K fix-up, every cluster size) and tile-aligned ummav grids of
# 2, 4 and 8 segments per tile (ordered tickets), with beta on half of them.
CLUSTER_CASES = [
    ("ummav_128x16x64_s6x2", 1, 14336, 4096, 2),
    ("ummav_128x16x64_s6x2", 3, 9472, 2048, 4),
    ("ummav_128x16x64_s6x2", 16, 4736, 4096, 8),
    ("ummav_128x16x64_s11", 5, 4736, 2048, 4),
    ("ummav_128x16x64_s11", 1, 2304, 8192, 8),
    ("gemv_64x256_ksm", 1, 4096, 4096, 8),
    ("gemv_64x256_ksm", 2, 9472, 2048, 4),
    ("gemv_128x256_ksm", 1, 37888, 1024, 2),
]


@pytest.mark.parametrize("impl,M,N,K,s", CLUSTER_CASES)
def test_cluster_fixup(cuda, impl, M, N, K, s):
    """Split fix-ups at s = 2, 4, 8 splits per tile (gemv: inside a
    thread-block cluster; ummav: grid = tiles x s, ordered tickets): results
    bitwise repeatable and within the oracle's bounds, with and without beta."""
    torch = cuda
    ctx = context(torch)
    p = ctx.plan(M, N, K, impl, ac.DTYPE_F16)
    if impl.startswith("ummav"):  # its plan reports a bound on segments per tile; the grid shows s
        assert p["grid"] == p["tiles"] * s, p
    else:
        assert p["splits"] == s, p
    beta = 0.5 if (M + s) % 2 else 0.0
    d = op.make_desc(M, N, K, 0, 0, K, N, N, 1.5, beta, 1, 0, 0, 0, "f16")
    g = ac.Generator(M * 7 + s)
    A, B, C0 = g.uniform(M * K), g.uniform(K * N), g.uniform(M * N)
    dA, dB = dev(torch, A), dev(torch, B)
    outs = []
    for _ in range(2):
        dC = dev(torch, C0)
        run(torch, ctx, d, dA, dB, dC, impl)
        outs.append(host(dC))
    assert np.array_equal(outs[0], outs[1]), impl
    check(d, A, B, C0, outs[0], op.gemm_ref(d, A, B, C0 if beta != 0 else None), f"{impl} {M}x{N}x{K} s={s}")
