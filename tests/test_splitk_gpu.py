"""Deterministic split-K on the GPU (the tall-K workload, M = N in {256, 512,
1024} x K = 65536, and the reference's
tests/test_splitk.cu pattern): tall-K shapes split by the SM count, 10 runs
bitwise identical, within tolerance of the FP64 oracle; odd split counts and
K tails; general layouts with beta; the first call for a stream inside CUDA
graph capture is refused without breaking the capture; later calls capture
and replay bit-identically."""
import numpy as np
import pytest

import aegis_capi as ac
import oracle_py as op
from gpu_util import check, context, dev, host, run

pytestmark = pytest.mark.gpu

SPLIT_IMPLS = ["umma_128x256x64_s4_ksm", "umma_128x128x64_s6_ksm", "umma_256x256x64_s7_c2_ksm",
               "umma_128x64x64_s8_ksm"]


@pytest.mark.parametrize("mn", [256, 512, 1024])
def test_config4_tall_k_bitwise_and_oracle(cuda, mn):
    torch = cuda
    K = 65536
    d = op.make_desc(mn, mn, K, dtype="bf16")
    g = ac.Generator(4)
    A, B = g.uniform(mn * K, "bf16"), g.uniform(K * mn, "bf16")
    ctx = context(torch)
    dA, dB = dev(torch, A), dev(torch, B)
    for impl in [None] + SPLIT_IMPLS:
        plan = ctx.plan(mn, mn, K, impl, ac.DTYPE_BF16)
        # Split-K is chosen when the tiles cannot fill the SMs (148 on B200);
        # 128 x 64 tiles already make 128 tiles at 1024^2.
        assert plan["splits"] > 1 or plan["tiles"] >= 74, plan
        first = None
        for _ in range(10):
            dC = dev(torch, np.zeros(mn * mn, np.uint16))
            run(torch, ctx, d, dA, dB, dC, impl)
            out = host(dC)
            if first is None:
                first = out
            else:
                assert np.array_equal(out, first), f"{impl}: run differs from run 0"
        rows = sorted(set([0, mn // 3, mn - 1] + list(np.random.RandomState(mn).choice(mn, 13, replace=False))))
        sub = op.make_desc(len(rows), mn, K, dtype="bf16")
        ref = op.gemm_ref(sub, A.reshape(mn, K)[rows].ravel(), B)
        tol = op.tolerance(d, A, B)
        res = op.compare(sub, first.reshape(mn, mn)[rows].ravel(), ref, None, tol)
        assert res["pass"], (impl, res)
        assert op.compare(sub, first.reshape(mn, mn)[rows].ravel(), ref, None,
                          op.tolerance(d, A, B, kind="north_star"))["pass"]


@pytest.mark.parametrize("shape", [(300, 200, 30001, 0, 0, 1.0, 0.0), (129, 136, 7777, 1, 0, -0.5, 0.75),
                                   (64, 520, 20480, 0, 1, 2.0, 1.0), (9, 1000, 4099, 1, 1, 1.0, -1.0)])
@pytest.mark.parametrize("impl", SPLIT_IMPLS)
def test_split_shapes_layouts(cuda, shape, impl):
    torch = cuda
    M, N, K, la, lb, alpha, beta = shape
    lda = (K if la == 0 else M) + 8
    ldb = (N if lb == 0 else K) + 8
    ldc = N + 1
    d = op.make_desc(M, N, K, la, lb, lda, ldb, ldc, alpha, beta, 1, 0, 0, 0, "f16")
    na, nb, nc = op.spans(d)
    g = ac.Generator(M + N)
    A, B, C0 = g.uniform(na), g.uniform(nb), g.uniform(nc)
    ctx = context(torch)
    dA, dB = dev(torch, A), dev(torch, B)
    outs = []
    for _ in range(3):
        dC = dev(torch, C0)
        run(torch, ctx, d, dA, dB, dC, impl)
        outs.append(host(dC))
    assert all(np.array_equal(o, outs[0]) for o in outs)
    check(d, A, B, C0, outs[0], op.gemm_ref(d, A, B, C0 if beta != 0 else None), f"{impl} {shape}")


@pytest.mark.parametrize("shape", [(256, 256, 20480, 0.0), (200, 262, 20480, 0.5)])
@pytest.mark.parametrize("impl", ["umma_128x128x64_s6_ksm", "umma_256x256x64_s7_c2_ksm"])
def test_forced_split_counts(cuda, monkeypatch, shape, impl):
    """Every slot-group count of the reduce (1, 2, 4, 8 groups; the last group
    short; more than 8 slots per group past S = 64), float4 and scalar columns
    (N % 4 == 0 and N = 262), with beta: bitwise repeatable and within the
    oracle's tolerance. AEGIS_UMMA_SPLITS sets the split count."""
    torch = cuda
    M, N, K, beta = shape
    d = op.make_desc(M, N, K, 0, 0, K, N, N, 1.0, beta, 1, 0, 0, 0, "bf16")
    g = ac.Generator(M + N + K)
    A, B, C0 = g.uniform(M * K, "bf16"), g.uniform(K * N, "bf16"), g.uniform(M * N, "bf16")
    ctx = context(torch)
    dA, dB = dev(torch, A), dev(torch, B)
    ref = op.gemm_ref(d, A, B, C0 if beta != 0 else None)
    # 320 k-blocks: each count is ceil(320 / ceil(320 / S)), so the plan keeps it.
    for S in [2, 7, 9, 16, 17, 40, 64, 80]:
        monkeypatch.setenv("AEGIS_UMMA_SPLITS", str(S))
        assert ctx.plan(M, N, K, impl, ac.DTYPE_BF16)["splits"] == S
        outs = []
        for _ in range(2):
            dC = dev(torch, C0)
            run(torch, ctx, d, dA, dB, dC, impl)
            outs.append(host(dC))
        assert np.array_equal(outs[0], outs[1]), (impl, S)
        check(d, A, B, C0, outs[0], ref, f"{impl} S={S} {shape}")


def test_odd_split_counts_occur(cuda):
    ctx = context(cuda)
    counts = {ctx.plan(m, n, k, impl)["splits"] for impl in SPLIT_IMPLS
              for (m, n, k) in [(256, 256, 65536), (512, 512, 65536), (300, 200, 30001), (129, 136, 7777),
                                (1024, 1024, 65536)]}
    assert any(s > 1 and s % 2 == 1 for s in counts), counts


def test_graph_capture_after_first_call(cuda):
    """Workspace contract (reference workspace.h): after one direct call per
    (stream, size class), calls capture in a CUDA graph with no allocation
    and replay bit-identically; a first call inside capture is refused."""
    torch = cuda
    M = N = 256
    K = 16384
    g = ac.Generator(2)
    A, B = g.uniform(M * K, "bf16"), g.uniform(K * N, "bf16")
    d = op.make_desc(M, N, K, dtype="bf16")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ctx = context(torch)
        dA, dB, dC = dev(torch, A), dev(torch, B), dev(torch, np.zeros(M * N, np.uint16))
        run(torch, ctx, d, dA, dB, dC, "umma_128x256x64_s4_ksm")
        direct = host(dC)
        dC.zero_()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            ctx.set_stream(torch.cuda.current_stream().cuda_stream)
            ctx.gemm_impl("umma_128x256x64_s4_ksm", ac.DTYPE_BF16, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, 0,
                          dB.data_ptr(), N, 0, 0.0, dC.data_ptr(), N, 0, 1)
        graph.replay()
        torch.cuda.synchronize()
        assert np.array_equal(host(dC), direct)
    # A fresh stream's first split-K call inside capture: refused, capture intact.
    s2 = torch.cuda.Stream()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s2):
        ctx2 = context(torch)
        with torch.cuda.graph(g2, stream=s2):
            ctx2.set_stream(torch.cuda.current_stream().cuda_stream)
            with pytest.raises(ac.AegisError) as e:
                ctx2.gemm_impl("umma_128x256x64_s4_ksm", ac.DTYPE_BF16, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, 0,
                               dB.data_ptr(), N, 0, 0.0, dC.data_ptr(), N, 0, 1)
            assert e.value.status == ac.AEGIS_ERR_CUDA

