"""aegis_gemv_noalloc: the decode GEMV for callers that cannot allocate.

Some callers cannot let a library call cudaMalloc: inference engines that
give all device memory to their own allocator at start-up and forbid later
allocations, code running while a CUDA graph is being captured, processes on
a hard device-memory budget. The regular entry points take split-K scratch
from a per-stream cache that allocates on a stream's first use;
aegis_gemv_noalloc runs the same kernel with its scratch in a fixed array
inside the library. These tests call it through the C ABI and check that its
output matches the regular entry point's (aegis_gemm_*_ex) within the
tolerance the other tests use, on two calls in a row (the second call finds
the array as the first one left it), and that the calls allocate nothing.
The one planning step that differs from the regular entry point (fewer,
longer K splits when the partials would overflow the array) is reached only
on devices with several hundred SMs; tests/test_plan_cpu.py checks it on a
modelled device.
This file is collected last on purpose; it passes alone or after the rest.
"""
import numpy as np
import pytest

import aegis_capi as ac
import oracle_py as op
from gpu_util import context, dev, host

pytestmark = pytest.mark.gpu

CASES = [  # M, K, N, dtype, layout_a, layout_b, pad, alpha, beta
    (1, 4096, 4096, "f16", 0, 0, 0, 1.0, 0.0),
    (4, 4096, 14336, "f16", 0, 0, 0, 1.0, 0.0),
    (16, 14336, 4096, "f16", 0, 0, 0, 1.0, 0.0),
    (7, 2053, 333, "bf16", 1, 0, 8, -0.5, 0.75),
    (3, 777, 1001, "f16", 0, 1, 3, 2.0, 1.0),
]


@pytest.mark.parametrize("case", CASES)
def test_matches_regular_entry_point_twice(cuda, case):
    torch = cuda
    M, K, N, dtype, la, lb, pad, alpha, beta = case
    lda = (K if la == 0 else M) + pad
    ldb = (N if lb == 0 else K) + pad
    ldc = N + pad
    d = op.make_desc(M, N, K, la, lb, lda, ldb, ldc, alpha, beta, 1, 0, 0, 0, dtype)
    na, nb, nc = op.spans(d)
    g = ac.Generator(M * 1000 + N)
    A, B, C0 = g.normal(na, dtype, 0, 1), g.normal(nb, dtype, 0, 0.02), g.normal(nc, dtype, 0, 1)
    code = ac.DTYPE_BF16 if dtype == "bf16" else ac.DTYPE_F16
    ctx = context(torch)
    dA, dB = dev(torch, A), dev(torch, B)
    # The regular entry point (per-stream workspace).
    dC = dev(torch, C0)
    ctx.gemm_ex(la, lb, M, N, K, alpha, dA.data_ptr(), lda, dB.data_ptr(), ldb, beta, dC.data_ptr(), ldc, code)
    ctx.synchronize()
    regular = host(dC)
    tol = op.tolerance(d, A, B, C0 if beta != 0 else None)  # the reference's bound, as every parity test uses
    ref = op.gemm_ref(d, A, B, C0 if beta != 0 else None)
    for call in range(2):
        dC = dev(torch, C0)
        ctx.gemv_noalloc(code, la, lb, M, N, K, alpha, dA.data_ptr(), lda, dB.data_ptr(), ldb, beta, dC.data_ptr(),
                         ldc)
        ctx.synchronize()
        out = host(dC)
        diff = np.abs(ac.to_f32(out, dtype).astype(np.float64) - ac.to_f32(regular, dtype).astype(np.float64))
        assert np.nanmax(diff) <= tol, f"call {call}: max |noalloc - regular| {np.nanmax(diff)} > {tol}"
        r = op.compare(d, out, ref, C0, tol)
        assert r["pass"], (call, r)


def test_rejects_problems_beyond_its_limits(cuda):
    torch = cuda
    ctx = context(torch)
    buf = torch.zeros(1 << 20, dtype=torch.int16, device="cuda")
    p = buf.data_ptr()
    for (M, N, K) in [(17, 64, 64), (1, 65537, 8)]:
        with pytest.raises(ac.AegisError) as e:
            ctx.gemv_noalloc(ac.DTYPE_F16, 0, 0, M, N, K, 1.0, p, K, p, N, 0.0, p, N)
        assert e.value.status == ac.AEGIS_ERR_INVALID_ARGUMENT
        assert "M <= 16" in e.value.detail  # the reason names the limit
    ctx.synchronize()  # the context stays usable


def test_calls_allocate_no_device_memory(cuda):
    torch = cuda
    M, K, N = 1, 4096, 4096
    g = ac.Generator(77)
    A, B = g.normal(M * K, "f16", 0, 1), g.normal(K * N, "f16", 0, 0.02)
    ctx = context(torch)
    dA, dB, dC = dev(torch, A), dev(torch, B), dev(torch, np.zeros(M * N, np.uint16))
    assert ctx.plan(M, N, K, "gemv_256x256_ksm")["splits"] > 1  # the split-K scratch is in use
    # First call on this device: looks up the fixed array's address (may load the module).
    ctx.gemv_noalloc(ac.DTYPE_F16, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), N, 0.0, dC.data_ptr(), N)
    ctx.synchronize()
    first = host(dC)
    s = torch.cuda.Stream()  # a stream the per-stream workspace cache has never seen
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    with torch.cuda.stream(s):
        ctx.set_stream(s.cuda_stream)
        for _ in range(3):
            ctx.gemv_noalloc(ac.DTYPE_F16, 0, 0, M, N, K, 1.0, dA.data_ptr(), K, dB.data_ptr(), N, 0.0,
                             dC.data_ptr(), N)
        ctx.synchronize()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert np.array_equal(host(dC), first)  # deterministic across calls
