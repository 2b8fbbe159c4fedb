"""Helpers for the GPU tests: device buffers from uint16 host arrays (torch is
only the allocator), a C-ABI context bound to torch's current stream, and
oracle comparisons with both tolerance forms the project uses:
  - the reference's bound c*sqrt(K)*eps*max|A|*max|B|*|alpha| + eps*|beta|*max|C0|
    (c = 2, src/bench/reference.cu:186-194), and
  - the north-star bound eps*K*max|A|*max|B|*|alpha| (+ the beta term), eps = 2^-10
    for f16 outputs as stated, 2^-7 for bf16 outputs."""
import numpy as np

import aegis_capi as ac
import oracle_py as op


def dev(torch, host_u16):
    return torch.from_numpy(np.ascontiguousarray(host_u16, dtype=np.uint16).view(np.int16)).cuda()


def host(t):
    return t.cpu().numpy().view(np.uint16)


def context(torch):
    ctx = ac.Context(torch.cuda.current_device())
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    return ctx


def dtype_code(name):
    return ac.DTYPE_BF16 if name == "bf16" else ac.DTYPE_F16


def run(torch, ctx, d, dA, dB, dC, impl=None):
    """One GEMM described by oracle Desc `d` through the C ABI (dispatcher, or a named registry kernel)."""
    dt = ac.DTYPE_BF16 if d.dtype == 1 else ac.DTYPE_F16
    if impl:
        ctx.gemm_impl(impl, dt, d.layout_a, d.layout_b, d.M, d.N, d.K, d.alpha, dA.data_ptr(), d.lda, d.stride_a,
                      dB.data_ptr(), d.ldb, d.stride_b, d.beta, dC.data_ptr(), d.ldc, d.stride_c, d.batch)
    else:
        ctx.gemm_strided_batched(d.layout_a, d.layout_b, d.M, d.N, d.K, d.alpha, dA.data_ptr(), d.lda, d.stride_a,
                                 dB.data_ptr(), d.ldb, d.stride_b, d.beta, dC.data_ptr(), d.ldc, d.stride_c, d.batch,
                                 dt)
    ctx.synchronize()


def check(d, A, B, C0, out, ref, name=""):
    """Both tolerance forms; returns the comparison under the reference's bound."""
    c0 = C0 if d.beta != 0 else None
    tol_ref = op.tolerance(d, A, B, c0, kind="reference")
    tol_ns = op.tolerance(d, A, B, c0, kind="north_star")
    r = op.compare(d, out, ref, C0, tol_ref)
    assert r["pass"], f"{name}: {r}"
    assert op.compare(d, out, ref, C0, tol_ns)["pass"]
    return r
