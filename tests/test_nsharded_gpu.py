"""N-sharded GEMM with the all-gather fused into the epilogue.

On one GPU every rank is emulated in turn: rank r's call computes its column
shard and stores it into every "rank's" C (all local buffers here, peers'
IPC-mapped memory on a multi-GPU node). Each C must then equal the 1-GPU
GEMM bit for bit (the per-element K order does not depend on the column
offset). Nothing waits on anything: each emulated rank is one ordinary
launch. The multi-process NVLink run is tests/test_nsharded_multigpu.py."""
import numpy as np
import pytest

import aegis_capi as ac
from gpu_util import context, dev, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nranks", [1, 2, 4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_emulated_ranks_match_single_gpu_bitwise(cuda, nranks, dtype):
    torch = cuda
    M, N, K = 512, 2048, 1024
    code = ac.DTYPE_BF16 if dtype == "bf16" else ac.DTYPE_F16
    g = ac.Generator(16384)
    A, B = g.uniform(M * K, dtype), g.uniform(K * N, dtype)
    ctx = context(torch)
    dA, dB = dev(torch, A), dev(torch, B)
    full = dev(torch, np.zeros(M * N, np.uint16))
    ctx.gemm(dA.data_ptr(), dB.data_ptr(), full.data_ptr(), M, N, K, code)
    ctx.synchronize()
    want = host(full)
    ns = N // nranks
    Bm = B.reshape(K, N)
    shards = [dev(torch, np.ascontiguousarray(Bm[:, r * ns:(r + 1) * ns])) for r in range(nranks)]
    cs = [dev(torch, np.full(M * N, 0x7E00, np.uint16)) for _ in range(nranks)]
    for r in range(nranks):
        ctx.nsharded(M, N, K, dA.data_ptr(), K, shards[r].data_ptr(), ns, [c.data_ptr() for c in cs], N, nranks, r,
                     code)
    ctx.synchronize()
    for r in range(nranks):
        assert np.array_equal(host(cs[r]), want), f"rank {r} of {nranks}"


def test_argument_checks(cuda):
    torch = cuda
    ctx = context(torch)
    buf = torch.zeros(1024, dtype=torch.int16, device="cuda")
    p = buf.data_ptr()
    with pytest.raises(ac.AegisError):
        ctx.nsharded(16, 30, 16, p, 16, p, 10, [p, p, p, p], 30, 4, 0)   # N % nranks != 0
    with pytest.raises(ac.AegisError):
        ctx.nsharded(16, 32, 16, p, 16, p, 8, [p, p], 16, 2, 0)          # ldc < N
    with pytest.raises(ac.AegisError):
        ctx.nsharded(16, 32, 16, p, 16, p, 8, [p, p], 32, 2, 2)          # rank out of range


@pytest.mark.parametrize("nranks", [2, 4])
def test_emulated_ranks_ragged_tiles_and_padded_ldc(cuda, nranks):
    """Partial tiles in M and in the shard's columns (ns = 208 at 4 ranks, 416 at
    2) and an odd padded ldc: the peer copy takes its element-wise path, and
    C's padding columns stay untouched."""
    torch = cuda
    M, N, K, pad = 300, 832, 264, 3
    ldc = N + pad
    g = ac.Generator(77)
    A, B = g.uniform(M * K, "bf16"), g.uniform(K * N, "bf16")
    ctx = context(torch)
    dA, dB = dev(torch, A), dev(torch, B)
    full = dev(torch, np.zeros(M * N, np.uint16))
    ctx.gemm(dA.data_ptr(), dB.data_ptr(), full.data_ptr(), M, N, K, ac.DTYPE_BF16)
    ctx.synchronize()
    want = host(full).reshape(M, N)
    ns = N // nranks
    Bm = B.reshape(K, N)
    shards = [dev(torch, np.ascontiguousarray(Bm[:, r * ns:(r + 1) * ns])) for r in range(nranks)]
    cs = [dev(torch, np.full(M * ldc, 0x7FC0, np.uint16)) for _ in range(nranks)]
    for r in range(nranks):
        ctx.nsharded(M, N, K, dA.data_ptr(), K, shards[r].data_ptr(), ns, [c.data_ptr() for c in cs], ldc, nranks,
                     r, ac.DTYPE_BF16)
    ctx.synchronize()
    for r in range(nranks):
        got = host(cs[r]).reshape(M, ldc)
        assert np.array_equal(got[:, :N], want), f"rank {r} of {nranks}"
        assert (got[:, N:] == 0x7FC0).all(), "padding columns written"


def test_headline_16384_against_the_oracle_and_emulated_ranks(cuda):
    """The bench's headline workload at its full size: C = A*B, M = N = K =
    16384, bf16, uniform[-1, 1] from std::mt19937(0), A then B. The 1-rank
    call's C is checked on 16 sampled rows (0, M-1 and seeded random rows)
    against the FP64 oracle under both bounds, the size switch of the
    reference's fuzzer (tools/aegis_fuzz.cu:448); then 8 emulated ranks each
    store their column shard into all 8 C buffers (4 GiB), and every one must
    equal the 1-rank result bit for bit (compared on the device)."""
    import oracle_py as op
    from gpu_util import check
    torch = cuda
    n = 16384
    g = ac.Generator(0)
    A, B = g.uniform(n * n, "bf16"), g.uniform(n * n, "bf16")
    ctx = context(torch)
    dA, dB = dev(torch, A), dev(torch, B)
    one = torch.full((n * n,), 0x7FC0, dtype=torch.int16, device="cuda")
    ctx.nsharded(n, n, n, dA.data_ptr(), n, dB.data_ptr(), n, [one.data_ptr()], n, 1, 0, ac.DTYPE_BF16)
    ctx.synchronize()
    rows = sorted({0, n - 1} | set(int(x) for x in np.random.RandomState(20261202).choice(n, 14, replace=False)))
    got = host(one.view(n, n)[rows].contiguous()).reshape(-1)
    A_s = np.ascontiguousarray(A.reshape(n, n)[rows]).reshape(-1)
    d = op.make_desc(len(rows), n, n, dtype="bf16")
    check(d, A_s, B, None, got, op.gemm_ref(d, A_s, B), name="16384^3 sampled rows")

    P = 8
    ns = n // P
    Bm = B.reshape(n, n)
    cs = [torch.full((n * n,), 0x7E00, dtype=torch.int16, device="cuda") for _ in range(P)]
    for r in range(P):
        shard = dev(torch, np.ascontiguousarray(Bm[:, r * ns:(r + 1) * ns]))
        ctx.nsharded(n, n, n, dA.data_ptr(), n, shard.data_ptr(), ns, [c.data_ptr() for c in cs], n, P, r,
                     ac.DTYPE_BF16)
        ctx.synchronize()
        del shard
    for r in range(P):
        assert torch.equal(cs[r], one), f"emulated rank {r} of {P}"
