"""torch.ops.aegis.matmul on the GPU: equal to an FP32 torch reference within
the north-star bound (eps*K*max|A|*max|B|, eps of the output type) for row-
and column-major operands, decode and square shapes, f16 and bf16; ordered on
torch's current stream with no explicit synchronisation."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("M,N,K,ta,tb", [(512, 384, 256, False, False), (300, 520, 264, True, False),
                                         (256, 256, 1024, False, True), (1, 4096, 4096, False, False),
                                         (16, 1000, 777, True, True)])
def test_matches_fp32_reference(cuda, dtype, M, N, K, ta, tb):
    torch = cuda
    import aegis_torch  # noqa: F401  (registers the op)
    dt = getattr(torch, dtype)
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    a = torch.rand((K, M) if ta else (M, K), generator=g, device="cuda", dtype=torch.float32).mul_(2).sub_(1).to(dt)
    b = torch.rand((N, K) if tb else (K, N), generator=g, device="cuda", dtype=torch.float32).mul_(2).sub_(1).to(dt)
    a = a.t() if ta else a
    b = b.t() if tb else b
    c = torch.ops.aegis.matmul(a, b)
    ref = a.float() @ b.float()
    eps = 2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -10
    tol = eps * K * a.float().abs().max().item() * b.float().abs().max().item()
    assert c.shape == (M, N) and c.dtype == dt
    assert (c.float() - ref).abs().max().item() <= tol


def test_stream_ordering_without_sync(cuda):
    torch = cuda
    import aegis_torch  # noqa: F401
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = torch.ones(256, 512, device="cuda", dtype=torch.bfloat16)
        b = torch.full((512, 128), 0.5, device="cuda", dtype=torch.bfloat16)
        c = torch.ops.aegis.matmul(a, b)
        total = c.float().sum()  # consumes c on the same stream
    s.synchronize()
    assert total.item() == 256 * 128 * 256.0
