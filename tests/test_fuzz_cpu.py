"""The fuzzer's generator and checker on CPU (no GPU): cases replay from
(seed, index) and cover the reference's case kinds, and the oracle-side check
passes an exact result, then fails it once one element is pushed past the
bound (the --corrupt self-test, planted in the host copy)."""
import numpy as np

import aegis_capi as ac
import oracle_py as op
from fuzz_cases import make_case
from test_fuzz_gpu import build, corrupt_first

IMPLS = [None, "umma_128x256x64_s4", "gemv_256x256_ksm", "simt_64x64x16"]


def test_cases_replay_and_cover_the_kinds():
    a = [make_case(1, i, IMPLS).describe() for i in range(300)]
    assert a == [make_case(1, i, IMPLS).describe() for i in range(300)]
    cs = [make_case(1, i, IMPLS) for i in range(300)]
    assert any(c.batch > 1 for c in cs) and any(c.off_a or c.off_b or c.off_c for c in cs)
    assert any(c.inject for c in cs) and any(c.beta == 0 for c in cs) and any(c.alpha == 0 for c in cs)
    assert any(c.layout_a == 1 for c in cs) and any(c.ldc > c.N for c in cs)
    assert {c.dtype for c in cs} == {"f16", "bf16"}
    assert all(c.M * c.N * c.K * c.batch <= 1 << 26 for c in cs)
    dec = [make_case(1, i, IMPLS, "decode") for i in range(100)]
    assert all(c.M <= 40 for c in dec) and max(c.K for c in dec) > 4096
    lk = [make_case(1, i, IMPLS, "large_k") for i in range(20)]
    assert all(14000 <= c.K <= 20000 and c.M <= 64 for c in lk)


def test_checker_passes_exact_and_catches_a_corrupted_element():
    tried = 0
    for i in range(60):
        case = make_case(3, i, IMPLS)
        if case.M * case.N * case.K * case.batch > 1 << 20 or case.inject:
            continue
        tried += 1
        d, A, B, C0 = build(case, poison=False, seed=3)
        c0 = C0 if d.beta != 0 else None
        ref = op.gemm_ref(d, A, B, c0)
        # The exact result rounded to the output type, in C's span (padding keeps C0).
        out = C0.copy()
        enc = ac.f32_to_16(ref.astype(np.float32).ravel(), case.dtype == "bf16").reshape(ref.shape)
        for bb in range(d.batch):
            for r in range(d.M):
                base = bb * d.stride_c + r * d.ldc
                out[base:base + d.N] = enc[bb, r]
        tol = op.tolerance(d, A, B, c0)
        assert op.compare(d, out, ref, C0, tol)["pass"], case.describe()
        assert op.compare(d, out, ref, C0, op.tolerance(d, A, B, c0, kind="north_star"))["pass"], case.describe()
        corrupt_first(out, ref, tol, case.dtype == "bf16")
        assert not op.compare(d, out, ref, C0, tol)["pass"], case.describe()
    assert tried >= 10
