"""The oracle (oracle/oracle.c) pinned against the reference's own outputs.

- Known answers of the reference's aegis::bench::cpu_reference on BASELINE
  512^3 f16 workload (M = N = K = 512, std::mt19937(0), uniform[-1, 1], A then B).
- Golden fixtures written by tests/golden/make_golden.py from the reference's
  own oracle (compiled from its source into oracle/_ref): layouts, padded
  leading dimensions, alpha/beta, strided batch, NaN/Inf, alpha == 0.
- When oracle/_ref is built here, fresh seeded cases against it, bit for bit.
- The comparer's NaN/Inf/padding rules, with mistakes planted on the CPU.
"""
import os

import numpy as np
import pytest

import aegis_capi as ac
import oracle_py as op
from conftest import GOLDEN, golden_cases, load_golden


def test_known_answers_config1():
    d = op.make_desc(512, 512, 512)
    g = ac.Generator(0)
    A = g.uniform(512 * 512)
    B = g.uniform(512 * 512)
    assert int(A[0]) == 0x2E40 and int(B[0]) == 0xAF0B
    C = op.gemm_ref(d, A, B)[0]
    # Values the reference's own cpu_reference printed for this problem.
    assert C[0, 0] == pytest.approx(4.95359320863, abs=1e-10)
    assert C[0, 1] == pytest.approx(-9.85570906356, abs=1e-10)
    assert C[511, 511] == pytest.approx(-11.8105152465, abs=1e-10)
    assert C.sum() == pytest.approx(-978.485808516, abs=1e-8)
    assert (C * C).sum() == pytest.approx(14869180.3291, abs=1e-3)
    assert np.abs(C).max() == pytest.approx(34.9640666416, abs=1e-10)
    z = np.load(os.path.join(GOLDEN, "config1_512.npz"))
    assert np.array_equal(C.ravel()[z["sample_index"]], z["sample"])  # bit for bit
    assert op.tolerance(d, A, B) == pytest.approx(float(z["ref_tol"]), rel=1e-15)
    assert op.tolerance(d, A, B, kind="north_star") == pytest.approx(2.0 ** -10 * 512 * np.abs(
        ac.to_f32(A, "f16")).max() * np.abs(ac.to_f32(B, "f16")).max(), rel=1e-12)


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_golden(name):
    d, A, B, C0, ref, ref_tol = load_golden(name)
    got = op.gemm_ref(d, A, B, C0 if d.beta != 0 else None)
    assert np.array_equal(got, ref, equal_nan=True), name
    assert op.tolerance(d, A, B, C0 if d.beta != 0 else None) == pytest.approx(ref_tol, rel=1e-15)


def _random_case(rng, dtype="f16"):
    M, N, K = (int(x) for x in rng.randint(1, 70, 3))
    la, lb = (int(x) for x in rng.randint(0, 2, 2))
    pad = int(rng.randint(0, 4))
    batch = int(rng.randint(1, 4))
    alpha = float(rng.choice([1.0, -0.5, 2.0, 0.0]))
    beta = float(rng.choice([0.0, 1.0, 0.25]))
    lda = (K if la == 0 else M) + pad
    ldb = (N if lb == 0 else K) + pad
    ldc = N + pad
    sa = lda * (M if la == 0 else K) + int(rng.randint(0, 3)) if batch > 1 else 0
    sb = ldb * (K if lb == 0 else N) + int(rng.randint(0, 3)) if batch > 1 else 0
    sc = ldc * M if batch > 1 else 0
    d = op.make_desc(M, N, K, la, lb, lda, ldb, ldc, alpha, beta, batch, sa, sb, sc, dtype)
    na, nb, nc = op.spans(d)
    g = ac.Generator(int(rng.randint(0, 1 << 30)))
    return d, g.uniform(na, dtype), g.uniform(nb, dtype), g.uniform(nc, dtype)


@pytest.mark.skipif(not op.ref_available(), reason="oracle/_ref (the reference's own oracle) not built here")
def test_oracle_matches_reference_live():
    rng = np.random.RandomState(20261201)
    for _ in range(40):
        d, A, B, C0 = _random_case(rng)
        c0 = C0 if d.beta != 0 else None
        assert np.array_equal(op.gemm_ref(d, A, B, c0), op.ref_cpu_reference(d, A, B, c0), equal_nan=True)
        assert op.tolerance(d, A, B, c0) == pytest.approx(op.ref_tolerance(d, A, B, c0), rel=1e-15)
    # Above the reference's 1e7-MAC threading threshold: still bit-identical.
    d = op.make_desc(300, 200, 300)
    g = ac.Generator(5)
    A, B = g.uniform(300 * 300), g.uniform(300 * 200)
    assert np.array_equal(op.gemm_ref(d, A, B, nthreads=8), op.ref_cpu_reference(d, A, B))


def test_oracle_bf16_decode_and_sum():
    # bf16 has no reference implementation: check the decode and one sum against numpy in float64.
    rng = np.random.RandomState(3)
    d, A, B, C0 = _random_case(rng, "bf16")
    d.batch, d.beta, d.alpha = 1, 0.0, 1.0
    Af = ac.to_f32(A, "bf16").astype(np.float64)
    Bf = ac.to_f32(B, "bf16").astype(np.float64)
    a = np.array([[Af[(i * d.lda + k) if d.layout_a == 0 else (i + k * d.lda)] for k in range(d.K)]
                  for i in range(d.M)])
    b = np.array([[Bf[(k * d.ldb + j) if d.layout_b == 0 else (k + j * d.ldb)] for j in range(d.N)]
                  for k in range(d.K)])
    got = op.gemm_ref(d, A, B)[0]
    assert np.allclose(got, a @ b, rtol=1e-12, atol=1e-12)


def test_compare_semantics_planted_mistakes():
    d, A, B, C0, ref, tol = load_golden("rr_37x60x131_half")
    # A correct answer: the reference rounded to f16, padding copied from C0.
    out = C0.copy()
    for i in range(d.M):
        out[i * d.ldc: i * d.ldc + d.N] = ac.f32_to_16(ref[0, i].astype(np.float32), False)
    assert op.compare(d, out, ref, C0, tol)["pass"]
    bad = out.copy()  # one element off by 2 * tol
    bad[5 * d.ldc + 7] = ac.f32_to_16(np.float32(ref[0, 5, 7] + 2 * tol), False)
    r = op.compare(d, bad, ref, C0, tol)
    assert not r["pass"] and r["out_of_tol"] == 1 and r["first_index"] == 5 * d.ldc + 7
    bad = out.copy()  # a NaN where the reference is finite
    bad[3] = 0x7E00
    assert not op.compare(d, bad, ref, C0, tol)["pass"]
    bad = out.copy()  # a padding column written
    bad[d.N] ^= 1
    assert not op.compare(d, bad, ref, C0, tol)["pass"]


def test_compare_nan_inf_rules():
    d, A, B, C0, ref, tol = load_golden("rr_16x16x16_naninf")
    assert np.isnan(ref[0, 3]).all()                # NaN in A row 3 poisons the row
    assert np.isinf(ref[0][[0, 1, 2], 5]).all()     # Inf in B column 5 (sign of A[i, 4])
    out = ac.f32_to_16(ref[0].astype(np.float32), False).ravel()
    assert op.compare(d, out, ref, None, tol)["pass"]
    bad = out.copy()
    bad[0 * 16 + 5] ^= 0x8000                        # the Inf with the wrong sign
    assert op.compare(d, bad, ref, None, tol)["inf_mismatch"] == 1


def test_alpha_zero_golden_ignores_nan():
    d, A, B, C0, ref, tol = load_golden("rr_8x8x8_alpha0_nan")
    assert np.isfinite(ref).all()
    assert np.allclose(ref[0], 0.5 * ac.to_f32(C0, "f16").reshape(8, 8))


def test_datagen_conversions_match_numpy_and_torch():
    rng = np.random.RandomState(0)
    x = np.concatenate([rng.uniform(-1, 1, 200000), rng.uniform(-1, 1, 50000) * 1e-4,
                        rng.uniform(-1, 1, 50000) * 1e-7, [65504, 65519.99, 65520, 1e6, -1e6, 0.0, -0.0,
                                                         2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26]]).astype(np.float32)
    with np.errstate(over="ignore"):
        assert np.array_equal(ac.f32_to_16(x, False), x.astype(np.float16).view(np.uint16))
    import torch
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ac.f32_to_16(x, True), want)


def test_datagen_normal_distribution():
    g = ac.Generator(123)
    w = ac.to_f32(g.normal(1 << 20, "f16", 0.0, 0.02), "f16")
    assert abs(w.mean()) < 1e-3 and abs(w.std() - 0.02) < 1e-3
    g1, g2 = ac.Generator(9), ac.Generator(9)
    assert np.array_equal(g1.uniform(1000), g2.uniform(1000))


def test_north_star_bound_scales_with_the_output_type():
    """The north-star bound eps*K*max|A|*max|B| uses the output type's eps:
    2^-10 for f16 (as stated) and 2^-7 for bf16, whose rounding alone can
    exceed 2^-10*K*max|A|*max|B| at small K."""
    g = ac.Generator(5)
    for dtype, eps in (("f16", 2.0 ** -10), ("bf16", 2.0 ** -7)):
        A, B = g.uniform(4 * 3, dtype, -4, 4), g.uniform(3 * 5, dtype, -4, 4)
        d = op.make_desc(4, 5, 3, dtype=dtype)
        ma, mb = np.abs(ac.to_f32(A, dtype)).max(), np.abs(ac.to_f32(B, dtype)).max()
        assert op.tolerance(d, A, B, kind="north_star") == pytest.approx(eps * 3 * ma * mb, rel=1e-12)
