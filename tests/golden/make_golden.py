"""Generates tests/golden/*.npz from the reference's OWN oracle.

Runs aegis::bench::cpu_reference and aegis::bench::tolerance of the reference
(Riffe007/aegis-core src/bench/reference.cu:69-105, 186-194), compiled where
it lies by oracle/Makefile into oracle/_ref/libaegis_ref.so, on seeded inputs
from libaegis_datagen.so (std::mt19937 + uniform_real_distribution<float>,
as the reference's harness draws them, src/bench/harness.cu:48-54).

Run from the repository root after `make -C oracle` and `make -C aegis-core_b200`:
    python tests/golden/make_golden.py
The fixtures pin oracle/oracle.c (tests/test_oracle.py) and give the GPU
parity tests reference outputs that need no reference tree at run time.
"""
import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), "..", ".."))
sys.path.insert(0, os.path.join(ROOT, "aegis-core_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import aegis_capi as ac  # noqa: E402
import oracle_py as op  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))

# (name, M, N, K, layout_a, layout_b, pad, alpha, beta, batch, seed, inject)
CASES = [
    ("rr_127x129x65", 127, 129, 65, 0, 0, 0, 1.0, 0.0, 1, 42, None),      # reference ctest shape
    ("rr_200x136x72", 200, 136, 72, 0, 0, 0, 1.0, 0.0, 1, 42, None),      # reference ctest shape
    ("rr_1x896x896", 1, 896, 896, 0, 0, 0, 1.0, 0.0, 1, 42, None),        # decode
    ("rr_16x512x896", 16, 512, 896, 0, 0, 0, 1.0, 0.0, 1, 42, None),      # decode (N cut to keep the file small)
    ("cr_13x100x411_ab", 13, 100, 411, 1, 0, 3, -0.5, 0.75, 1, 7, None),
    ("rc_5x33x205_batch3", 5, 33, 205, 0, 1, 1, 2.0, 1.0, 3, 7, None),
    ("cc_9x13x777_beta", 9, 13, 777, 1, 1, 0, 1.0, -1.0, 1, 11, None),
    ("rr_37x60x131_half", 37, 60, 131, 0, 0, 5, 1.0, 0.5, 1, 11, None),
    ("rr_16x16x16_naninf", 16, 16, 16, 0, 0, 0, 1.0, 0.0, 1, 3, "naninf"),
    ("rr_8x8x8_alpha0_nan", 8, 8, 8, 0, 0, 0, 0.0, 0.5, 1, 3, "alpha0"),
]


def make_case(M, N, K, la, lb, pad, alpha, beta, batch, seed, inject):
    lda = (K if la == 0 else M) + pad
    ldb = (N if lb == 0 else K) + pad
    ldc = N + pad
    sa = sb = sc = 0
    if batch > 1:
        sa = lda * (M if la == 0 else K) + 8
        sb = ldb * (K if lb == 0 else N) + 8
        sc = ldc * M
    d = op.make_desc(M, N, K, la, lb, lda, ldb, ldc, alpha, beta, batch, sa, sb, sc, "f16")
    na, nb, nc = op.spans(d)
    g = ac.Generator(seed)
    A = g.uniform(na)
    B = g.uniform(nb)
    C0 = g.uniform(nc)
    if inject == "naninf":
        A[3 * lda + 2] = 0x7E00  # NaN in row 3
        B[4 * ldb + 5] = 0x7C00  # +Inf in column 5
        B[6 * ldb + 9] = 0xFC00  # -Inf in column 9
    if inject == "alpha0":
        A[0] = 0x7E00            # NaN in A: must not reach C when alpha == 0
    return d, A, B, C0


def main():
    if not op.ref_available():
        sys.exit("oracle/_ref/libaegis_ref.so is missing: build it with `make -C oracle` where the reference tree is")
    for case in CASES:
        name = case[0]
        d, A, B, C0 = make_case(*case[1:])
        ref = op.ref_cpu_reference(d, A, B, C0 if d.beta != 0 else None)
        tol = op.ref_tolerance(d, A, B, C0 if d.beta != 0 else None)
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), desc=np.array(
            [d.M, d.N, d.K, d.layout_a, d.layout_b, d.lda, d.ldb, d.ldc, d.batch, d.stride_a, d.stride_b,
             d.stride_c], dtype=np.int64), alpha_beta=np.array([d.alpha, d.beta], dtype=np.float32),
            A=A, B=B, C0=C0, ref=ref, ref_tol=np.array(tol))
        print(f"{name}: ref sum {np.nansum(ref[np.isfinite(ref)]):.6f} tol {tol:.6g}")
    # Config 1 (M = N = K = 512, seed 0, A then B): a summary and a fixed sample
    # of the reference's output (the full 2 MiB of doubles is not stored).
    d = op.make_desc(512, 512, 512)
    g = ac.Generator(0)
    A = g.uniform(512 * 512)
    B = g.uniform(512 * 512)
    ref = op.ref_cpu_reference(d, A, B)[0]
    idx = np.random.RandomState(1).choice(512 * 512, 4096, replace=False)
    idx.sort()
    np.savez_compressed(os.path.join(OUT, "config1_512.npz"), sample_index=idx, sample=ref.ravel()[idx],
                        summary=np.array([ref[0, 0], ref[0, 1], ref[511, 511], ref.sum(), (ref * ref).sum(),
                                          np.abs(ref).max()]), a0=A[0], b0=B[0],
                        ref_tol=np.array(op.ref_tolerance(d, A, B)))
    print("config1_512:", ref[0, 0], ref[0, 1], ref[511, 511], ref.sum(), (ref * ref).sum(), np.abs(ref).max(),
          hex(int(A[0])), hex(int(B[0])))


if __name__ == "__main__":
    main()
