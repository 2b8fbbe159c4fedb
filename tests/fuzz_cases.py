"""Case generator of the GEMM fuzzer (tests/test_fuzz_gpu.py).

The reference's tools/aegis_fuzz.cu:1-58 draws, per case:
- an implementation;
- M, N, K (primes, tiny, multiples of 8, log-uniform);
- layouts, padded leading dimensions and misaligned pointers;
- alpha and beta from a fixed set or uniform;
- strided batches;
- data at three scales, with NaN/Inf injected into a few cases.

Every case checks against the FP64 reference. This module draws the same kinds of cases
with its own generator: case i of seed s comes from numpy's PCG64 seeded with (s, i), so a
failure replays alone from (seed, case). It does not reproduce the reference's
mt19937_64 stream.

Modes (the reference's flags):
- default;
- decode: M in 1..16 (85%) or 17..40, K up to 16384;
- large_k: K in 14000..20000, M 1..64, every product long;
- poison: NaN in every element outside the logical matrices, plus NaN guards around each
  allocation. It must pass: no kernel may read past K, M or N into a product, and
  beta == 0 must not read C.

Sizes are capped so the FP64 reference (the C oracle, multi-threaded) runs in
milliseconds to a fraction of a second per case.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

MAX_DIM = 4096
DECODE_MAX_K = 16384
LARGE_K = (14000, 20000)
GUARD = 64  # elements before and after every device allocation


def _primes_upto(n):
    sieve = np.ones(n + 1, dtype=bool)
    sieve[:2] = False
    for p in range(2, int(n ** 0.5) + 1):
        if sieve[p]:
            sieve[p * p::p] = False
    return np.nonzero(sieve)[0]


_PRIMES = {}


def primes(n):
    if n not in _PRIMES:
        _PRIMES[n] = _primes_upto(n)
    return _PRIMES[n]


def draw_dim(rng, hi):
    u = rng.random()
    if u < 0.30:
        ps = primes(hi)
        return int(ps[rng.integers(len(ps))])
    if u < 0.55:
        return int(rng.integers(1, min(64, hi) + 1))
    if u < 0.75:
        return int(8 * rng.integers(1, max(1, hi // 8) + 1))
    return int(min(hi, max(1, round(math.exp(rng.uniform(0.0, math.log(hi)))))))


@dataclasses.dataclass
class Case:
    index: int
    impl: str | None  # None: aegis::matmul's dispatcher
    dtype: str
    M: int
    N: int
    K: int
    layout_a: int
    layout_b: int
    lda: int
    ldb: int
    ldc: int
    batch: int
    stride_a: int
    stride_b: int
    stride_c: int
    off_a: int
    off_b: int
    off_c: int
    alpha: float
    beta: float
    scale: float
    inject: list  # (operand, row, col, value)

    def describe(self):
        return (f"case {self.index}: {self.impl or 'matmul'} {self.dtype} {self.M}x{self.N}x{self.K} "
                f"layouts {'RC'[self.layout_a]}{'RC'[self.layout_b]} ld {self.lda}/{self.ldb}/{self.ldc} "
                f"batch {self.batch} strides {self.stride_a}/{self.stride_b}/{self.stride_c} "
                f"offsets {self.off_a}/{self.off_b}/{self.off_c} alpha {self.alpha:g} beta {self.beta:g} "
                f"scale {self.scale:g} inject {len(self.inject)}")


def _one_span(rows, cols, row_major, ld):
    return (rows - 1) * ld + cols if row_major else (cols - 1) * ld + rows


def make_case(seed, i, impls, mode="default"):
    rng = np.random.default_rng([seed, i])
    impl = impls[rng.integers(len(impls))]
    dtype = "bf16" if rng.random() < 0.5 else "f16"
    if mode == "large_k":
        if rng.random() < 0.4:
            ps = primes(LARGE_K[1])
            ps = ps[np.searchsorted(ps, LARGE_K[0]):]
            K = int(ps[rng.integers(len(ps))])
        else:
            K = int(rng.integers(LARGE_K[0], LARGE_K[1] + 1))
        M = int(rng.integers(1, 65))
        N = draw_dim(rng, MAX_DIM)
        while M * N * K > (1 << 30):
            N = max(1, N // 2)
    elif mode == "decode":
        M = int(rng.integers(1, 17)) if rng.random() < 0.85 else int(rng.integers(17, 41))
        K = draw_dim(rng, DECODE_MAX_K)
        N = draw_dim(rng, MAX_DIM)
        while N * K > (1 << 24):
            N = max(1, N // 2)
    else:
        M, N, K = draw_dim(rng, MAX_DIM), draw_dim(rng, MAX_DIM), draw_dim(rng, MAX_DIM)
        while M * N * K > (1 << 26):
            big = max(("M", M), ("N", N), ("K", K), key=lambda t: t[1])[0]
            if big == "M":
                M = max(1, M // 2)
            elif big == "N":
                N = max(1, N // 2)
            else:
                K = max(1, K // 2)
    la, lb = int(rng.integers(2)), int(rng.integers(2))

    def pad():
        return int(rng.integers(1, 18)) if rng.random() < 0.5 else 0

    lda = (K if la == 0 else M) + pad()
    ldb = (N if lb == 0 else K) + pad()
    ldc = N + pad()
    batch, sa, sb, sc = 1, 0, 0, 0
    if rng.random() < 0.15 and mode != "large_k":
        batch = int(rng.integers(2, 5))
        sa = _one_span(M, K, la == 0, lda) + int(rng.integers(0, 65))
        sb = _one_span(K, N, lb == 0, ldb) + int(rng.integers(0, 65))
        sc = _one_span(M, N, True, ldc) + int(rng.integers(0, 65))
        while M * N * K * batch > (1 << 26) and batch > 1:
            batch -= 1

    def off():
        return int(rng.integers(1, 8)) if rng.random() < 0.2 else 0

    alphas = [1.0, 0.0, -1.0, 0.5, -2.25]
    betas = [0.0, 1.0, -1.0, 0.5]
    a_pick = int(rng.integers(len(alphas) + 1))
    alpha = alphas[a_pick] if a_pick < len(alphas) else float(rng.uniform(-3, 3))
    b_pick = int(rng.integers(len(betas) + 1))
    beta = betas[b_pick] if b_pick < len(betas) else float(rng.uniform(-2, 2))
    scale = float([1.0, 0.25, 4.0][rng.integers(3)])
    inject = []
    if rng.random() < 0.05 and mode != "large_k":
        for _ in range(int(rng.integers(1, 4))):
            which = "A" if rng.random() < 0.5 else "B"
            val = [np.nan, np.inf, -np.inf][rng.integers(3)]
            r = int(rng.integers(M if which == "A" else K))
            c = int(rng.integers(K if which == "A" else N))
            inject.append((which, r, c, val))
    return Case(i, impl, dtype, M, N, K, la, lb, lda, ldb, ldc, batch, sa, sb, sc, off(), off(), off(), alpha,
                beta, scale, inject)
