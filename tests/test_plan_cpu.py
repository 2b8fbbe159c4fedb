"""Dispatch rules and launch plans on a simulated B200, without a GPU
(aegis_plan_simulated_json).

The reference tests its dispatcher on its device (tests/test_matmul.cu); here
the same host logic runs against a simulated device profile:
  - every row of the tuned winners header is chosen for its exact shape;
  - other M with a tuned (N, K) take the nearest M in log2, ties to the larger
    M (reference src/matmul.cu:432-467, include/aegis/matmul.h:8-45);
  - untuned (N, K) fall back to the built-in rule (decode / TMA-addressable /
    general kernel), and no winners row is used on a device that is not sm_100;
  - GEMV plans stay one wave of resident CTAs, split-K plans cover K with no
    empty split, ummav plans fit the SMs, all as functions of the SM count.
"""
import math
import os
import re

import pytest

import aegis_capi as ac
from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "aegis", "winners", "sm_100a.h")
BF16 = ac.DTYPE_BF16


def winner_rows(dtype="bf16"):
    """(M, N, K, impl) of the header's rows tuned on `dtype`."""
    rows = []
    for line in open(HEADER):
        m = re.match(r'\s*\{(\d+), (\d+), (\d+), "([^"]+)".*DType::(BF16|F16)\}', line)
        if m and m.group(5).lower() == dtype:
            rows.append((int(m.group(1)), int(m.group(2)), int(m.group(3)), m.group(4)))
    return rows


def plan(M, N, K, impl=None, sms=148, arch=100, dtype=BF16):
    return ac.plan_simulated(M, N, K, impl=impl, dtype=dtype, arch=arch, sm_count=sms)


def test_header_has_rows():
    assert len(winner_rows("bf16")) >= 17 and len(winner_rows("f16")) >= 17


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_winner_rows_are_chosen_for_their_shape_and_type(dtype):
    code = BF16 if dtype == "bf16" else ac.DTYPE_F16
    for M, N, K, impl in winner_rows(dtype):
        p = plan(M, N, K, dtype=code)
        assert p["kind"] == "winner" and p["dispatch"] == impl and p["impl"] == impl, (dtype, M, N, K, p)


def test_rows_of_the_other_type_serve_an_untuned_type():
    """(N, K) tuned in only one type: a call of the other type takes that
    type's rows (nearest M), not the built-in rule. Checked on every bf16 (N, K)
    with no f16 row, else vacuously."""
    f16_nk = {(n, k) for (_, n, k, _) in winner_rows("f16")}
    for (M, N, K, impl) in winner_rows("bf16"):
        if (N, K) not in f16_nk:
            p = plan(M, N, K, dtype=ac.DTYPE_F16)
            assert p["kind"] == "winner" and p["dispatch"] == impl


def nearest(rows, M, N, K):
    """The nearest-M rule restated: same (N, K), smallest |log2 M' - log2 M|
    (an exact M first), ties to the larger M'."""
    best = None
    for (m, n, k, impl) in rows:
        if (n, k) != (N, K):
            continue
        d = -1.0 if m == M else abs(math.log2(m) - math.log2(M))
        if best is None or d < best[0] or (d == best[0] and m > best[1]):
            best = (d, m, impl)
    return best[2] if best else None


@pytest.mark.parametrize("M", [2, 3, 6, 8, 12, 24, 64, 200, 1000, 3000, 6000, 12000])
def test_nearest_m_for_tuned_n_k(M):
    rows = winner_rows()
    for (N, K) in sorted({(n, k) for (_, n, k, _) in rows}):
        want = nearest(rows, M, N, K)
        p = plan(M, N, K)
        assert p["kind"] == "winner" and p["dispatch"] == want, (M, N, K, p)


@pytest.mark.parametrize("shape,kernel", [
    ((1, 1000, 3000), "gemv_256x256_ksm"),            # M <= 2: CUDA-core weight stream
    ((2, 1000, 3000), "gemv_256x256_ksm"),
    ((3, 1000, 3000), "ummav_128x16x64_s6x2"),        # 2 < M <= 8, TMA-addressable
    ((8, 1000, 3000), "ummav_128x16x64_s6x2"),
    ((9, 1000, 3000), "umma_128x128x64_s6_ksm"),      # 8 < M <= 16: split-K 128 x 128 tiles
    ((16, 1000, 3000), "umma_128x128x64_s6_ksm"),
    ((8, 1001, 3000), "gemv_128x256_ksm"),            # ldb not a multiple of 8: no TMA
    ((12, 1001, 3000), "gemv_64x256_ksm"),
    ((2000, 120, 3000), "umma_128x128x64_s6_ksm"),    # N <= 128
    ((100, 2000, 3000), "umma_128x256x64_s4_ksm"),    # M <= 128
    ((600, 600, 600), "umma_128x64x64_s8_ksm"),       # one wave of 128 x 64 tiles, short K
    ((1000, 1000, 4096), "umma_128x64x64_s8_ksm"),
    ((384, 384, 40000), "umma_128x128x64_s6_ksm"),    # < 12 tiles of 256 x 256, long K
    ((1000, 1000, 40000), "umma_256x256x64_s7_c2_ksm"),
    ((2000, 2000, 3000), "umma_256x256x64_s7_c2_ksm"),
    ((1536, 1536, 1536), "umma_256x256x64_s7_c2_ksm"),
    ((2000, 2001, 3000), "simt_64x64x16"),            # not TMA-addressable
])
def test_built_in_rule_for_untuned_shapes(shape, kernel):
    p = plan(*shape)
    assert p["kind"] == "rule" and p["dispatch"] == kernel, (shape, p)


def test_rule_follows_the_sm_count():
    # 50 tiles of 128 x 64 are one wave on 148 SMs but not on 16.
    assert plan(600, 600, 600)["dispatch"] == "umma_128x64x64_s8_ksm"
    assert plan(600, 600, 600, sms=16)["dispatch"] == "umma_256x256x64_s7_c2_ksm"


def test_no_winner_rows_off_sm100():
    for (M, N, K, _) in winner_rows():
        p = plan(M, N, K, arch=90)
        assert p["kind"] == "rule", p
        if M > 16:
            assert p["dispatch"] == "simt_64x64x16", p


DECODE = [(m, n, k) for m in (1, 2, 4, 8, 16) for (n, k) in ((4096, 4096), (14336, 4096), (4096, 14336))]
GEMV_CTAS_PER_SM = {1: 4, 2: 4, 4: 4, 8: 2, 16: 1}  # by row tile MT (gemv.cu gemv_ctas_per_sm)


@pytest.mark.parametrize("sms", [148, 132, 74])
@pytest.mark.parametrize("impl", ["gemv_256x256_ksm", "gemv_128x256_ksm", "gemv_64x256_ksm", "gemv_32x256_ksm"])
def test_gemv_plans_are_one_wave(impl, sms):
    bn = int(impl.split("_")[1].split("x")[0])
    for (M, N, K) in DECODE:
        mt = 1
        while mt < M and mt < 16 and mt < 1024 // bn:
            mt *= 2
        p = plan(M, N, K, impl, sms=sms)
        assert p["grid"] <= GEMV_CTAS_PER_SM[mt] * sms or p["splits"] == 1, (M, N, K, sms, p)
        assert (p["splits"] - 1) * p["k_chunk"] < K <= p["splits"] * p["k_chunk"], (M, N, K, p)


SPLIT_IMPLS = {"umma_128x256x64_s4_ksm": 1, "umma_128x128x64_s6_ksm": 1, "umma_256x256x64_s7_c2_ksm": 2,
               "umma_128x64x64_s8_ksm": 1}
TALL_K = [(256, 256, 65536), (512, 512, 65536), (1024, 1024, 65536), (300, 200, 30001), (129, 136, 7777),
          (16, 4096, 14336), (1, 14336, 4096)]


@pytest.mark.parametrize("sms", [148, 74])
@pytest.mark.parametrize("impl", list(SPLIT_IMPLS))
def test_split_k_plans_cover_k_without_empty_splits(impl, sms):
    ctas = SPLIT_IMPLS[impl]
    for (M, N, K) in TALL_K:
        p = plan(M, N, K, impl, sms=sms)
        assert p == plan(M, N, K, impl, sms=sms)  # a pure function of shape and device
        S, kc = p["splits"], p["k_chunk"]
        assert S >= 1 and (S == 1 or kc % 64 == 0), p
        assert (S - 1) * kc < K <= S * kc, (M, N, K, p)
        assert p["grid"] == p["tiles"] * S * ctas, p


def test_tall_k_shapes_split_when_tiles_cannot_fill_the_sms():
    for (M, N, K) in [(256, 256, 65536), (512, 512, 65536)]:
        for impl, ctas in SPLIT_IMPLS.items():
            p = plan(M, N, K, impl)
            assert p["splits"] > 1, (M, N, K, p)


def test_unsplit_configs_never_split():
    for impl in ["umma_128x256x64_s4", "umma_128x128x64_s6", "umma_256x256x64_s7_c2", "umma_128x64x64_s8"]:
        for (M, N, K) in TALL_K:
            assert plan(M, N, K, impl)["splits"] == 1


@pytest.mark.parametrize("sms", [148, 132])
@pytest.mark.parametrize("impl,per_sm", [("ummav_128x16x64_s11", 1), ("ummav_128x16x64_s6x2", 2)])
def test_ummav_plans_fit_the_sms(impl, per_sm, sms):
    """Grids stay within the resident slots and the k-block count (so no CTA
    has an empty range: the segment and ticket accounting counts every CTA
    between a tile's first and last owner); when whole-tile splits fill 3/4
    of the slots, the grid is tiles x s, so no tile is cut unevenly."""
    for (M, N, K) in DECODE + [(1, 896, 896), (3, 640, 192), (1, 128, 64)]:
        p = plan(M, N, K, impl, sms=sms)
        kb = math.ceil(K / 64)
        tiles = math.ceil(N / 128)
        slots = per_sm * sms
        assert p["tiles"] == tiles, p
        assert 1 <= p["grid"] <= min(slots, tiles * kb), p
        s = min(slots // tiles, kb) if tiles <= slots else 0
        if s >= 1 and 4 * tiles * s >= 3 * slots:
            assert p["grid"] == tiles * s, p


MAX_DIM = (1 << 31) - (1 << 20)  # gemm::kMaxDim
FAMILIES = ["umma_128x256x64_s4", "umma_128x128x64_s6", "umma_128x256x64_s4_ksm", "umma_128x128x64_s6_ksm",
            "umma_256x256x64_s7_c2", "umma_256x256x64_s7_c2_ksm", "umma_128x64x64_s8", "umma_128x64x64_s8_ksm",
            "umma_256x256x64_s7_c2_kw", "gemv_256x256_ksm", "gemv_128x256_ksm", "gemv_64x256_ksm", "gemv_32x256_ksm", "ummav_128x16x64_s11",
            "ummav_128x16x64_s6x2"]


def test_random_plans_keep_their_invariants():
    """Seeded random shapes up to the size limit, every planner and SM count:
    positive tiles and grids below 2^32, and for the umma and gemv families
    K chunks that cover K with no empty split (no 32-bit overflow anywhere)."""
    import random
    rnd = random.Random(20261202)
    sizes = [1, 2, 3, 15, 16, 17, 64, 65, 100, 1000, 4096, 14336, 65536, 1 << 20, MAX_DIM - 1, MAX_DIM]
    for _ in range(3000):
        M, N, K = [rnd.choice(sizes + [rnd.randint(1, 1 << 24), rnd.randint(1, MAX_DIM)]) for _ in range(3)]
        impl = rnd.choice(FAMILIES + [None])
        p = plan(M, N, K, impl, sms=rnd.choice([148, 132, 74, 16, 1]))
        if p["impl"].startswith("simt"):
            continue  # the general kernel has no split plan
        assert p["splits"] >= 1 and p["tiles"] >= 1 and 1 <= p["grid"] < 2 ** 32, (M, N, K, p)
        if p["impl"].startswith(("umma_", "gemv_")):
            S, kc = p["splits"], p["k_chunk"]
            assert 0 < kc <= K and (S - 1) * kc < K <= S * kc, (M, N, K, p)


def test_sizes_above_the_limit_are_refused():
    for shape in [(MAX_DIM + 1, 8, 8), (8, MAX_DIM + 1, 8), (8, 8, (1 << 31) - 1)]:
        with pytest.raises(ac.AegisError) as e:
            ac.plan_simulated(*shape)
        assert e.value.status == ac.AEGIS_ERR_INVALID_ARGUMENT
    assert plan(MAX_DIM, 8, 8)["tiles"] >= 1


def test_arguments_are_checked():
    for bad in [dict(M=0, N=8, K=8), dict(M=8, N=-1, K=8)]:
        with pytest.raises(ac.AegisError) as e:
            ac.plan_simulated(**bad)
        assert e.value.status == ac.AEGIS_ERR_INVALID_ARGUMENT
    with pytest.raises(ac.AegisError):
        ac.plan_simulated(8, 8, 8, impl="no_such_kernel")
    with pytest.raises(ac.AegisError):
        ac.plan_simulated(8, 8, 8, sm_count=0)
    with pytest.raises(ac.AegisError):
        ac.plan_simulated(8, 8, 8, dtype=7)


NOALLOC_PARTIAL_BYTES = 4 << 20  # the fixed partials array of aegis_gemv_noalloc


def _noalloc_cfg(M):
    """(impl, BN, MT) of the CUDA-core GEMV config aegis_gemv_noalloc runs for M."""
    impl, bn = ("gemv_256x256_ksm", 256) if M <= 4 else (("gemv_128x256_ksm", 128) if M <= 8 else
                                                         ("gemv_64x256_ksm", 64))
    mt = 1
    while mt < M and mt < 16 and mt < 1024 // bn:
        mt *= 2
    return impl, bn, mt


@pytest.mark.parametrize("sms", [148, 592, 2048, 4096])
@pytest.mark.parametrize("M", [1, 4, 8, 16])
@pytest.mark.parametrize("N,K", [(4096, 4096), (14336, 4096), (4096, 14336), (65536, 65536), (512, 131072)])
def test_noalloc_plan_fits_the_fixed_array(sms, M, N, K):
    """The allocation-free GEMV keeps the regular plan while its FP32 partials
    fit the 4 MiB array, and otherwise re-splits K into fewer, longer chunks
    that still cover K with no empty split. On 148 SMs the regular plan always
    fits; the many-SM devices force the re-split branch."""
    impl, bn, mt = _noalloc_cfg(M)
    got = plan(M, N, K, impl="gemv_noalloc", sms=sms)
    reg = plan(M, N, K, impl=impl, sms=sms)
    assert got["tiles"] == reg["tiles"]
    slot = got["tiles"] * mt * bn * 4  # one split's partials: tiles x MT x BN floats
    S, kc = got["splits"], got["k_chunk"]
    assert kc % 16 == 0 or kc == K
    assert S == math.ceil(K / kc) and (S - 1) * kc < K <= S * kc
    if S > 1:
        assert S * slot <= NOALLOC_PARTIAL_BYTES
    if reg["splits"] * slot <= NOALLOC_PARTIAL_BYTES:
        assert (S, kc) == (reg["splits"], reg["k_chunk"])
    else:
        assert S < reg["splits"]


def test_noalloc_plan_re_splits_on_a_many_sm_device():
    """At least one shape takes the fewer-splits branch on a 4096-SM device,
    and none does on a B200's 148 SMs."""
    shapes = [(M, N, K) for M in (1, 4, 8, 16) for N, K in ((4096, 4096), (14336, 4096), (4096, 14336))]
    def re_split(sms):
        out = []
        for M, N, K in shapes:
            impl = _noalloc_cfg(M)[0]
            if plan(M, N, K, impl="gemv_noalloc", sms=sms)["splits"] != plan(M, N, K, impl=impl, sms=sms)["splits"]:
                out.append((M, N, K))
        return out
    assert re_split(148) == []
    assert len(re_split(4096)) > 0


def test_noalloc_plan_refuses_out_of_limit_shapes():
    with pytest.raises(ac.AegisError):
        plan(17, 4096, 4096, impl="gemv_noalloc")
    with pytest.raises(ac.AegisError):
        plan(1, 65537, 4096, impl="gemv_noalloc")


@pytest.mark.parametrize("shape", [(16384, 16384, 16384), (8192, 8192, 8192), (1024, 1024, 65536), (512, 512, 512),
                                   (16384, 2048, 16384), (300, 70000, 1000)])
def test_k_walk_by_wave_only_on_unsplit_multi_wave_launches(shape):
    """The _kw pair config walks K by wave (74 resident pairs on 148 SMs) when
    the launch is unsplit and has more than one wave of tiles; everything else
    walks K forward."""
    kw = plan(*shape, impl="umma_256x256x64_s7_c2_kw")
    fw = plan(*shape, impl="umma_256x256x64_s7_c2")
    assert (kw["splits"], kw["tiles"], kw["grid"]) == (fw["splits"], fw["tiles"], fw["grid"])
    assert fw["kdir_wave"] == 0
    assert kw["kdir_wave"] == (74 if kw["splits"] == 1 and kw["tiles"] > 74 else 0), kw
    for impl in ["umma_128x256x64_s4", "umma_128x128x64_s6_ksm", "umma_256x256x64_s7_c2_ksm", "umma_128x64x64_s8"]:
        assert plan(*shape, impl=impl)["kdir_wave"] == 0


def test_gemv_nine_splits_become_eight_at_small_m():
    """The cluster split-K fix-up takes at most 8 splits (portable cluster
    size): at MT <= 2 a plan of nine splits is trimmed to eight; at M = 4 the
    split count stays (measured slower trimmed). 4096 x 4096 with 64-column
    tiles: 64 tiles x 9 = 576 CTAs would fill 592 slots."""
    for M in (1, 2):
        p = plan(M, 4096, 4096, "gemv_64x256_ksm")
        assert p["splits"] == 8 and p["grid"] == 64 * 8, p
    p = plan(4, 4096, 4096, "gemv_64x256_ksm")
    assert p["splits"] == 9 and p["grid"] == 64 * 9, p
    # Ten splits are not trimmed (64 x 10 <= 148 x 4 needs N = 3648: 57 tiles -> 10 splits).
    p = plan(1, 3648, 4096, "gemv_64x256_ksm")
    assert p["splits"] == 10, p
