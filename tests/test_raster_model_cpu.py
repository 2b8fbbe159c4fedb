"""The tile-walk L2 model (aegis-core_b200/tune/raster_model.py): its
mechanics at the limits. With no cache every block access misses; with an
unbounded cache only the compulsory reads remain; the raster covers every
tile once; results are a pure function of the seed."""
import os
import sys

from conftest import ROOT

sys.path.insert(0, os.path.join(ROOT, "aegis-core_b200", "tune"))
import raster_model as rm  # noqa: E402

BLK = rm.BLK


def test_raster_covers_every_tile_once():
    for (tm, tn, g) in [(16, 16, 8), (13, 7, 4), (5, 9, 8)]:
        o = rm.order_grouped(tm, tn, g)
        assert sorted(o) == [(m, n) for m in range(tm) for n in range(tn)]


def test_no_cache_every_access_misses():
    o = rm.order_grouped(8, 8, 4)
    r = rm.simulate(o, kb=16, slots=10, l2_mb=BLK / 2**20 / 2, c_lines=0)  # capacity 0 blocks
    assert r["a_misses"] == r["b_misses"] == 64 * 16


def test_unbounded_cache_reads_each_block_once():
    o = rm.order_grouped(8, 12, 4)
    r = rm.simulate(o, kb=16, slots=10, l2_mb=1e6)
    assert r["a_misses"] == 8 * 16 and r["b_misses"] == 12 * 16
    assert r["ab_read_gb"] == (8 + 12) * 16 * BLK / 1e9


def test_reversal_keeps_the_access_count():
    o = rm.order_grouped(8, 8, 4)
    full = rm.simulate(o, kb=16, slots=10, l2_mb=1e6, reverse=lambda ti, m, n: n % 2 == 1)
    assert full["a_misses"] == 8 * 16 and full["b_misses"] == 8 * 16


def test_deterministic_for_a_seed():
    o = rm.order_grouped(16, 16, 8)
    a = rm.simulate(o, kb=64, slots=37, l2_mb=8, jitter=0.1, seed=3)
    b = rm.simulate(o, kb=64, slots=37, l2_mb=8, jitter=0.1, seed=3)
    assert a == b
