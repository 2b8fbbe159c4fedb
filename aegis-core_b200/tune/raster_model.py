#!/usr/bin/env python
"""L2 traffic model of the umma tile walk: DRAM reads of a raster order.

    python aegis-core_b200/tune/raster_model.py [--size 16384] [--l2-mb 126] [--jitter 0.03]

The CTA-pair kernel runs 256 x 256 tiles on `slots` clusters (74 on B200).
Tiles are handed out in raster order as clusters finish (the in-order dynamic
schedule of csrc/tile_sched.cuh). A running tile reads one A block
(256 rows x 64 k, 32 KB) and one B block (64 k x 256 columns, 32 KB) per
k-step; each k-step takes 1 +- `jitter` time units, so clusters drift apart.
L2 is modelled as one LRU over 32 KB blocks. Each finished C tile is
inserted as four 32 KB lines, so it occupies capacity as the real stores
do. The result is the number of block misses x 32 KB, with C counted
separately.

Calibration at 16384^3, grouped raster with 8 tile rows per group: 8.8 GB of
A/B reads, against 9.6-10.4 GB measured by ncu (dram__bytes_read.sum). The
measured ordering of group sizes (4 and 16 worse than 8) is reproduced.

The model then ranks K-direction alternation (a tile walks its k-blocks
last to first), at 126 MB / 63 MB of L2:
  - odd column tiles reversed: 6.8 GB / 10.0 GB;
  - odd waves reversed (runs of `slots` tiles of the raster): 6.8 GB / 7.9 GB;
  - the same wave rule in global tile coordinates: 7.2 GB / 8.8 GB.
The forward order's prediction hardly depends on L2 capacity, so only a
measurement can decide. `--l2-mb 63` gives the second column. A tuning aid;
nothing in the library imports it.
"""
from __future__ import annotations

import argparse
import heapq
import random
from collections import OrderedDict

BLK = 32 * 1024


def order_grouped(tm: int, tn: int, g: int) -> list[tuple[int, int]]:
    """The kernel's raster (decode_unit_tm): groups of g tile rows, m fastest
    inside a group, groups walked along n."""
    out = []
    for first in range(0, tm, g):
        gs = min(g, tm - first)
        for ni in range(tn):
            for mi in range(gs):
                out.append((first + mi, ni))
    return out


def simulate(order, kb: int, slots: int = 74, l2_mb: float = 126, jitter: float = 0.03, seed: int = 0,
             c_lines: int = 4, reverse=None) -> dict:
    """DRAM bytes of the A/B block misses and of the C lines for `order`.
    reverse(ti, m, n) -> True walks that tile's k-blocks last to first."""
    rnd = random.Random(seed)
    cap = int(l2_mb * 1024 * 1024) // BLK
    lru: OrderedDict = OrderedDict()
    miss = {"A": 0, "B": 0, "C": 0}

    def touch(key):
        if key in lru:
            lru.move_to_end(key)
            return
        miss[key[0]] += 1
        lru[key] = True
        if len(lru) > cap:
            lru.popitem(last=False)

    nxt = 0
    ev: list = []
    for c in range(min(slots, len(order))):
        heapq.heappush(ev, (c * 1e-6, c, nxt, 0))
        nxt += 1
    while ev:
        t, c, ti, k = heapq.heappop(ev)
        m, n = order[ti]
        kk = kb - 1 - k if (reverse is not None and reverse(ti, m, n)) else k
        touch(("A", m, kk))
        touch(("B", n, kk))
        dt = 1.0 + rnd.gauss(0.0, jitter)
        if k + 1 < kb:
            heapq.heappush(ev, (t + dt, c, ti, k + 1))
        else:
            for j in range(c_lines):
                touch(("C", m, n, j))
            if nxt < len(order):
                heapq.heappush(ev, (t + dt + 0.5, c, nxt, 0))  # the next tile starts under this epilogue
                nxt += 1
    return {"ab_read_gb": (miss["A"] + miss["B"]) * BLK / 1e9, "c_gb": miss["C"] * BLK / 1e9,
            "a_misses": miss["A"], "b_misses": miss["B"]}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--size", type=int, default=16384, help="M = N = K")
    p.add_argument("--tile", type=int, default=256)
    p.add_argument("--slots", type=int, default=74, help="clusters resident at once")
    p.add_argument("--l2-mb", type=float, default=126)
    p.add_argument("--jitter", type=float, default=0.03)
    a = p.parse_args(argv)
    t = -(-a.size // a.tile)
    kb = -(-a.size // 64)
    W = a.slots
    cases = [(f"grouped g={g}", order_grouped(t, t, g), None) for g in (4, 8, 16)]
    o8 = order_grouped(t, t, 8)
    cases += [("g=8, odd n reversed", o8, lambda ti, m, n: n % 2 == 1),
              ("g=8, odd m reversed", o8, lambda ti, m, n: m % 2 == 1),
              # odd waves (runs of `slots` consecutive tiles of the raster) reversed
              ("g=8, by wave", o8, lambda ti, m, n: (ti // W) % 2 == 1),
              # the same rule in global tile coordinates (independent of N-sharding)
              ("g=8, by wave, global", o8, lambda ti, m, n: (((m // 8) * t * 8 + n * 8) // W) % 2 == 1),
              ("g=12, by wave", order_grouped(t, t, 12), lambda ti, m, n: (ti // W) % 2 == 1)]
    for name, order, rev in cases:
        r = simulate(order, kb, a.slots, a.l2_mb, a.jitter, reverse=rev)
        print(f"{name:22s} A/B reads {r['ab_read_gb']:6.2f} GB   C {r['c_gb']:.2f} GB", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
