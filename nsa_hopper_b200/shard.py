"""Multi-GPU partition of the selected-branch forward: independent (batch*KV-head,
query-block range) shards, one process per GPU, no collective on the data path.

Each work row (b*Hkv+kvh, t) depends only on its own Q rows, its own K/V head and its own
selection row, so any partition of the rows is exact.  The planner keeps a KV head on as few
ranks as possible (each rank then needs only K/V of the heads it owns) and balances the
estimated work per rank: a query token costs in proportion to the blocks it gathers,
min(top_n, t // block + 1) under the BASELINE index rules.
"""
from __future__ import annotations

from typing import List, Tuple

import numpy as np

Rect = Tuple[int, int, int, int]  # (bkv_begin, bkv_end, qb_begin, qb_end)


def token_cost(T: int, top_n: int = 16, block: int = 64) -> np.ndarray:
    t = np.arange(T, dtype=np.float64)
    return np.minimum(top_n, t // block + 1)


def plan(B: int, Hkv: int, T: int, world: int, top_n: int = 16, block: int = 64) -> List[List[Rect]]:
    """Shards for `world` ranks: a list (per rank) of rectangles covering every (bkv, t) row
    exactly once."""
    rows = B * Hkv
    if world <= 0:
        raise ValueError("world must be positive")
    if world > rows * T:
        raise ValueError(f"world={world} exceeds the {rows * T} (batch*KV-head, token) rows to share")
    if world <= rows and rows % world == 0:
        per = rows // world
        return [[(r * per, (r + 1) * per, 0, T)] for r in range(world)]
    cost = token_cost(T, top_n, block)
    if world % rows == 0:
        k = world // rows  # token ranges per KV head
        cuts = _balanced_cuts(cost, k)
        out = []
        for bkv in range(rows):
            for j in range(k):
                out.append([(bkv, bkv + 1, cuts[j], cuts[j + 1])])
        return out
    # General case: walk rows in bkv-major order and cut by cumulative cost.
    flat = np.tile(cost, rows)
    cuts = _balanced_cuts(flat, world)
    out = []
    for r in range(world):
        lo, hi = cuts[r], cuts[r + 1]
        rects = []
        while lo < hi:
            bkv, t0 = divmod(lo, T)
            t1 = min(T, t0 + (hi - lo))
            rects.append((bkv, bkv + 1, t0, t1))
            lo += t1 - t0
        out.append(rects)
    return out


def _balanced_cuts(cost: np.ndarray, k: int) -> List[int]:
    """k + 1 strictly increasing cuts 0 = c_0 < ... < c_k = len(cost) that split `cost` into k
    non-empty ranges of nearly equal total cost."""
    n = len(cost)
    if k <= 0 or k > n:
        raise ValueError(f"cannot cut {n} rows into {k} non-empty ranges")
    c = np.concatenate([[0.0], np.cumsum(cost)])
    targets = c[-1] * np.arange(1, k) / k
    inner = np.searchsorted(c, targets, side="left").tolist()
    cuts = [0] + [int(x) for x in inner] + [n]
    for i in range(1, k):  # strictly increasing, and room left for the ranges after cut i
        cuts[i] = min(max(cuts[i], cuts[i - 1] + 1), n - (k - i))
    cuts[k] = n
    return cuts


def plan_strong(B: int, Hkv: int, T: int, world: int) -> Rect:
    """Single-rectangle shard of each rank (bench --scaling strong); requires a plan where every
    rank holds exactly one rectangle."""
    p = plan(B, Hkv, T, world)
    if any(len(r) != 1 for r in p):
        raise ValueError(f"world={world} does not split B*Hkv={B * Hkv} rows into single rectangles")
    return [r[0] for r in p]
