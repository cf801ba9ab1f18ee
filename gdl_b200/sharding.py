"""Splitting a batch of packed clouds over ranks (one process per GPU).

Clouds are independent, so a batch is sharded by whole clouds: each rank takes a contiguous
range of clouds whose estimated work is about 1/world of the total, runs the operators on its
slice with no collective, and results can be gathered afterwards. Work estimates per cloud:
FPS ~ n_b * k_b, brute-force KNN ~ n_q * n_s, radius graph / segment reduce ~ n_b.
"""

from __future__ import annotations

from typing import Sequence, Tuple

import numpy as np


def shard_clouds(cost: Sequence[float], world: int, rank: int) -> Tuple[int, int]:
    """Contiguous cloud range [c0, c1) of `rank`: cloud b goes to the rank whose share of the
    cumulative cost contains the midpoint of b's own cost interval (deterministic; every cloud
    belongs to exactly one rank)."""
    c = np.asarray(cost, dtype=np.float64)
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    if c.size == 0:
        return 0, 0
    total = c.sum()
    if total <= 0:
        c = np.ones_like(c)
        total = c.sum()
    mid = np.cumsum(c) - 0.5 * c
    owner = np.minimum((mid / total * world).astype(np.int64), world - 1)
    idx = np.nonzero(owner == rank)[0]
    if idx.size == 0:
        # an empty share sits where the owners cross this rank's boundary
        c0 = int(np.searchsorted(owner, rank))
        return c0, c0
    return int(idx[0]), int(idx[-1]) + 1


def local_slice(ptr: Sequence[int], c0: int, c1: int):
    """(point offset, rebased ptr [c1-c0+1]) of clouds [c0, c1) of a packed batch."""
    p = np.asarray(ptr, dtype=np.int64)
    return int(p[c0]), p[c0:c1 + 1] - p[c0]
