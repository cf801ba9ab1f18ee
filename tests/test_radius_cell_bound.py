"""The radius query's cell-skip bound, restated in float32 on the CPU (no GPU).

``rg_query_warp_kernel`` (gdl_b200/csrc/radius.cu) skips a neighbouring column, or the z-cell
below or above the query's own, when a lower bound on the squared distance to anything binned into
it exceeds the selection bound (or r^2 before there is one). The skip keeps the kernel's result
exact only if that lower bound never exceeds the distance the kernel computes (``dist2``) to a
point binned into the cell. The bound comes from ``face_gaps``: the query's scaled coordinate
against the faces of its own cell, less a margin for the binning arithmetic's rounding, then
scaled down by more than ``dist2``'s rounding. This test restates both sides in float32, operation
by operation, and checks the inequality on points placed within a few ulps of cell faces, on grids
far from the origin, with a cell size that is not a power of two, and in the clamped last cell of
a grid capped at 1024 cells (radius_graph_kernel.cu:280-299 for the grid rules).
"""

import itertools

import numpy as np
import pytest

F = np.float32


def _grid(lo, hi, r):
    # radius_graph_kernel.cu:280-299 as restated by rg_grid_kernel: box -/+ 1e-5, cell = r,
    # res = ceil(extent / r) + 1 capped at 1024
    mn = (lo - F(1e-5)).astype(F)
    ext = ((hi + F(1e-5)).astype(F) - mn).astype(F)
    res = np.minimum(np.ceil(ext / F(r)).astype(np.int64) + 1, 1024)
    return mn, res


def _scaled(p, mn, inv):
    return ((p - mn).astype(F) * inv).astype(F)  # cell_coord before the floor (FTZ irrelevant here)


def _face_gaps(u, qc, res):
    eps = (F(2.0 ** -19) * (np.abs(u) + F(2.0)).astype(F)).astype(F)
    below = np.where(qc < res, np.maximum((u - qc.astype(F)).astype(F) - eps, F(0.0)), F(0.0)).astype(F)
    above = np.maximum(((qc + 1).astype(F) - u).astype(F) - eps, F(0.0)).astype(F)
    return below, above


def _dist2(q, p):
    # dist2: dx, dy, dz rounded; fma(dz, dz, fma(dx, dx, dy * dy)) (each fma rounded once: the
    # float64 product of two float32 values is exact)
    d = (q[:, None, :] - p[None, :, :]).astype(F)
    dy2 = (d[..., 1] * d[..., 1]).astype(F)
    t = (d[..., 0].astype(np.float64) ** 2 + dy2).astype(F)
    return (d[..., 2].astype(np.float64) ** 2 + t).astype(F)


def _near_faces(rng, mn, r, cells, n, ulps=4):
    """Coordinates within a few ulps of the faces mn + k r (k in cells), per axis."""
    k = rng.choice(cells, size=(n, 3))
    base = (mn + (k * F(r)).astype(F)).astype(F)
    step = rng.integers(-ulps, ulps + 1, size=(n, 3))
    out = base.copy()
    for i in range(n):
        for a in range(3):
            out[i, a] = base[i, a]
            s = step[i, a]
            for _ in range(abs(s)):
                out[i, a] = np.nextafter(out[i, a], F(np.inf) if s > 0 else F(-np.inf))
    jitter = rng.random((n, 3)) < 0.3  # some points anywhere inside their cell
    out[jitter] = (base[jitter] + F(r) * rng.random(int(jitter.sum())).astype(F)).astype(F)
    return out


def _check(q, p, mn, res, r):
    inv = F(1.0) / F(r)
    r_sq = F(F(r) * F(r))
    shrink = F(r_sq * F(1.0 - 2.0 ** -19))
    uq = _scaled(q, mn, inv)
    qc = np.floor(uq).astype(np.int64)
    up = _scaled(p, mn, inv)
    pc = np.clip(np.floor(up).astype(np.int64), 0, res - 1)  # the points are binned clamped
    gl, gh = _face_gaps(uq, qc, res)
    d = _dist2(q, p)
    checked = 0
    for dx, dy, dz in itertools.product((-1, 0, 1), repeat=3):
        if dx == dy == dz == 0:
            continue
        cell = qc[:, None, :] + np.array([dx, dy, dz])[None, None, :]
        inside = np.all(pc[None, :, :] == cell, axis=2)  # point binned into this neighbour of the query
        if not inside.any():
            continue
        gx = gl[:, 0] if dx < 0 else (gh[:, 0] if dx > 0 else np.zeros(len(q), F))
        gy = gl[:, 1] if dy < 0 else (gh[:, 1] if dy > 0 else np.zeros(len(q), F))
        gz = gl[:, 2] if dz < 0 else (gh[:, 2] if dz > 0 else np.zeros(len(q), F))
        gxy = ((gx * gx).astype(F) + (gy * gy).astype(F)).astype(F)
        lb = (((gxy + (gz * gz).astype(F)).astype(F)) * shrink).astype(F)
        bad = inside & (lb[:, None] > d)
        assert not bad.any(), (dx, dy, dz, np.argwhere(bad)[:3])
        checked += int(inside.sum())
    return checked


@pytest.mark.parametrize("origin,r", [(0.0, 1.0), (1000.0, 0.37), (-250.0, 0.125), (3.0e4, 2.5)])
def test_skip_bound_below_binned_distances(origin, r):
    rng = np.random.default_rng(int(abs(origin)) + 7)
    lo = np.full(3, origin, F)
    hi = (lo + F(12 * r)).astype(F)
    mn, res = _grid(lo, hi, r)
    cells = np.arange(0, 12)
    q = _near_faces(rng, mn, r, cells, 600)
    p = _near_faces(rng, mn, r, cells, 1500)
    q = np.clip(q, lo, hi).astype(F)
    p = np.clip(p, lo, hi).astype(F)
    assert _check(q, p, mn, res, r) > 10000


def test_skip_bound_in_the_clamped_last_cell():
    # an extent of 1500 cells caps the grid at 1024: the last cell holds every point beyond it,
    # and queries there have unclamped cells past the grid
    rng = np.random.default_rng(3)
    r = 0.5
    lo = np.zeros(3, F)
    hi = np.array([1500 * r, 6 * r, 6 * r], F)
    mn, res = _grid(lo, hi, r)
    assert res[0] == 1024
    cells = np.arange(1018, 1030)
    q = _near_faces(rng, mn, r, cells, 500)
    p = _near_faces(rng, mn, r, cells, 1500)
    q[:, 1:] = np.clip(q[:, 1:], lo[1:], hi[1:])
    p[:, 1:] = np.clip(p[:, 1:], lo[1:], hi[1:])
    assert _check(q, p, mn, res, r) > 1000
