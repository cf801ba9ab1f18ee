"""The graph-operator calls of the reference's MultiScaleSE3Net, as recorded on its CPU path.

TEST INFRASTRUCTURE. ``tests/golden/golden_caller.npz`` (made by
``tests/golden/make_caller_golden.py``) holds, in call order, every FPS, KNN, radius-graph,
CSR-build and segment-reduce call that one forward and backward of the unchanged caller
(``nn/modules/multi_scale_se3_net.py:427``) made, with its arguments and the reference's
results. This module loads them and holds the comparison rules shared by the CPU check of the
restatement (``test_caller_golden.py``) and the GPU replay (``test_gpu_caller_replay.py``).

The reference's CPU path computes distances with torch ops whose rounding is not the CUDA
kernels': ``cdist(p=2).pow(2)`` in the radius graph (``functional/radius_graph.py`` single-cloud
path) and ``(diff * diff).sum(-1)`` in KNN (``csrc/__init__.py`` brute-force fallback). Where the
recorded result and a CUDA-rounded one differ, the difference must be explained by that rounding:
a pair within a relative 1e-5 of the radius, or of the distance at which a capped row was cut, or
two neighbours whose distances agree to 1e-5.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

FIXTURE = Path(__file__).resolve().parent / "golden" / "golden_caller.npz"
REL = 1e-5


def load():
    z = np.load(FIXTURE)
    meta = json.loads(str(z["meta"]))
    out = []
    for i, c in enumerate(meta["calls"]):
        d = dict(c)
        d["i"] = i
        pre = f"c{i}_"
        for k in z.files:
            if k.startswith(pre):
                a = z[k]
                d[k[len(pre):]] = a.astype(np.int64) if a.dtype == np.int32 else a
        out.append(d)
    return meta, out


def call_id(c) -> str:
    return f"{c['i']:02d}-{c['op']}"


def ptr_of_batch(batch: np.ndarray) -> np.ndarray:
    B = int(batch.max()) + 1 if batch.size else 0
    counts = np.bincount(batch, minlength=B)
    assert np.all(np.diff(batch) >= 0), "the recorded clouds are contiguous"
    return np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)


def csr_matches_unordered(got, want):
    """CSR arrays (col_sorted, perm, node_start, node_end) equal, ``perm`` up to the order inside
    each destination's segment: the reference's CPU path sorts with an unstable ``torch.sort``
    (``functional/segment_reduce.py`` _sort_and_build_csr_pytorch); its CUDA path, like this
    library, keeps edge order within a segment."""
    cs, pm, ns, ne = (np.asarray(a, np.int64) for a in got)
    wcs, wpm, wns, wne = (np.asarray(a, np.int64) for a in want)
    if not (np.array_equal(cs, wcs) and np.array_equal(ns, wns) and np.array_equal(ne, wne)):
        return False
    key = lambda p: np.lexsort((p, cs))  # noqa: E731  (segment, then edge id)
    return bool(np.array_equal(pm[key(pm)], wpm[key(wpm)]))


def _d2(x: np.ndarray, a, b) -> np.ndarray:
    x = x.astype(np.float64)
    return ((x[a] - x[b]) ** 2).sum(-1)


def radius_difference_explained(x, r, max_nn, row_a, col_a, row_b, col_b):
    """(ok, n_diff): edges (row = source, col = target) of two radius graphs over the same points
    agree, or every edge in only one of them sits at the rounding edge of the radius or of its
    target's cut (the max_nn-th nearest in radius, when the row is capped)."""
    ka = np.unique(np.asarray(col_a, np.int64) * (1 << 32) + np.asarray(row_a, np.int64))
    kb = np.unique(np.asarray(col_b, np.int64) * (1 << 32) + np.asarray(row_b, np.int64))
    diff = np.setxor1d(ka, kb)
    if diff.size == 0:
        return True, 0
    r2 = float(r) * float(r)
    src, dst = diff & 0xFFFFFFFF, diff >> 32
    d = _d2(x, src, dst)
    near_r = np.abs(d - r2) <= REL * r2
    ok = near_r.copy()
    for j in np.nonzero(~near_r)[0]:
        t = int(dst[j])
        # the target's cut: the max_nn-th nearest within r (its candidates from either graph)
        cand = np.unique(np.concatenate([np.asarray(row_a)[np.asarray(col_a) == t],
                                         np.asarray(row_b)[np.asarray(col_b) == t]]))
        dc = np.sort(_d2(x, cand, np.full(cand.shape, t)))
        if dc.size >= max_nn:
            cut = dc[max_nn - 1]
            ok[j] = abs(d[j] - cut) <= REL * max(cut, 1e-30)
    return bool(ok.all()), int(diff.size)


def knn_difference_explained(idx_a, dist_a, idx_b, dist_b):
    """(ok, n_diff): two KNN results agree, or where their indices differ the distances of the
    swapped neighbours agree to 1e-5 (a near-tie that rounding may order either way); the
    distances themselves must agree to 1e-5 relative (1e-7 absolute for a point's own)."""
    da = np.asarray(dist_a, np.float64)
    db = np.asarray(dist_b, np.float64)
    if not np.allclose(da, db, rtol=REL, atol=1e-7):
        return False, int((~np.isclose(da, db, rtol=REL, atol=1e-7)).sum())
    bad = np.asarray(idx_a) != np.asarray(idx_b)
    if not bad.any():
        return True, 0
    ok = True
    for q in np.nonzero(bad.any(1))[0]:
        # the rows must hold the same neighbours up to reordering among near-equal distances,
        # except at the last slot, where a near-tie may pick a different neighbour
        row_a, row_b = np.asarray(idx_a[q]), np.asarray(idx_b[q])
        for j in np.nonzero(row_a != row_b)[0]:
            near = np.abs(db[q] - da[q, j]) <= REL * max(da[q, j], 1e-30)
            if not (near.any() and (row_a[j] in row_b[near] or j == len(row_a) - 1 or
                                    np.isclose(da[q, -1], da[q, j], rtol=REL))):
                ok = False
    return ok, int(bad.sum())
