"""Pin the CPU checker's KNN aggregation (oracle/) against the reference's CPU path.

tests/golden/golden_aggregate.npz holds EquivariantInterpolate forward/backward
(nn/modules/equivariant_interp.py:58-139) and the weighted-sum lines of EquivariantPool
(nn/modules/equivariant_pool.py:395-420) with their gradients, computed by the reference on the
CPU (tests/golden/make_golden.py). The sums are floating point and torch's CPU reduction order
over k depends on the shape (sequential up to k = 8, blocked beyond), and its vectorised sqrt is
not correctly rounded, so the bar is the one the reference's fp32 sums get: per element
|ours - ref| <= 1e-5 * sum_j |w_j f_j| + 1e-7. The neighbour lists and the weight rule are
exact (indices equal).
"""

import numpy as np
import pytest


@pytest.fixture(scope="module")
def ga():
    from tests.conftest import ROOT

    return np.load(ROOT / "tests" / "golden" / "golden_aggregate.npz")


def close(got, ref, bound, rel=1e-5, abs_=1e-7):
    got, ref, bound = (np.asarray(a, np.float64) for a in (got, ref, bound))
    return got.shape == ref.shape and bool(np.all(np.abs(got - ref) <= rel * bound + abs_))


def test_interpolate_forward_backward(ga, oracle):
    d, c = ga["interp_dense"], ga["interp_coarse"]
    idx, dist = oracle.knn(d, c, ga["interp_ptr_d"], ga["interp_ptr_c"], 3, dist=oracle.DIST_TORCH)
    assert (idx < 0).sum() == 37  # the 2-point coarse cloud pads one slot of each of its 37 queries
    w = oracle.knn_idw_weights(idx, dist)
    assert np.allclose(w.sum(1), 1.0, atol=1e-6)
    s, v, t2 = ga["interp_s"], ga["interp_v"], ga["interp_t2"]
    for f, name, skip in ((s, "s", ga["interp_s_skip"]), (v, "v", ga["interp_v_skip"]), (t2, "t2", None)):
        out = oracle.knn_weighted_sum(f, idx, w)
        bound = oracle.knn_weighted_sum(np.abs(f), idx, np.abs(w))
        if skip is not None:
            out = np.concatenate([out, skip], axis=1)
            bound = np.concatenate([bound, np.abs(skip)], axis=1)
        assert close(out, ga[f"interp_{name}_out"], bound)
    # backward w.r.t. the coarse tables (skip channels carry no gradient to them)
    gs = ga["interp_g_s"][:, :16]
    gv = ga["interp_g_v"][:, :8]
    for g, f, name in ((gs, s, "s"), (gv, v, "v"), (ga["interp_g_t2"], t2, "t2")):
        got = oracle.knn_weighted_sum_backward(g, idx, w, f.shape[0])
        bound = oracle.knn_weighted_sum_backward(np.abs(g), idx, np.abs(w), f.shape[0])
        assert close(got, ga[f"interp_grad_{name}"], bound)


def test_pool_weighted_sums(ga, oracle):
    idx, w = ga["pool_idx"], ga["pool_w"]
    assert (idx < 0).any() and np.all(w[idx < 0] == 0)
    sc, vc = ga["pool_scalars"], ga["pool_vectors"]
    for f, name in ((sc, "s"), (vc, "v")):
        out = oracle.knn_weighted_sum(f, idx, w)
        assert close(out, ga[f"pool_{name}_out"], oracle.knn_weighted_sum(np.abs(f), idx, np.abs(w)))
    gs, gv = ga["pool_g_s"], ga["pool_g_v"]
    for g, f, name in ((gs, sc, "s"), (gv, vc, "v")):
        got = oracle.knn_weighted_sum_backward(g, idx, w, f.shape[0])
        assert close(got, ga[f"pool_grad_{name}"], oracle.knn_weighted_sum_backward(np.abs(g), idx, np.abs(w),
                                                                                     f.shape[0]))
    gw = oracle.knn_weighted_sum_weight_grad([gs, gv], [sc, vc], idx)
    bound = oracle.knn_weighted_sum_weight_grad([np.abs(gs), np.abs(gv)], [np.abs(sc), np.abs(vc)], idx)
    ref = ga["pool_grad_w"].copy()
    # the reference's padded slots gather row 0 with weight 0 and still get a weight gradient
    # (grad_out . feat[0]); this build skips padded slots and gives them 0
    pad = idx < 0
    assert np.all(gw[pad] == 0)
    assert close(gw[~pad], ref[~pad], bound[~pad])


def test_weighted_sum_rules(oracle):
    rng = np.random.default_rng(0)
    src = rng.standard_normal((10, 6)).astype(np.float32)
    idx = np.array([[0, 3, -1], [9, 9, 2], [-1, -1, -1], [12, 1, 1]], np.int64)
    w = rng.random((4, 3)).astype(np.float32)
    out = oracle.knn_weighted_sum(src, idx, w)
    want0 = np.float32(np.float32(w[0, 0] * src[0]) + np.float32(w[0, 1] * src[3]))
    assert np.array_equal(out[0], want0)
    assert np.all(out[2] == 0)  # no valid neighbour
    assert np.array_equal(out[3], np.float32(np.float32(w[3, 1] * src[1]) + np.float32(w[3, 2] * src[1])))
    # IDW: all-padding rows get 0 weights; dist below 1e-4 is clamped
    wi = oracle.knn_idw_weights(np.array([[-1, -1], [0, 1]]), np.array([[1.0, 2.0], [0.0, 1e-4]], np.float32))
    assert np.all(wi[0] == 0) and np.allclose(wi[1], [0.5, 0.5])
