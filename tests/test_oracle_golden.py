"""Pin the CPU checker (oracle/) against golden vectors of the reference's own CPU path.

The fixtures in tests/golden/golden_cpu.npz were produced by tests/golden/make_golden.py,
which imports the reference package and calls its public entry points on the CPU.
Where the reference's CPU fallbacks and its CUDA kernels are documented to differ,
the test states the difference and checks the checker follows the CUDA kernel:

* CPU distances are ((dx*dx+dy*dy)+dz*dz) without FMA/FTZ -> checked with dist mode "torch".
* KNN with k > 64: the CPU path returns min(k, n) neighbours, the kernel at most 64
  (MinK<64>, knn_kernel.cu:281-288).
* sort_and_build_csr: CPU argsort is not stable (segment_reduce.py:93); the kernel's
  CUB radix sort is, so perms agree as per-segment sets and the fold order is pinned by
  replaying the CPU perm.
* segment mean/max in bf16: torch keeps bf16 outputs; the build accumulates and
  returns fp32 (tolerance 1e-2).
"""

import hashlib

import numpy as np
import pytest

from tests.golden import inputs


def _edges(row, col):
    return set(zip(np.asarray(row).tolist(), np.asarray(col).tolist()))


def test_fps_config1(golden, oracle):
    pos, ptr = inputs.config1_points()
    for tie in (oracle.TIE_LOWEST_INDEX, oracle.TIE_REFERENCE):
        idx = oracle.fps(pos, ptr, [512] * 4, tie=tie, dist=oracle.DIST_TORCH)
        assert np.array_equal(idx, golden["fps_c1_idx"])


def test_fps_variable_and_single(golden, oracle):
    pv, pp = golden["fps_var_pos"], golden["fps_var_ptr"]
    k = np.minimum(np.diff(pp), 64)
    assert np.array_equal(oracle.fps(pv, pp, k, tie=oracle.TIE_LOWEST_INDEX, dist=oracle.DIST_TORCH),
                          golden["fps_var_idx"])
    assert np.array_equal(oracle.fps(pv[:300], [0, 300], [50], tie=oracle.TIE_LOWEST_INDEX,
                                     dist=oracle.DIST_TORCH), golden["fps_single_idx"])


def test_fps_edge_cases(oracle):
    pos = np.random.default_rng(0).random((50, 3), dtype=np.float32)
    # k > n: n indices, remaining slots -1, selection starts at the first point
    out = oracle.fps(pos, [0, 10, 50], [20, 5])
    assert out.shape == (25,)
    assert sorted(out[:10].tolist()) == list(range(10)) and out[0] == 0
    assert (out[10:20] == -1).all() and out[20] == 10
    # empty cloud / k = 0
    out = oracle.fps(pos, [0, 0, 50], [3, 0])
    assert (out == -1).all()


def test_fps_reference_tie_rule(oracle):
    """All points equidistant from the seed: the kernel's reduction order decides."""
    n = 1500
    pos = np.zeros((n, 3), np.float32)
    pos[1:, 0] = 1.0  # every point but the seed sits at the same place
    out = oracle.fps(pos, [0, n], [2], tie=oracle.TIE_REFERENCE)
    pri = [oracle.fps_priority(i) for i in range(1, n)]
    assert out[1] == 1 + int(np.argmin(pri))
    out = oracle.fps(pos, [0, n], [2], tie=oracle.TIE_LOWEST_INDEX)
    assert out[1] == 1
    # bit-reversal: among lanes 1 and 2 of warp 0, lane 2 (brev5=01000b) beats lane 1 (10000b)
    assert oracle.fps_priority(2) < oracle.fps_priority(1)
    # warp 8 beats warp 1 (brev4: 0001b vs 1000b); same lane, thread-strided round breaks last
    assert oracle.fps_priority(8 * 32) < oracle.fps_priority(32)
    assert oracle.fps_priority(5) < oracle.fps_priority(5 + 512)


def test_knn_config1(golden, oracle):
    pos, ptr = inputs.config1_points()
    q = pos[golden["fps_c1_idx"].astype(np.int64)]
    idx, d = oracle.knn(q, pos, np.arange(0, 2049, 512), ptr, 16, dist=oracle.DIST_TORCH)
    assert np.array_equal(idx, golden["knn_c1_idx"])
    assert np.array_equal(d, golden["knn_c1_dist"])


@pytest.mark.parametrize("k", [1, 5, 16, 33, 70])
def test_knn_variable(golden, oracle, k):
    i, d = oracle.knn(golden["knn_var_q"], golden["knn_var_s"], golden["knn_var_ptr_q"], golden["knn_var_ptr_s"], k,
                      dist=oracle.DIST_TORCH)
    gi, gd = golden[f"knn_var_k{k}_idx"], golden[f"knn_var_k{k}_dist"]
    m = min(k, 64)
    assert np.array_equal(i[:, :m], gi[:, :m]) and np.array_equal(d[:, :m], gd[:, :m])
    assert (i[:, m:] == -1).all() and (d[:, m:] == np.float32(1e30)).all()


def test_knn_heap_ties(oracle):
    """Duplicated sources: output order follows the heap, not the index."""
    rng = np.random.default_rng(3)
    s = rng.random((40, 3), dtype=np.float32)
    s[10:20] = s[0]  # 11 coincident points
    idx, d = oracle.knn(s[:1], s, [0, 1], [0, 40], 4)
    assert (d[0] == 0).all()
    assert set(idx[0].tolist()) <= set([0] + list(range(10, 20)))


@pytest.mark.parametrize("loop", [False, True])
@pytest.mark.parametrize("use_mask", [False, True])
def test_radius_batched(golden, oracle, loop, use_mask):
    x, mask = golden["rad_x"], golden["rad_mask"]
    B, n, K = golden["rad_meta"]
    r = float(golden["rad_r"][0])
    rp, src = oracle.radius_graph(x, np.arange(0, B * n + 1, n), r, int(K), loop, mask if use_mask else None,
                                  dist=oracle.DIST_TORCH)
    row, col = oracle.csr_to_coo(rp, src)
    tag = f"rad_b_loop{int(loop)}_mask{int(use_mask)}"
    assert _edges(row, col) == _edges(golden[tag + "_row"], golden[tag + "_col"])
    # CSR order: destinations ascending, sources ascending within a destination
    assert np.all(np.diff(col) >= 0)
    for a, b in zip(rp[:-1], rp[1:]):
        assert np.all(np.diff(src[a:b]) > 0)


def test_radius_single_and_kat(golden, oracle):
    x = golden["rad_x"]
    n = int(golden["rad_meta"][1])
    rp, src = oracle.radius_graph(x[:n], [0, n], float(golden["rad_r"][0]), 32, dist=oracle.DIST_TORCH)
    assert _edges(*oracle.csr_to_coo(rp, src)) == _edges(golden["rad_single_row"], golden["rad_single_col"])
    kat = np.array([[0.0, 0.0, 0.0], [0.1, 0.0, 0.0], [10.0, 0.0, 0.0]], np.float32)
    rp, src = oracle.radius_graph(kat, [0, 3], 1.0, 32)
    assert _edges(*oracle.csr_to_coo(rp, src)) == _edges(golden["rad_kat3_row"], golden["rad_kat3_col"])
    # tests/test_phase1.py:273-280: points of different clouds never connect
    two = np.array([[0.0, 0.0, 0.0], [0.1, 0.0, 0.0]], np.float32)
    rp, src = oracle.radius_graph(two, [0, 1, 2], 100.0, 32)
    assert src.size == 0
    # r <= 0 and single-point clouds give no edges (radius_graph_kernel.cu:269-272)
    assert oracle.radius_graph(kat, [0, 3], 0.0, 32)[1].size == 0


def test_radius_truncation_keeps_nearest(oracle):
    rng = np.random.default_rng(5)
    x = rng.random((400, 3), dtype=np.float32) * 0.3  # dense: every point has > 16 in radius
    rp, src = oracle.radius_graph(x, [0, 400], 0.25, 16, dist=oracle.DIST_FMA_ZYX)
    deg = np.diff(rp)
    assert deg.max() == 16
    # the kept set of query 0 is its 16 nearest (distinct distances here)
    d = ((x - x[0]) ** 2).sum(1).astype(np.float64)
    d[0] = np.inf
    assert set(src[rp[0]:rp[1]].tolist()) == set(np.argsort(d)[:16].tolist())


def test_csr_build(golden, oracle):
    cs, pm, ns, ne = oracle.sort_and_build_csr(golden["seg_r_col"], 500)
    assert np.array_equal(cs, golden["seg_r_cs"])
    assert np.array_equal(ns, golden["seg_r_ns"]) and np.array_equal(ne, golden["seg_r_ne"])
    for a, b in zip(ns, ne):  # same per-segment edge sets, ours ascending (stable)
        assert sorted(pm[a:b].tolist()) == sorted(golden["seg_r_perm"][a:b].tolist())
        assert np.all(np.diff(pm[a:b]) > 0)
    # empty nodes keep 0/0 like the CUDA offsets kernel
    cs, pm, ns, ne = oracle.sort_and_build_csr(np.array([3, 3, 1], np.int64), 5)
    assert ns.tolist() == [0, 0, 0, 1, 0] and ne.tolist() == [0, 1, 0, 3, 0]
    assert pm.tolist() == [2, 0, 1]
    with pytest.raises(ValueError):
        oracle.sort_and_build_csr(np.array([5], np.int64), 5)


def test_segment_sum_fold_order(golden, oracle):
    """Replaying the reference CPU perm gives its sum bit-for-bit: same sequential fold."""
    o = oracle.segment_reduce(golden["seg_r_msg"], golden["seg_r_perm"], golden["seg_r_ns"], golden["seg_r_ne"],
                              500, "sum")
    assert np.array_equal(o, golden["seg_r_sum"])
    g = oracle.segment_reduce_backward(golden["seg_r_gout"], golden["seg_r_msg"], o, golden["seg_r_perm"],
                                       golden["seg_r_ns"], golden["seg_r_ne"], 500, "sum")
    assert np.array_equal(g, golden["seg_r_sum_grad"])


@pytest.mark.parametrize("red", ["mean", "max"])
def test_segment_mean_max(golden, oracle, red):
    msg = golden["seg_r_msg"]
    cs, pm, ns, ne = oracle.sort_and_build_csr(golden["seg_r_col"], 500)
    o = oracle.segment_reduce(msg, pm, ns, ne, 500, red)
    assert np.array_equal(o, golden[f"seg_r_{red}_f32"])
    g = oracle.segment_reduce_backward(golden["seg_r_gout"], msg, o, pm, ns, ne, 500, red)
    assert np.array_equal(g, golden[f"seg_r_{red}_f32_grad"])
    # bf16 inputs, fp32 accumulation: within 1e-2 of torch's bf16 results
    mb = oracle.bf16_bits(msg)
    o = oracle.segment_reduce(mb, pm, ns, ne, 500, red)
    assert np.allclose(o, golden[f"seg_r_{red}_bf16"], rtol=1e-2, atol=1e-2)
    g = oracle.bf16_to_f32(oracle.segment_reduce_backward(golden["seg_r_gout"], mb, o, pm, ns, ne, 500, red))
    assert np.allclose(g, golden[f"seg_r_{red}_bf16_grad"], rtol=1e-2, atol=1e-2)


def test_segment_config1_hashes(golden, oracle):
    col, msg = inputs.config1_segment_inputs()
    cs, pm, ns, ne = oracle.sort_and_build_csr(col, 2048)
    gout = inputs.config1_grad_out()

    def sha(a):
        return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()

    o = oracle.segment_reduce(msg, pm, ns, ne, 2048, "sum")
    assert sha(o) == bytes(golden["seg_c1_sum_sha"]).decode()
    g = oracle.segment_reduce_backward(gout, msg, o, pm, ns, ne, 2048, "sum")
    assert sha(g) == bytes(golden["seg_c1_sum_grad_sha"]).decode()
    o = oracle.segment_reduce(msg, pm, ns, ne, 2048, "max")
    assert sha(o) == bytes(golden["seg_c1_max_sha"]).decode()
    g = oracle.segment_reduce_backward(gout, msg, o, pm, ns, ne, 2048, "max")
    assert sha(g) == bytes(golden["seg_c1_max_grad_sha"]).decode()
