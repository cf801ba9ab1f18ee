"""Pin the CPU checker's graph geometry (oracle/) against the reference's own CPU path.

tests/golden/golden_graph.npz holds what the reference's ``SpatialGraph.build`` /
``from_edge_index`` (nn/modules/spatial_graph.py:88-246) and ``compute_edge_vectors`` +
spherical harmonics (functional/radius_graph.py:338-358, kernels/triton_sph_harm.py:200-240)
return on the CPU for seeded inputs (tests/golden/make_golden.py). Geometry is compared bit
for bit (NaN patterns included); edge lists as sets, since the reference's edge order carries
no meaning.
"""

import numpy as np
import pytest

@pytest.fixture(scope="module")
def gg():
    from tests.conftest import ROOT

    return np.load(ROOT / "tests" / "golden" / "golden_graph.npz")


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    same = a.view(np.uint32) == b.view(np.uint32)
    both_nan = np.isnan(a) & np.isnan(b)
    return a.shape == b.shape and bool(np.all(same | both_nan))


def same_csr(ns, ne, ref_ns, ref_ne):
    """Equal segments; nodes without edges are empty in both. (The reference's CPU CSR build,
    functional/segment_reduce.py:77-109, gives an empty node its position as start and end;
    its CUDA kernel, segment_reduce_kernel.cu:30-50, and this build give 0 / 0.)"""
    ns, ne, ref_ns, ref_ne = (np.asarray(a, np.int64) for a in (ns, ne, ref_ns, ref_ne))
    deg, ref_deg = ne - ns, ref_ne - ref_ns
    full = deg > 0
    return (np.array_equal(deg, ref_deg) and np.array_equal(ns[full], ref_ns[full])
            and bool(np.all(ns[~full] == 0)) and bool(np.all(ne[~full] == 0)))


def by_edge(row, col, *vals):
    order = np.lexsort((np.asarray(row), np.asarray(col)))
    return [np.asarray(v)[order] for v in (row, col, *vals)]


def test_edge_geometry_handmade(gg, oracle):
    x, row, col = gg["geo_x"], gg["geo_row"], gg["geo_col"]
    for lmax in (0, 1, 2):
        diff, dist, direction, sph = oracle.edge_geometry(x, row, col, max_l=lmax)
        assert bits_equal(diff, gg["geo_diff"])
        assert bits_equal(dist, gg["geo_dist"])
        assert bits_equal(direction, gg["geo_dir"])
        assert bits_equal(sph, gg[f"geo_Y{lmax}"])
    # the edge cases are present: clamp at 1e-8 (zero and tiny vectors), overflow, NaN
    assert (gg["geo_dist"][:14] == np.float32(1e-8)).sum() >= 2
    assert np.isinf(gg["geo_dist"]).any() and np.isnan(gg["geo_dir"]).any()


def _oracle_graph(oracle, x, ptr, r, K, max_l=2, batch=None, num_clouds=None):
    rp, src = oracle.radius_graph(x, ptr, r, K, dist=oracle.DIST_TORCH)
    row, col = oracle.csr_to_coo(rp, src)
    _, dist, direction, sph = oracle.edge_geometry(x, row, col, max_l=max_l)
    cs, pm, ns, ne = oracle.sort_and_build_csr(col, x.shape[0])
    avg = oracle.cloud_avg_degree(ns, ne, batch=batch, num_clouds=num_clouds)
    return row, col, dist, direction, sph, cs, ns, ne, avg


@pytest.mark.parametrize("case", ["batch", "single", "shuffled"])
def test_spatial_graph_build(gg, oracle, case):
    x = gg["graph_x"]
    B, n, K, _ = (int(v) for v in gg["graph_meta"])
    r = float(gg["graph_r"][0])
    batch = np.repeat(np.arange(B), n)
    if case == "single":
        x, ptr, bt, nc = x[:n], [0, n], None, None
    elif case == "batch":
        ptr, bt, nc = np.arange(B + 1) * n, batch, B
    else:  # unequal clouds interleaved: build on the cloud-sorted order, map indices back
        sel, perm = gg["graph_sel"], gg["graph_perm"]
        xs, bs = x[sel][perm], batch[sel][perm]
        order = np.argsort(bs, kind="stable")
        ptr = np.concatenate([[0], np.cumsum(np.bincount(bs, minlength=B))])
        row, col, dist, direction, sph, *_ = _oracle_graph(oracle, xs[order], ptr, r, K)
        row, col = order[row], order[col]
        _, _, ns, ne = oracle.sort_and_build_csr(col, xs.shape[0])
        avg = oracle.cloud_avg_degree(ns, ne, batch=bs, num_clouds=B)
        got = by_edge(row, col, dist, direction, sph)
        ref = by_edge(gg[f"graph_{case}_row"], gg[f"graph_{case}_col"], gg[f"graph_{case}_dist"],
                      gg[f"graph_{case}_direction"], gg[f"graph_{case}_Y"])
        assert np.array_equal(got[0], ref[0]) and np.array_equal(got[1], ref[1])
        for a, b in zip(got[2:], ref[2:]):
            assert bits_equal(a, b)
        assert same_csr(ns, ne, gg[f"graph_{case}_node_start"], gg[f"graph_{case}_node_end"])
        assert bits_equal(avg, gg[f"graph_{case}_avg_degree"])
        return
    row, col, dist, direction, sph, cs, ns, ne, avg = _oracle_graph(oracle, x, ptr, r, K, batch=bt,
                                                                    num_clouds=nc)
    got = by_edge(row, col, dist, direction, sph)
    ref = by_edge(gg[f"graph_{case}_row"], gg[f"graph_{case}_col"], gg[f"graph_{case}_dist"],
                  gg[f"graph_{case}_direction"], gg[f"graph_{case}_Y"])
    assert np.array_equal(got[0], ref[0]) and np.array_equal(got[1], ref[1])
    for a, b in zip(got[2:], ref[2:]):
        assert bits_equal(a, b)
    assert same_csr(ns, ne, gg[f"graph_{case}_node_start"], gg[f"graph_{case}_node_end"])
    if case == "single":
        # the reference averages with degree.mean(); exact integers / n here
        assert np.allclose(avg, gg[f"graph_{case}_avg_degree"], rtol=2e-7, atol=0)
    else:
        assert bits_equal(avg, gg[f"graph_{case}_avg_degree"])
    assert avg.min() >= 1.0 and avg.max() > 5.0  # the fixture is dense enough to leave the clamp


def test_from_edge_index(gg, oracle):
    x = gg["graph_x"]
    B, n, _, _ = (int(v) for v in gg["graph_meta"])
    row, col = gg["graph_batch_row"], gg["graph_batch_col"]
    cs, pm, ns, ne = oracle.sort_and_build_csr(col, B * n)
    assert np.array_equal(cs, gg["graph_fei_col_sorted"])
    assert same_csr(ns, ne, gg["graph_fei_node_start"], gg["graph_fei_node_end"])
    avg = oracle.cloud_avg_degree(ns, ne, batch=np.repeat(np.arange(B), n), num_clouds=B)
    assert bits_equal(avg, gg["graph_fei_avg_degree"])
    assert bits_equal(oracle.edge_geometry(x, row, col, max_l=1)[3], gg["graph_fei_Y"])


def test_cloud_avg_degree_rules(oracle):
    ns = np.array([0, 0, 3, 3, 9], np.int32)
    ne = np.array([0, 3, 3, 9, 10], np.int32)
    # degrees 0 3 0 6 1; ptr clouds {0,1}, {2,3}; node 4 is outside every cloud and gets 1
    out = oracle.cloud_avg_degree(ns, ne, ptr=[0, 2, 4])
    assert out.tolist() == [1.5, 1.5, 3.0, 3.0, 1.0]
    # batch clouds {1,3} (9 / 2) and {0,2} (0 / 2, clamped to 1); label 7 is out of range
    out = oracle.cloud_avg_degree(ns, ne, batch=[1, 0, 1, 0, 7], num_clouds=2)
    assert out.tolist() == [1.0, 4.5, 1.0, 4.5, 1.0]
    assert oracle.cloud_avg_degree(ns, ne).tolist() == [2.0] * 5


def _oracle_hybrid(oracle, x, ptr, r, K, kf):
    rp, src = oracle.radius_graph(x, ptr, r, K, dist=oracle.DIST_TORCH)
    knn_idx, knn_d = oracle.knn(x, x, ptr, ptr, kf + 1, dist=oracle.DIST_TORCH)
    return oracle.hybrid_graph(rp, src, knn_idx, kf), rp


@pytest.mark.parametrize("tag", ["nobatch", "batch"])
def test_hybrid_graph(gg, oracle, tag):
    """_EncoderStage._build_hybrid_graph: same edges in the same (row, col) order, same CSR."""
    x = gg["hyb_x"]
    K, kf, _ = (int(v) for v in gg["hyb_meta"])
    r = float(gg["hyb_r"][0])
    ptr = np.array([0, 200, 400, 600])
    (row, col), rp = _oracle_hybrid(oracle, x, ptr, r, K, kf)
    t = f"hyb_{tag}_"
    assert np.array_equal(row, gg[t + "row"]) and np.array_equal(col, gg[t + "col"])
    # the fixture exercises the fallback: isolated nodes exist and gained edges both ways
    assert (np.diff(rp) < kf).sum() > 50 and row.shape[0] > rp[-1]
    cs, pm, ns, ne = oracle.sort_and_build_csr(col, x.shape[0])
    assert np.array_equal(cs, gg[t + "col_sorted"])
    assert same_csr(ns, ne, gg[t + "node_start"], gg[t + "node_end"])
    for a, b in zip(ns, ne):  # the CPU argsort is unstable: same slots per segment
        assert sorted(pm[a:b].tolist()) == sorted(gg[t + "perm"][a:b].tolist())
    _, dist, _, _ = oracle.edge_geometry(x, row, col)
    assert bits_equal(dist, gg[t + "dist"])
    batch = np.repeat(np.arange(3), 200) if tag == "batch" else None
    avg = oracle.cloud_avg_degree(ns, ne, batch=batch, num_clouds=3 if tag == "batch" else None)
    if tag == "batch":
        assert bits_equal(avg, gg[t + "avg_degree"])
    else:
        assert np.allclose(avg, gg[t + "avg_degree"], rtol=2e-7, atol=0)


def test_adaptive_radius(gg, oracle):
    x = gg["hyb_x"]
    ptr = np.array([0, 200, 400, 600])
    _, d = oracle.knn(x, x, ptr, ptr, 2, dist=oracle.DIST_TORCH)
    est = np.sqrt(np.clip(d[:, 1].astype(np.float64), 1e-8, 1e20)).mean() * 4.0
    assert abs(est - gg["hyb_adaptive_radius"][0]) <= 1e-6 * est
