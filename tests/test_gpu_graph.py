"""GPU parity of the graph geometry row: edge vectors, distances, directions and spherical
harmonics written by the radius graph's emission kernel (gdl_radius_graph_geometry), the same
values over COO edges (gdl_edge_geometry_coo), the sort-free CSR fields and per-cloud average
degree (gdl_radius_csr_finish, gdl_cloud_avg_degree), and SpatialGraph built on them.

Everything is bit-exact against the CPU checker (oracle/), which is itself pinned bit-exact
against the reference's CPU path in tests/test_oracle_graph.py; the golden fixtures of the
reference's SpatialGraph are compared directly as well (edge lists as sets: the reference's
edge order is its atomic counter's). The one tolerance: SpatialGraph.build without a batch
vector averages with the reference's ``degree.mean()``, matched to 2e-7 relative.
"""

import numpy as np
import pytest
import torch

from gdl_b200 import csrc, synthetic
from gdl_b200 import functional as F
from gdl_b200.spatial_graph import SpatialGraph
from tests.test_oracle_graph import bits_equal, by_edge, same_csr

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = "cuda"


@pytest.fixture(scope="module")
def gg():
    from tests.conftest import ROOT

    return np.load(ROOT / "tests" / "golden" / "golden_graph.npz")


def _clouds(seed, sizes, scale=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.random((int(sum(sizes)), 3), dtype=np.float32) * scale).astype(np.float32)
    return x, synthetic.ptr_of(sizes)


@pytest.mark.parametrize("path", ["fused", "general"])
@pytest.mark.parametrize("max_l", [None, 0, 1, 2])
def test_radius_geometry_matches_oracle(oracle, path, max_l):
    sizes = [0, 1, 700, 3000, 2500] if path == "fused" else [0, 1, 700, 3000, 9000]
    x, ptr = _clouds(17, sizes)
    rng = np.random.default_rng(3)
    mask = rng.random(x.shape[0]) > 0.05
    for r, K, m in ((0.08, 32, None), (0.15, 16, mask), (0.11, 64, None)):
        pt = torch.from_numpy(ptr) if path == "fused" else torch.from_numpy(ptr).to(DEV)
        xd = torch.from_numpy(x).to(DEV)
        out = csrc.radius_graph_geometry_csr(xd, r, pt, max_num_neighbors=K, max_l=max_l, with_diff=True,
                                             mask=None if m is None else torch.from_numpy(m).to(DEV))
        # identical edges to the plain radius graph
        rp, src, dst = csrc.radius_graph_csr(xd, r, pt, max_num_neighbors=K,
                                             mask=None if m is None else torch.from_numpy(m).to(DEV))
        E = int(rp[-1])
        assert torch.equal(out["row_ptr"], rp) and torch.equal(out["src"][:E], src[:E])
        assert torch.equal(out["dst"][:E], dst[:E])
        assert torch.equal(out["src32"][:E].long(), src[:E]) and torch.equal(out["row_ptr32"].long(), rp)
        row, col = src[:E].cpu().numpy(), dst[:E].cpu().numpy()
        diff, dist, direction, sph = oracle.edge_geometry(x, row, col, max_l=2 if max_l is None else max_l)
        assert bits_equal(out["diff"][:E].cpu().numpy(), diff)
        assert bits_equal(out["dist"][:E].cpu().numpy(), dist)
        assert bits_equal(out["direction"][:E].cpu().numpy(), direction)
        if max_l is None:
            assert out["sph"] is None
        else:
            assert bits_equal(out["sph"][:E].cpu().numpy(), sph)


def test_edge_geometry_coo_golden(gg):
    """Hand-made edges of the reference fixture: zero / tiny / overflowing / non-finite vectors."""
    x = torch.from_numpy(gg["geo_x"]).to(DEV)
    row = torch.from_numpy(gg["geo_row"]).to(DEV)
    col = torch.from_numpy(gg["geo_col"]).to(DEV)
    for lmax in (0, 1, 2):
        diff, dist, direction, sph = csrc.edge_geometry_cuda(x, row, col, max_l=lmax)
        assert bits_equal(diff.cpu().numpy(), gg["geo_diff"])
        assert bits_equal(dist.cpu().numpy(), gg["geo_dist"])
        assert bits_equal(direction.cpu().numpy(), gg["geo_dir"])
        assert bits_equal(sph.cpu().numpy(), gg[f"geo_Y{lmax}"])
    d2, n2, u2 = F.compute_edge_vectors(x, row, col)
    assert bits_equal(d2.cpu().numpy(), gg["geo_diff"]) and bits_equal(u2.cpu().numpy(), gg["geo_dir"])
    assert bits_equal(n2.cpu().numpy(), gg["geo_dist"])
    # out-of-range indices give NaN rows; no edges is a no-op
    bad = torch.tensor([0, x.shape[0]], device=DEV)
    _, dist, _, _ = csrc.edge_geometry_cuda(x, bad, torch.tensor([1, 1], device=DEV))
    assert np.isnan(dist.cpu().numpy()[1]) and not np.isnan(dist.cpu().numpy()[0])
    e = torch.empty(0, dtype=torch.int64, device=DEV)
    assert csrc.edge_geometry_cuda(x, e, e, max_l=2)[3].shape == (0, 9)


def test_edge_geometry_coo_large_matches_oracle(oracle):
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((50000, 3)) * 3).astype(np.float32)
    row = rng.integers(0, 50000, 400000)
    col = rng.integers(0, 50000, 400000)
    got = csrc.edge_geometry_cuda(torch.from_numpy(x).to(DEV), torch.from_numpy(row).to(DEV),
                                  torch.from_numpy(col).to(DEV), max_l=2)
    for a, b in zip(got, oracle.edge_geometry(x, row, col, max_l=2)):
        assert bits_equal(a.cpu().numpy(), b)


@pytest.mark.parametrize("case", ["batch", "single", "shuffled"])
def test_spatial_graph_build_golden(gg, case):
    x = gg["graph_x"]
    B, n, K, _ = (int(v) for v in gg["graph_meta"])
    r = float(gg["graph_r"][0])
    batch = np.repeat(np.arange(B), n)
    if case == "batch":
        pos, kw = x, dict(batch=torch.from_numpy(batch).to(DEV), num_batch_elements=B)
    elif case == "single":
        pos, kw = x[:n], {}
    else:
        sel, perm = gg["graph_sel"], gg["graph_perm"]
        pos, kw = x[sel][perm], dict(batch=torch.from_numpy(batch[sel][perm]).to(DEV))
    g = SpatialGraph.build(torch.from_numpy(pos).to(DEV), r, max_num_neighbors=K, **kw)
    t = f"graph_{case}_"
    assert g.E == gg[t + "row"].shape[0] and g.N == pos.shape[0]
    got = by_edge(g.row.cpu().numpy(), g.col.cpu().numpy(), g.dist.cpu().numpy(), g.direction.cpu().numpy(),
                  g.Y.cpu().numpy())
    ref = by_edge(gg[t + "row"], gg[t + "col"], gg[t + "dist"], gg[t + "direction"], gg[t + "Y"])
    assert np.array_equal(got[0], ref[0]) and np.array_equal(got[1], ref[1])
    for a, b in zip(got[2:], ref[2:]):
        assert bits_equal(a, b)
    assert same_csr(g.node_start.cpu().numpy(), g.node_end.cpu().numpy(), gg[t + "node_start"], gg[t + "node_end"])
    # CSR consistency: col_sorted[perm] slots point at edges whose col is that destination
    cs, pm = g.col_sorted.cpu().numpy(), g.perm.cpu().numpy().astype(np.int64)
    assert np.all(np.diff(cs) >= 0) and np.array_equal(g.col.cpu().numpy()[pm], cs)
    avg = g.avg_degree.cpu().numpy()
    if case == "single":
        assert np.allclose(avg, gg[t + "avg_degree"], rtol=2e-7, atol=0)
    else:
        assert bits_equal(avg, gg[t + "avg_degree"])


def test_spatial_graph_from_edge_index_golden(gg):
    x = torch.from_numpy(gg["graph_x"]).to(DEV)
    B, n, _, _ = (int(v) for v in gg["graph_meta"])
    row = torch.from_numpy(gg["graph_batch_row"]).to(DEV)
    col = torch.from_numpy(gg["graph_batch_col"]).to(DEV)
    batch = torch.arange(B, device=DEV).repeat_interleave(n)
    g = SpatialGraph.from_edge_index(row, col, x, B * n, max_l=1, batch=batch, num_batch_elements=B)
    assert np.array_equal(g.col_sorted.cpu().numpy(), gg["graph_fei_col_sorted"])
    assert same_csr(g.node_start.cpu().numpy(), g.node_end.cpu().numpy(), gg["graph_fei_node_start"],
                    gg["graph_fei_node_end"])
    assert bits_equal(g.avg_degree.cpu().numpy(), gg["graph_fei_avg_degree"])
    assert bits_equal(g.Y.cpu().numpy(), gg["graph_fei_Y"])
    # no edges: the empty graph of the reference (avg degree 1)
    e = torch.empty(0, dtype=torch.int64, device=DEV)
    g0 = SpatialGraph.from_edge_index(e, e, x, B * n)
    assert g0.E == 0 and g0.Y.shape == (0, 9) and torch.all(g0.avg_degree == 1)


def test_radius_csr_finish_and_avg_degree(oracle):
    x, ptr = _clouds(5, [0, 500, 3, 4000, 1200])
    xd = torch.from_numpy(x).to(DEV)
    rp, src, dst = csrc.radius_graph_csr(xd, 0.09, torch.from_numpy(ptr), max_num_neighbors=32)
    N = x.shape[0]
    E = int(rp[-1])
    pd = torch.from_numpy(ptr).to(DEV)
    for p in (pd, None):
        cs, pm, ns, ne, avg = csrc.radius_csr_finish(rp, dst, N, ptr=p)
        col = dst[:E].cpu().numpy()
        wcs, wpm, wns, wne = oracle.sort_and_build_csr(col, N)
        assert np.array_equal(cs[:E].cpu().numpy(), wcs) and np.array_equal(pm[:E].cpu().numpy(), wpm)
        assert np.array_equal(ns.cpu().numpy(), wns) and np.array_equal(ne.cpu().numpy(), wne)
        want = oracle.cloud_avg_degree(wns, wne, ptr=None if p is None else ptr)
        assert bits_equal(avg.cpu().numpy(), want)
        # the general entry point agrees, with clouds from ptr, a batch vector, or one cloud
        if p is not None:
            bt = torch.from_numpy(np.repeat(np.arange(len(ptr) - 1), np.diff(ptr))).to(DEV)
            a2 = csrc.cloud_avg_degree_cuda(ns, ne, batch=bt, num_clouds=len(ptr) - 1)
            a3 = csrc.cloud_avg_degree_cuda(ns, ne, ptr=pd)
            assert bits_equal(a2.cpu().numpy(), want) and bits_equal(a3.cpu().numpy(), want)
        else:
            assert bits_equal(csrc.cloud_avg_degree_cuda(ns, ne).cpu().numpy(), want)
    # shuffled labels, one label out of range
    rng = np.random.default_rng(2)
    labels = rng.integers(0, 4, N)
    labels[7] = 11
    a = csrc.cloud_avg_degree_cuda(ns, ne, batch=torch.from_numpy(labels).to(DEV), num_clouds=4)
    want = oracle.cloud_avg_degree(ns.cpu().numpy(), ne.cpu().numpy(), batch=labels, num_clouds=4)
    assert bits_equal(a.cpu().numpy(), want)


def test_spatial_graph_full_size_lidar_geometry(oracle):
    """Config 5 clouds, radius graph over all points of two clouds (the c5g workload):
    geometry per slot against the checker on a sample of destinations, exact CSR fields."""
    pos, ptr = synthetic.c5_points(B=2)
    xd = torch.from_numpy(pos).to(DEV)
    out = csrc.radius_graph_geometry_csr(xd, 1.0, torch.from_numpy(ptr), max_num_neighbors=64, max_l=2)
    rp = out["row_ptr"].cpu().numpy()
    E = int(rp[-1])
    assert E > 1_000_000
    src, dst = out["src"][:E].cpu().numpy(), out["dst"][:E].cpu().numpy()
    pick = np.random.default_rng(0).choice(E, 200_000, replace=False)
    diff, dist, direction, sph = oracle.edge_geometry(pos, src[pick], dst[pick], max_l=2)
    assert bits_equal(out["dist"][:E].cpu().numpy()[pick], dist)
    assert bits_equal(out["direction"][:E].cpu().numpy()[pick], direction)
    assert bits_equal(out["sph"][:E].cpu().numpy()[pick], sph)
    assert float(out["dist"][:E].max()) < 1.0
    # the COO entry point over the same edges writes the same bits on every edge
    _, d2, u2, y2 = csrc.edge_geometry_cuda(xd, out["src"][:E], out["dst"][:E], max_l=2, with_diff=False)
    assert torch.equal(d2.view(torch.int32), out["dist"][:E].view(torch.int32))
    assert torch.equal(u2.view(torch.int32), out["direction"][:E].view(torch.int32))
    assert torch.equal(y2.view(torch.int32), out["sph"][:E].view(torch.int32))


# ------------------------------------------------------------------------- hybrid graph
from gdl_b200.hybrid_graph import HybridGraphBuilder, build_hybrid_graph, estimate_adaptive_radius  # noqa: E402


@pytest.mark.parametrize("tag", ["nobatch", "batch"])
def test_hybrid_graph_golden(gg, oracle, tag):
    x = gg["hyb_x"]
    K, kf, _ = (int(v) for v in gg["hyb_meta"])
    r = float(gg["hyb_r"][0])
    ptr = torch.tensor([0, 200, 400, 600])
    batch = torch.arange(3, device=DEV).repeat_interleave(200) if tag == "batch" else None
    g = HybridGraphBuilder(max_num_neighbors=K, knn_fallback_k=kf)._build_hybrid_graph(
        torch.from_numpy(x).to(DEV), r, ptr, batch)
    t = f"hyb_{tag}_"
    row, col = g.row.cpu().numpy(), g.col.cpu().numpy()
    assert np.array_equal(row, gg[t + "row"]) and np.array_equal(col, gg[t + "col"])  # same order too
    cs, pm, ns, ne = oracle.sort_and_build_csr(col, x.shape[0])  # stable, as the reference's CUDA sort
    assert np.array_equal(g.col_sorted.cpu().numpy(), cs) and np.array_equal(g.perm.cpu().numpy(), pm)
    assert np.array_equal(g.node_start.cpu().numpy(), ns) and np.array_equal(g.node_end.cpu().numpy(), ne)
    assert same_csr(ns, ne, gg[t + "node_start"], gg[t + "node_end"])
    _, dist, direction, sph = oracle.edge_geometry(x, row, col)
    assert bits_equal(g.dist.cpu().numpy(), dist) and bits_equal(g.dist.cpu().numpy(), gg[t + "dist"])
    assert bits_equal(g.direction.cpu().numpy(), direction) and bits_equal(g.Y.cpu().numpy(), sph)
    avg = g.avg_degree.cpu().numpy()
    if tag == "batch":
        assert bits_equal(avg, gg[t + "avg_degree"])
    else:
        assert np.allclose(avg, gg[t + "avg_degree"], rtol=2e-7, atol=0)
    est = estimate_adaptive_radius(torch.from_numpy(x).to(DEV), ptr.to(DEV), 4.0)
    assert abs(est - gg["hyb_adaptive_radius"][0]) <= 2e-6 * est


@pytest.mark.parametrize("kf", [0, 1, 3, 8])
@pytest.mark.parametrize("kind", ["uniform", "hub"])
def test_hybrid_graph_matches_oracle(oracle, kf, kind):
    rng = np.random.default_rng(kf + 10)
    if kind == "uniform":
        sizes = [1, 0, 300, 2000, 5000]
        x = rng.random((sum(sizes), 3)).astype(np.float32)
        r, K = 0.04, 16
    else:  # 300 copies of one point among scattered ones, no radius edges: rows far beyond 128
        sizes = [700, 50]
        x = rng.random((750, 3)).astype(np.float32) * 10
        x[100:400] = x[100]
        r, K = 0.0, 32
    ptr = synthetic.ptr_of(sizes)
    xd = torch.from_numpy(x).to(DEV)
    pt = torch.from_numpy(ptr)
    rp, src, _ = csrc.radius_graph_csr(xd, r, pt, max_num_neighbors=K, with_dst=False)
    knn_idx = csrc.knn_cuda(xd, xd, pt.to(DEV), pt.to(DEV), kf + 1)[0] if kf > 0 else None
    h = csrc.hybrid_graph_cuda(rp, src, knn_idx, x.shape[0], K, kf, x=xd, max_l=2)
    E = int(h["row_ptr"][-1])
    want_row, want_col = oracle.hybrid_graph(rp.cpu().numpy(), src.cpu().numpy(),
                                             None if knn_idx is None else knn_idx.cpu().numpy(), kf)
    assert E == want_row.shape[0]
    assert np.array_equal(h["row"][:E].cpu().numpy(), want_row) and np.array_equal(h["col"][:E].cpu().numpy(),
                                                                                    want_col)
    cs, pm, ns, ne = oracle.sort_and_build_csr(want_col, x.shape[0])
    assert np.array_equal(h["col_sorted"][:E].cpu().numpy(), cs) and np.array_equal(h["perm"][:E].cpu().numpy(), pm)
    assert np.array_equal(h["node_start"].cpu().numpy(), ns) and np.array_equal(h["node_end"].cpu().numpy(), ne)
    assert np.array_equal(h["src_sorted"][:E].cpu().numpy(), want_row[pm])
    _, dist, direction, sph = oracle.edge_geometry(x, want_row, want_col, max_l=2)
    assert bits_equal(h["dist"][:E].cpu().numpy(), dist) and bits_equal(h["direction"][:E].cpu().numpy(), direction)
    assert bits_equal(h["sph"][:E].cpu().numpy(), sph)
    if kind == "hub" and kf > 0:
        assert np.diff(h["row_ptr"].cpu().numpy()).max() > 128  # the one-lane sort path ran


def test_hybrid_graph_empty():
    e64 = torch.zeros(1, dtype=torch.int64, device=DEV)
    h = csrc.hybrid_graph_cuda(e64, e64, None, 0, 32, 3)
    assert int(h["row_ptr"][0]) == 0
