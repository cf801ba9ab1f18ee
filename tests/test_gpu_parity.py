"""GPU parity of every operator against the CPU checker (oracle/), through the C ABI.

Integer outputs (FPS / KNN / radius indices, CSR arrays) and segment max must be
bit-identical; so must the segment sum of segments up to 4096 slots (same sequential fp32
fold as the reference kernel). Longer segments use a fixed-order tree: |err| <= 1e-5 *
sum|x| + 1e-6. Mean: 1e-5 relative (fp32); bf16 inputs: 1e-2. Sizes are chosen so the
CPU checker finishes in seconds; full-size configurations are checked through
size-independent properties.
"""

import numpy as np
import pytest
import torch

from gdl_b200 import csrc, synthetic
from gdl_b200 import functional as F
from tests.golden import inputs

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = "cuda"


def _rand_clouds(seed, sizes, kind="uniform"):
    rng = np.random.default_rng(seed)
    n = int(sum(sizes))
    if kind == "lattice":
        x = rng.integers(0, 6, (n, 3)).astype(np.float32) * 0.25
    else:
        x = (rng.random((n, 3), dtype=np.float32) * 2 - 1).astype(np.float32)
    return x, synthetic.ptr_of(sizes)


# ----------------------------------------------------------------------------- FPS
@pytest.mark.parametrize("tie", ["reference", "lowest_index"])
@pytest.mark.parametrize("sizes,k", [([2048] * 4, 512), ([1, 2, 3, 600, 0, 1025], 300), ([4097, 8192], 1000),
                                     ([20000], 300), ([9000, 30000, 13824, 13825], 200), ([140000], 64),
                                     ([222000], 48)])
@pytest.mark.parametrize("kind", ["uniform", "lattice"])
def test_fps_matches_oracle(oracle, tie, sizes, k, kind):
    x, ptr = _rand_clouds(sum(sizes) + k, sizes, kind)
    kk = np.minimum(np.diff(ptr), k)
    kk[0] = kk[0] + 3  # one cloud asks for more than it has when small
    tmode = oracle.TIE_REFERENCE if tie == "reference" else oracle.TIE_LOWEST_INDEX
    want = oracle.fps(x, ptr, kk, tie=tmode, dist=oracle.DIST_CUDA)
    got = csrc.fps_cuda(torch.from_numpy(x).to(DEV), torch.from_numpy(ptr), torch.from_numpy(kk), tie_break=tie)
    assert np.array_equal(got.cpu().numpy(), want)


def test_fps_golden_config1(golden):
    pos, ptr = inputs.config1_points()
    got = F.farthest_point_sampling(torch.from_numpy(pos).to(DEV), 512, ptr=torch.from_numpy(ptr).to(DEV),
                                    tie_break="lowest_index")
    assert np.array_equal(got.cpu().numpy(), golden["fps_c1_idx"])


def test_fps_api_paths(golden):
    pv = torch.from_numpy(golden["fps_var_pos"]).to(DEV)
    pp = torch.from_numpy(golden["fps_var_ptr"]).to(DEV)
    assert np.array_equal(F.farthest_point_sampling(pv, 64, ptr=pp, tie_break="lowest_index").cpu().numpy(),
                          golden["fps_var_idx"])
    assert np.array_equal(F.farthest_point_sampling(pv[:300], 50, tie_break="lowest_index").cpu().numpy(),
                          golden["fps_single_idx"])
    assert torch.equal(F.farthest_point_sampling(pv[:10], 50).cpu(), torch.arange(10))
    # legacy batch vector, unsorted: per cloud in cloud order, small clouds -> arange
    batch = torch.tensor([1, 0, 1, 1, 0, 2] * 20, device=DEV)
    x = torch.rand(120, 3, device=DEV)
    out = F.farthest_point_sampling(x, 30, batch=batch).cpu()
    assert out.numel() == 30 + 30 + 20
    assert torch.equal(out[60:], torch.nonzero(batch.cpu() == 2).flatten())


def test_fps_full_size_prefix(oracle):
    """config 5 scale: one 131072-point LiDAR cloud, first 300 picks vs the checker."""
    x, ptr = synthetic.c5_points(B=1)
    got = csrc.fps_cuda(torch.from_numpy(x).to(DEV), torch.from_numpy(ptr), torch.tensor([300])).cpu().numpy()
    want = oracle.fps(x, ptr, [300], dist=oracle.DIST_CUDA)
    assert np.array_equal(got, want)


# ----------------------------------------------------------------------------- KNN
@pytest.mark.parametrize("k", [1, 3, 8, 16, 17, 32, 64, 70])
@pytest.mark.parametrize("kind", ["uniform", "lattice"])
def test_knn_matches_oracle(oracle, k, kind):
    x, ps = _rand_clouds(k, [700, 0, 5, 2500], kind)
    q, pq = _rand_clouds(k + 1, [100, 7, 3, 900], kind)
    wi, wd = oracle.knn(q, x, pq, ps, k, dist=oracle.DIST_CUDA)
    gi, gd = csrc.knn_cuda(torch.from_numpy(q).to(DEV), torch.from_numpy(x).to(DEV), torch.from_numpy(pq).to(DEV),
                           torch.from_numpy(ps).to(DEV), k)
    assert np.array_equal(gi.cpu().numpy(), wi)
    assert np.array_equal(gd.cpu().numpy().view(np.uint32), wd.view(np.uint32))


def test_knn_golden_config1(golden, oracle):
    pos, ptr = inputs.config1_points()
    q = pos[golden["fps_c1_idx"].astype(np.int64)]
    pq = np.arange(0, 2049, 512)
    gi, gd = F.knn(torch.from_numpy(q).to(DEV), torch.from_numpy(pos).to(DEV), torch.from_numpy(pq).to(DEV),
                   torch.from_numpy(ptr).to(DEV), 16)
    assert np.array_equal(gi.cpu().numpy(), golden["knn_c1_idx"])
    _, wd = oracle.knn(q, pos, pq, ptr, 16, dist=oracle.DIST_CUDA)
    assert np.array_equal(gd.cpu().numpy(), wd)


def test_knn_queries_outside_clouds_and_self():
    x = torch.rand(50, 3, device=DEV)
    i, d = csrc.knn_cuda(x, x, torch.tensor([10, 30], device=DEV), torch.tensor([10, 30], device=DEV), 4)
    assert (i[:10] == -1).all() and (i[30:] == -1).all() and (d[:10] == 1e30).all()
    i, d = F.knn_self(x, torch.tensor([0, 50], device=DEV), 3)
    assert torch.equal(i[:, 0].cpu(), torch.arange(50)) and (d[:, 0] == 0).all()


def test_knn_full_size_config4_sample(oracle):
    """config 4 scale (16384 x 16384 per cloud, k=1) for 2 clouds; checker on 512 queries."""
    src, tgt, ptr = synthetic.c4_pairs(B=2)
    gi, gd = csrc.knn_cuda(torch.from_numpy(tgt).to(DEV), torch.from_numpy(src).to(DEV), torch.from_numpy(ptr).to(DEV),
                           torch.from_numpy(ptr).to(DEV), 1)
    sel = np.r_[0:256, 16384:16384 + 256]
    wi, wd = oracle.knn(tgt[sel], src, np.array([0, 256, 512]), ptr, 1, dist=oracle.DIST_CUDA)
    assert np.array_equal(gi.cpu().numpy()[sel], wi)
    assert np.array_equal(gd.cpu().numpy()[sel], wd)


# ----------------------------------------------------------------------------- radius graph
@pytest.mark.parametrize("max_nn", [16, 20, 32, 64])
@pytest.mark.parametrize("loop", [False, True])
@pytest.mark.parametrize("kind", ["uniform", "lattice"])
@pytest.mark.parametrize("path", ["fused", "general"])
def test_radius_matches_oracle(oracle, max_nn, loop, kind, path):
    sizes = [1, 0, 400, 2500, 3000] if path == "fused" else [1, 0, 400, 2500, 9000]
    x, ptr = _rand_clouds(max_nn, sizes, kind)
    rng = np.random.default_rng(1)
    mask = rng.random(x.shape[0]) > 0.1
    for r in (0.12, 0.35):
        for m in (None, mask):
            wrp, wsrc = oracle.radius_graph(x, ptr, r, max_nn, loop, m, dist=oracle.DIST_CUDA)
            # a CPU ptr tells the wrapper the largest cloud (fused kernels up to 4096 points)
            pt = torch.from_numpy(ptr) if path == "fused" else torch.from_numpy(ptr).to(DEV)
            rp, src, dst = csrc.radius_graph_csr(torch.from_numpy(x).to(DEV), r, pt,
                                                 max_num_neighbors=max_nn, loop=loop,
                                                 mask=None if m is None else torch.from_numpy(m).to(DEV))
            rp = rp.cpu().numpy()
            E = rp[-1]
            assert np.array_equal(rp, wrp)
            assert np.array_equal(src.cpu().numpy()[:E], wsrc)
            assert np.array_equal(dst.cpu().numpy()[:E], np.repeat(np.arange(x.shape[0]), np.diff(wrp)))


@pytest.mark.parametrize("max_nn", [16, 64])
@pytest.mark.parametrize("loop", [False, True])
def test_radius_dense_rows_match_oracle(oracle, max_nn, loop):
    """Rows with far more than 1024 sources in range on the general path (clouds over 4096
    points): a tight ball, stacks of duplicated points and a fine lattice among spread points, so
    that a query warp bounds its selection many times over, skips the cells beyond the bound and
    meets ties at the cut (the heap replay), with and without a mask."""
    rng = np.random.default_rng(7)
    ball = rng.normal(0.0, 0.06, (3000, 3))
    dup = np.repeat(rng.random((3, 3)) * 0.4, 500, axis=0)
    lat = rng.integers(0, 8, (2500, 3)) * 0.05
    spread = rng.random((3000, 3)) * 2 - 1
    x = np.concatenate([ball, dup, lat, spread]).astype(np.float32)
    x = np.ascontiguousarray(x[rng.permutation(len(x))])
    ptr = synthetic.ptr_of([len(x) - 4500, 4500])
    mask = rng.random(len(x)) > 0.05
    for r in (0.1, 0.3):
        for m in (None, mask):
            wrp, wsrc = oracle.radius_graph(x, ptr, r, max_nn, loop, m, dist=oracle.DIST_CUDA)
            rp, src, _ = csrc.radius_graph_csr(torch.from_numpy(x).to(DEV), r, torch.from_numpy(ptr).to(DEV),
                                               max_num_neighbors=max_nn, loop=loop,
                                               mask=None if m is None else torch.from_numpy(m).to(DEV))
            rp = rp.cpu().numpy()
            assert np.array_equal(rp, wrp), (r, m is not None)
            assert np.array_equal(src.cpu().numpy()[:rp[-1]], wsrc), (r, m is not None)


@pytest.mark.parametrize("extent", [40.0, 400.0])
def test_radius_sparse_grids_match_oracle(oracle, extent):
    """Clouds whose grids have many more cells than points (clusters spread over a wide box):
    a 40 m box keeps a table of the grid's (x, y) columns, a 400 m box has none and searches the
    sorted cell keys directly."""
    rng = np.random.default_rng(int(extent))
    centres = rng.random((600, 3)) * np.array([extent, extent, 10.0])
    x = (np.repeat(centres, 10, axis=0) + rng.normal(0.0, 0.3, (6000, 3))).astype(np.float32)
    ptr = synthetic.ptr_of([6000])
    for max_nn in (16, 64):
        wrp, wsrc = oracle.radius_graph(x, ptr, 0.5, max_nn, False, None, dist=oracle.DIST_CUDA)
        rp, src, _ = csrc.radius_graph_csr(torch.from_numpy(x).to(DEV), 0.5, torch.from_numpy(ptr).to(DEV),
                                           max_num_neighbors=max_nn)
        rp = rp.cpu().numpy()
        assert rp[-1] > 10000
        assert np.array_equal(rp, wrp)
        assert np.array_equal(src.cpu().numpy()[:rp[-1]], wsrc)


def test_radius_golden_and_kat(golden):
    x = torch.from_numpy(golden["rad_x"]).to(DEV)
    B, n, K = (int(v) for v in golden["rad_meta"])
    r = float(golden["rad_r"][0])
    batch = torch.arange(B, device=DEV).repeat_interleave(n)
    for loop in (False, True):
        for um in (False, True):
            m = torch.from_numpy(golden["rad_mask"]).to(DEV) if um else None
            row, col = F.radius_graph(x, r, max_num_neighbors=K, batch=batch, loop=loop, mask=m)
            tag = f"rad_b_loop{int(loop)}_mask{int(um)}"
            got = set(zip(row.tolist(), col.tolist()))
            want = set(zip(golden[tag + "_row"].tolist(), golden[tag + "_col"].tolist()))
            assert got == want
    kat = torch.tensor([[0.0, 0.0, 0.0], [0.1, 0.0, 0.0], [10.0, 0.0, 0.0]], device=DEV)
    row, col = F.radius_graph(kat, r=1.0)
    assert sorted(zip(row.tolist(), col.tolist())) == [(0, 1), (1, 0)]
    two = torch.tensor([[0.0, 0.0, 0.0], [0.1, 0.0, 0.0]], device=DEV)
    row, _ = F.radius_graph(two, r=100.0, batch=torch.tensor([0, 1], device=DEV))
    assert row.numel() == 0
    row, _ = F.radius_graph(torch.randn(20, 3, device=DEV) * 10, r=0.001)
    assert row.numel() == 0
    # unsorted batch vector maps back to the caller's indices
    perm = torch.randperm(B * n, device=DEV)
    row2, col2 = F.radius_graph(x[perm], r, max_num_neighbors=K, batch=batch[perm])
    got = set(zip(perm[row2].tolist(), perm[col2].tolist()))
    want = set(zip(golden["rad_b_loop0_mask0_row"].tolist(), golden["rad_b_loop0_mask0_col"].tolist()))
    assert got == want


def test_radius_full_size_config2_properties(oracle):
    """config 2: FPS centroids, r=0.2, 32 neighbours; CSR sorted, symmetric where untruncated."""
    pos, ptr = synthetic.c2_points()
    idx = csrc.fps_cuda(torch.from_numpy(pos).to(DEV), torch.from_numpy(ptr), torch.full((16,), 512))
    cent = torch.from_numpy(pos).to(DEV)[idx]
    cptr = torch.arange(0, 16 * 512 + 1, 512, device=DEV)
    rp, src, _ = csrc.radius_graph_csr(cent, 0.2, cptr, max_num_neighbors=32)
    wrp, wsrc = oracle.radius_graph(cent.cpu().numpy(), cptr.cpu().numpy(), 0.2, 32, dist=oracle.DIST_CUDA)
    assert np.array_equal(rp.cpu().numpy(), wrp) and np.array_equal(src.cpu().numpy()[:wrp[-1]], wsrc)


# ----------------------------------------------------------------------------- CSR + segment reduce
@pytest.mark.parametrize("N,E", [(500, 3000), (1, 10), (70000, 300000), (10, 0), (3, 20000)])
def test_csr_matches_oracle(oracle, N, E):
    rng = np.random.default_rng(N + E)
    col = rng.integers(0, N, E)
    got = csrc.sort_and_build_csr_cuda(torch.from_numpy(col).to(DEV), N)
    want = oracle.sort_and_build_csr(col, N)
    for a, b in zip(got, want):
        assert np.array_equal(a.cpu().numpy(), b)


@pytest.mark.parametrize("C", [1, 6, 16, 32, 64, 128, 256])
@pytest.mark.parametrize("reduce", ["sum", "mean", "max"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_segment_matches_oracle(oracle, C, reduce, dtype):
    rng = np.random.default_rng(C)
    N, E = 700, 5000
    col = rng.integers(0, N, E)
    msg = rng.standard_normal((E, C)).astype(np.float32)
    msg[3] = msg[4]
    col[3] = col[4]
    cs, pm, ns, ne = oracle.sort_and_build_csr(col, N)
    m_np = oracle.bf16_bits(msg) if dtype == "bf16" else msg
    want = oracle.segment_reduce(m_np, pm, ns, ne, N, reduce)
    m_t = torch.from_numpy(msg).to(DEV)
    if dtype == "bf16":
        m_t = m_t.to(torch.bfloat16)
    args = [torch.from_numpy(a).to(DEV) for a in (cs, pm, ns, ne)]
    got = csrc.segment_reduce_cuda(m_t, args[1], args[2], args[3], N, reduce).cpu().numpy()
    if reduce == "mean":
        assert np.allclose(got, want, rtol=1e-5, atol=1e-6)
    else:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # backward through the autograd op vs the checker's backward
    gout = rng.standard_normal((N, C)).astype(np.float32)
    m_t.requires_grad_(True)
    out = F.segment_reduce(m_t, *args, N, reduce=reduce)
    out.backward(torch.from_numpy(gout).to(DEV))
    wg = oracle.segment_reduce_backward(gout, m_np, want, pm, ns, ne, N, reduce)
    gg = m_t.grad
    if dtype == "bf16":
        assert np.array_equal(gg.view(torch.int16).cpu().numpy().view(np.uint16), wg)
    else:
        assert np.array_equal(gg.cpu().numpy().view(np.uint32), wg.view(np.uint32))


@pytest.mark.parametrize("reduce", ["sum", "mean", "max"])
def test_segment_long_segments(oracle, reduce):
    """config 4 shape: 64 segments x 16384 rows, C=6, identity perm."""
    rng = np.random.default_rng(4)
    N, L, C = 64, 16384, 6
    msg = rng.standard_normal((N * L, C)).astype(np.float32)
    ns = (np.arange(N) * L).astype(np.int32)
    ne = ns + L
    want = oracle.segment_reduce(msg, None, ns, ne, N, reduce)
    got = csrc.segment_reduce_cuda(torch.from_numpy(msg).to(DEV), None, torch.from_numpy(ns).to(DEV),
                                   torch.from_numpy(ne).to(DEV), N, reduce).cpu().numpy()
    if reduce == "max":
        assert np.array_equal(got, want)
    else:
        scale = np.abs(msg).reshape(N, L, C).sum(1) / (L if reduce == "mean" else 1)
        assert np.all(np.abs(got - want) <= 1e-5 * scale + 1e-6)
    # deterministic run to run
    again = csrc.segment_reduce_cuda(torch.from_numpy(msg).to(DEV), None, torch.from_numpy(ns).to(DEV),
                                     torch.from_numpy(ne).to(DEV), N, reduce).cpu().numpy()
    assert np.array_equal(again.view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("reduce", ["sum", "max"])
def test_segment_long_queue_overflow(oracle, reduce):
    """More slots than rows (perm gathers rows repeatedly): more long segments than the queue
    was sized for; the overflow is folded in place (sum in reference order, bit-exact)."""
    rng = np.random.default_rng(9)
    rows, C = 300, 8
    msg = rng.standard_normal((rows, C)).astype(np.float32)
    lens = [5000, 4500, 6000, 3, 0, 7000]
    ns = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int32)
    ne = (ns + np.array(lens)).astype(np.int32)
    perm = rng.integers(0, rows, int(sum(lens))).astype(np.int32)
    want = oracle.segment_reduce(msg, perm, ns, ne, len(lens), reduce)
    got = csrc.segment_reduce_cuda(torch.from_numpy(msg).to(DEV), torch.from_numpy(perm).to(DEV),
                                   torch.from_numpy(ns).to(DEV), torch.from_numpy(ne).to(DEV), len(lens),
                                   reduce).cpu().numpy()
    if reduce == "max":
        assert np.array_equal(got, want)
    else:
        scale = np.array([np.abs(msg[perm[a:b]]).sum(0) for a, b in zip(ns, ne)])
        assert np.all(np.abs(got - want) <= 1e-5 * scale + 1e-6)


def test_segment_golden_and_reference_kats(golden, oracle):
    col = torch.from_numpy(golden["seg_r_col"]).to(DEV)
    msg = torch.from_numpy(golden["seg_r_msg"]).to(DEV)
    cs, pm, ns, ne = F.sort_and_build_csr(col, 500)
    # sum of the reference CPU path, replayed with its own (unstable) perm: bit-exact
    gp = torch.from_numpy(golden["seg_r_perm"]).to(DEV)
    out = csrc.segment_reduce_cuda(msg, gp, ns, ne, 500, "sum").cpu().numpy()
    assert np.array_equal(out, golden["seg_r_sum"])
    for red in ("mean", "max"):
        m = msg.clone().requires_grad_(True)
        o = F.segment_reduce(m, cs, pm, ns, ne, 500, reduce=red)
        o.backward(torch.from_numpy(golden["seg_r_gout"]).to(DEV))
        assert np.array_equal(o.detach().cpu().numpy(), golden[f"seg_r_{red}_f32"])
        assert np.array_equal(m.grad.cpu().numpy(), golden[f"seg_r_{red}_f32_grad"])
    # tests/test_segment_reduce.py KATs: single node, empty, backward of sum = ones, determinism
    c0 = torch.zeros(10, dtype=torch.long, device=DEV)
    o = F.segment_reduce(torch.ones(10, 4, device=DEV), *F.sort_and_build_csr(c0, 1), 1)
    assert torch.equal(o.cpu(), torch.full((1, 4), 10.0))
    e = F.sort_and_build_csr(torch.empty(0, dtype=torch.long, device=DEV), 10)
    o = F.segment_reduce(torch.empty(0, 8, device=DEV), *e, 10)
    assert o.shape == (10, 8) and o.abs().sum() == 0
    col = torch.randint(0, 50, (200,), device=DEV)
    m = torch.randn(200, 8, device=DEV, requires_grad=True)
    F.segment_reduce(m, *F.sort_and_build_csr(col, 50), 50).sum().backward()
    assert torch.equal(m.grad, torch.ones_like(m))
    csr = F.sort_and_build_csr(col, 50)
    first = F.segment_reduce(m.detach(), *csr, 50)
    for _ in range(19):
        assert torch.equal(F.segment_reduce(m.detach(), *csr, 50), first)


def test_segment_matches_scatter_add():
    """tests/test_segment_reduce.py:34-53: vs scatter_add_ within 1e-5."""
    torch.manual_seed(42)
    N, E, C = 500, 3000, 32
    col = torch.randint(0, N, (E,), device=DEV)
    msg = torch.randn(E, C, device=DEV)
    ref = torch.zeros(N, C, device=DEV).scatter_add_(0, col.unsqueeze(-1).expand(E, C), msg)
    out = F.segment_reduce(msg, *F.sort_and_build_csr(col, N), N)
    assert torch.allclose(out, ref, atol=1e-5)
