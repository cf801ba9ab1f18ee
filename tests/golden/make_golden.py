"""Generate golden vectors from the reference's own CPU code path.

Run in the build container, where the reference tree is importable:

    python tests/golden/make_golden.py [/path/to/reference]

It imports ``geoembodied`` read-only (PYTHONDONTWRITEBYTECODE) and records, for seeded
inputs, what the reference's public entry points return on the CPU:

* ``functional.fps.farthest_point_sampling`` (-> ``csrc._fps_iterative_fallback``)
* ``functional.knn.knn`` (-> ``csrc._knn_bruteforce``)
* ``functional.radius_graph.radius_graph`` (-> ``_radius_graph_single/_batched``)
* ``functional.segment_reduce.sort_and_build_csr`` / ``segment_reduce`` (+ autograd)
* ``torch.scatter_reduce(include_self=False)`` mean/amax (+ autograd), the semantics
  the reference's callers use for segment mean/max.
* ``nn.modules.spatial_graph.SpatialGraph.build`` / ``from_edge_index`` and
  ``functional.radius_graph.compute_edge_vectors`` + the spherical harmonics' torch path
  (``kernels.triton_sph_harm._spherical_harmonics_pytorch``) -> ``golden_graph.npz``.
* ``nn.modules.multi_scale_se3_net._EncoderStage._build_hybrid_graph`` / ``_estimate_adaptive_radius``
  -> ``golden_graph.npz`` (``hyb_*``).
* ``nn.modules.se3_conv.SE3Conv`` forward/backward over a reference-built graph -> ``golden_se3.npz``.
* ``nn.modules.equivariant_interp.EquivariantInterpolate`` forward/backward and the weighted-sum
  lines of ``EquivariantPool`` -> ``golden_aggregate.npz``.

Inputs that would make the CPU path and the CUDA kernels disagree for reasons the
reference itself documents (exact distance ties, pairs at the radius boundary where
``cdist``'s matmul rounding differs, radius truncation by near-tied distances) are
rejected and re-drawn, so each fixture pins the restated algorithm unambiguously.
Large arrays are regenerated from their seed in the tests; the fixtures hold the
outputs (and small inputs) only.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
sys.dont_write_bytecode = True

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import torch  # noqa: E402

from tests.golden import inputs  # noqa: E402


def _ref(root: str):
    sys.path.insert(0, root)
    import importlib

    mods = [importlib.import_module(f"geoembodied.functional.{m}") for m in ("fps", "knn", "radius_graph",
                                                                           "segment_reduce")]
    return tuple(mods)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def strictly_increasing_rows(d: np.ndarray, valid: np.ndarray) -> bool:
    for r in range(d.shape[0]):
        v = d[r][valid[r]]
        if v.size > 1 and not np.all(np.diff(v.astype(np.float64)) > 0):
            return False
    return True


def gen_fps(F, out):
    # config 1: B=4 x N=2048 U[-1,1]^3 seed 0, FPS -> 512 (ptr path)
    pos, ptr = inputs.config1_points()
    idx = F.farthest_point_sampling(torch.from_numpy(pos), 512, ptr=torch.from_numpy(ptr))
    out["fps_c1_idx"] = idx.numpy().astype(np.int32)
    # variable-size clouds, k < n everywhere (k >= n takes an arange shortcut on the CPU
    # path only, csrc/__init__.py:634-636)
    g = torch.Generator().manual_seed(7)
    sizes = [300, 257, 97, 1030]
    posv = (torch.randn(sum(sizes), 3, generator=g) * 0.7).numpy().astype(np.float32)
    ptrv = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    idxv = F.farthest_point_sampling(torch.from_numpy(posv), 64, ptr=torch.from_numpy(ptrv))
    out["fps_var_pos"] = posv
    out["fps_var_ptr"] = ptrv
    out["fps_var_idx"] = idxv.numpy().astype(np.int32)
    # single cloud path (functional/fps.py:121-162)
    poss = posv[:300]
    out["fps_single_idx"] = F.farthest_point_sampling(torch.from_numpy(poss), 50).numpy().astype(np.int32)


def gen_knn(K, out, fps_idx):
    pos, ptr = inputs.config1_points()
    q = pos[fps_idx.astype(np.int64)]
    ptr_q = np.arange(0, 4 * 512 + 1, 512, dtype=np.int64)
    idx, d = K.knn(torch.from_numpy(q), torch.from_numpy(pos), torch.from_numpy(ptr_q), torch.from_numpy(ptr), 16)
    idx, d = idx.numpy(), d.numpy()
    assert strictly_increasing_rows(d, idx >= 0), "config-1 KNN has a distance tie; fixture would be ambiguous"
    out["knn_c1_idx"] = idx.astype(np.int32)
    out["knn_c1_dist"] = d
    # variable sizes incl. a source cloud smaller than k, and an empty query cloud
    for seed in range(100, 200):
        g = torch.Generator().manual_seed(seed)
        qs, ss = [40, 0, 25, 60], [500, 30, 9, 333]
        qv = torch.rand(sum(qs), 3, generator=g).numpy().astype(np.float32)
        sv = torch.rand(sum(ss), 3, generator=g).numpy().astype(np.float32)
        pq = np.concatenate([[0], np.cumsum(qs)]).astype(np.int64)
        ps = np.concatenate([[0], np.cumsum(ss)]).astype(np.int64)
        ok = True
        res = {}
        for k in (1, 5, 16, 33, 70):
            i2, d2 = K.knn(torch.from_numpy(qv), torch.from_numpy(sv), torch.from_numpy(pq), torch.from_numpy(ps), k)
            i2, d2 = i2.numpy(), d2.numpy()
            if not strictly_increasing_rows(d2, i2 >= 0):
                ok = False
                break
            res[k] = (i2, d2)
        if ok:
            break
    else:
        raise RuntimeError("no tie-free KNN fixture found")
    out["knn_var_q"] = qv
    out["knn_var_s"] = sv
    out["knn_var_ptr_q"] = pq
    out["knn_var_ptr_s"] = ps
    for k, (i2, d2) in res.items():
        out[f"knn_var_k{k}_idx"] = i2.astype(np.int32)
        out[f"knn_var_k{k}_dist"] = d2


def _radius_safe(x: np.ndarray, B: int, r: float, K: int, mask=None) -> bool:
    """No pair near the boundary; no truncation (in-radius degree <= K)."""
    n = x.shape[0] // B
    r2 = np.float64(np.float32(r)) ** 2
    for b in range(B):
        p = x[b * n:(b + 1) * n].astype(np.float64)
        d = ((p[:, None, :] - p[None, :, :]) ** 2).sum(-1)
        if np.any(np.abs(d - r2) < 1e-4 * r2):
            return False
        valid = np.ones(n, bool) if mask is None else mask[b * n:(b + 1) * n]
        inr = (d < r2) & valid[None, :] & valid[:, None]
        np.fill_diagonal(inr, False)
        if inr.sum(0).max() > K - 1:
            return False
    return True


def gen_radius(R, out):
    # batched equal-size clouds (functional/radius_graph.py:70-85, :204-275)
    for seed in range(300, 400):
        g = torch.Generator().manual_seed(seed)
        B, n, r, K = 4, 200, 0.22, 32
        x = (torch.rand(B * n, 3, generator=g) * 2 - 1).numpy().astype(np.float32)
        mask = (torch.rand(B * n, generator=g) > 0.1).numpy()
        if _radius_safe(x, B, r, K) and _radius_safe(x, B, r, K, mask):
            break
    else:
        raise RuntimeError("no radius fixture without boundary pairs found")
    batch = torch.arange(B).repeat_interleave(n)
    out["rad_x"] = x
    out["rad_mask"] = mask
    out["rad_meta"] = np.array([B, n, K], np.int64)
    out["rad_r"] = np.array([r], np.float64)
    for loop in (False, True):
        for use_mask in (False, True):
            row, col = R.radius_graph(torch.from_numpy(x), r, max_num_neighbors=K, batch=batch, loop=loop,
                                      mask=torch.from_numpy(mask) if use_mask else None, num_batch_elements=B)
            tag = f"rad_b_loop{int(loop)}_mask{int(use_mask)}"
            out[tag + "_row"] = row.numpy().astype(np.int32)
            out[tag + "_col"] = col.numpy().astype(np.int32)
    # single cloud (functional/radius_graph.py:278-335)
    xs = x[:n]
    row, col = R.radius_graph(torch.from_numpy(xs), r, max_num_neighbors=K)
    out["rad_single_row"] = row.numpy().astype(np.int32)
    out["rad_single_col"] = col.numpy().astype(np.int32)
    # known-answer tests of tests/test_phase1.py:258-299
    kat = np.array([[0.0, 0.0, 0.0], [0.1, 0.0, 0.0], [10.0, 0.0, 0.0]], np.float32)
    row, col = R.radius_graph(torch.from_numpy(kat), r=1.0)
    out["rad_kat3_row"] = row.numpy().astype(np.int32)
    out["rad_kat3_col"] = col.numpy().astype(np.int32)


def gen_segment(S, out, knn_idx):
    # config 1 edge CSR: dst = centroid (2048), 16 edges each, msg ~ N(0,1) [32768, 64]
    col, msg = inputs.config1_segment_inputs()
    cs, pm, ns, ne = S.sort_and_build_csr(torch.from_numpy(col), 2048)
    m = torch.from_numpy(msg).requires_grad_(True)
    o = S.segment_reduce(m, cs, pm, ns, ne, 2048)
    gout = inputs.config1_grad_out()
    o.backward(torch.from_numpy(gout))
    out["seg_c1_sum_sha"] = np.frombuffer(sha(o.detach().numpy()).encode(), np.uint8)
    out["seg_c1_sum_head"] = o.detach().numpy()[:64]
    out["seg_c1_sum_grad_sha"] = np.frombuffer(sha(m.grad.numpy()).encode(), np.uint8)
    mx = torch.from_numpy(msg).requires_grad_(True)
    ref = torch.zeros(2048, 64).scatter_reduce(0, torch.from_numpy(col)[:, None].expand(-1, 64), mx, "amax",
                                              include_self=False)
    ref.backward(torch.from_numpy(gout))
    out["seg_c1_max_sha"] = np.frombuffer(sha(ref.detach().numpy()).encode(), np.uint8)
    out["seg_c1_max_head"] = ref.detach().numpy()[:64]
    out["seg_c1_max_grad_sha"] = np.frombuffer(sha(mx.grad.numpy()).encode(), np.uint8)

    # random CSR incl. empty nodes and ties (small, full fixture)
    g = torch.Generator().manual_seed(42)
    N, E, C = 500, 3000, 32
    colr = torch.randint(0, N, (E,), generator=g)
    msgr = torch.randn(E, C, generator=g)
    msgr[5, :] = msgr[6, :]  # duplicate rows -> max ties if they share a node
    colr[5] = colr[6]
    cs, pm, ns, ne = S.sort_and_build_csr(colr, N)
    out["seg_r_col"] = colr.numpy()
    out["seg_r_msg"] = msgr.numpy()
    out["seg_r_cs"] = cs.numpy()
    out["seg_r_perm"] = pm.numpy()
    out["seg_r_ns"] = ns.numpy()
    out["seg_r_ne"] = ne.numpy()
    gr = torch.randn(N, C, generator=g)
    out["seg_r_gout"] = gr.numpy()
    m = msgr.clone().requires_grad_(True)
    o = S.segment_reduce(m, cs, pm, ns, ne, N)
    o.backward(gr)
    out["seg_r_sum"] = o.detach().numpy()
    out["seg_r_sum_grad"] = m.grad.numpy()
    for red, tname in (("mean", "mean"), ("max", "amax")):
        for dt in (torch.float32, torch.bfloat16):
            m = msgr.to(dt).clone().requires_grad_(True)
            ref = torch.zeros(N, C, dtype=dt).scatter_reduce(0, colr[:, None].expand(-1, C), m, tname,
                                                             include_self=False)
            ref.backward(gr.to(dt))
            tag = f"seg_r_{red}_{'f32' if dt == torch.float32 else 'bf16'}"
            out[tag] = ref.detach().float().numpy()
            out[tag + "_grad"] = m.grad.float().numpy()


def _ref_spatial_graph(root: str):
    """The reference's SpatialGraph, loaded from its file: ``geoembodied.nn`` as a package
    imports modules (``geoembodied.data``) that the reference tree does not ship."""
    import importlib.util

    path = Path(root) / "geoembodied" / "nn" / "modules" / "spatial_graph.py"
    spec = importlib.util.spec_from_file_location("ref_spatial_graph", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_spatial_graph"] = mod
    spec.loader.exec_module(mod)
    return mod.SpatialGraph


def gen_graph(root: str, R, out):
    """SpatialGraph.build / from_edge_index (nn/modules/spatial_graph.py:88-246) and the
    geometry of hand-made edges (compute_edge_vectors + spherical harmonics, l <= 0, 1, 2)."""
    import importlib

    SG = _ref_spatial_graph(root)
    sph = importlib.import_module("geoembodied.kernels.triton_sph_harm")._spherical_harmonics_pytorch
    for seed in range(500, 600):
        g = torch.Generator().manual_seed(seed)
        B, n, r, K = 3, 300, 0.2, 32
        x = torch.rand(B * n, 3, generator=g).numpy().astype(np.float32)
        if _radius_safe(x, B, r, K) and _radius_safe(x[:n], 1, r, K):
            break
    else:
        raise RuntimeError("no graph fixture without boundary pairs found")
    out["graph_x"] = x
    out["graph_meta"] = np.array([B, n, K, seed], np.int64)
    out["graph_r"] = np.array([r], np.float64)
    batch = torch.arange(B).repeat_interleave(n)
    # unequal clouds (300, 250, 280 points) in shuffled order: without num_batch_elements the
    # reference takes its per-cloud loop, which honours the batch labels (radius_graph.py:
    # 181-198; equal-size batches are cut into consecutive blocks whatever the labels say)
    sel = torch.cat([torch.arange(0, 300), torch.arange(300, 550), torch.arange(600, 880)])
    perm = torch.randperm(sel.numel(), generator=torch.Generator().manual_seed(seed + 1))
    out["graph_sel"] = sel.numpy()
    out["graph_perm"] = perm.numpy()
    cases = {
        "batch": (torch.from_numpy(x), dict(batch=batch, num_batch_elements=B)),
        "single": (torch.from_numpy(x[:n]), {}),
        "shuffled": (torch.from_numpy(x)[sel][perm], dict(batch=batch[sel][perm])),
    }
    for tag, (pos, kw) in cases.items():
        gr = SG.build(pos, r, max_num_neighbors=K, **kw)
        for f in ("row", "col", "dist", "direction", "Y", "node_start", "node_end", "avg_degree"):
            out[f"graph_{tag}_{f}"] = getattr(gr, f).numpy()
    # from_edge_index on the batch graph's edges (same values, CSR re-derived)
    gb = SG.from_edge_index(torch.from_numpy(out["graph_batch_row"]), torch.from_numpy(out["graph_batch_col"]),
                            torch.from_numpy(x), B * n, max_l=1, batch=batch, num_batch_elements=B)
    for f in ("col_sorted", "perm", "node_start", "node_end", "avg_degree", "Y"):
        out[f"graph_fei_{f}"] = getattr(gb, f).numpy()

    # hand-made edges: ordinary, self edge (zero vector), a vector shorter than the 1e-8 clamp,
    # axis-aligned, huge coordinates (|diff|^2 overflows), non-finite coordinates
    pts = np.array([[0.1, -0.2, 0.3], [0.7, 0.25, -0.4], [0.1, -0.2, 0.3 + 4e-9], [1e20, 0, 0], [-1e20, 0, 0],
                    [np.inf, 0, 0], [np.nan, 1, 2], [0, 0, 0], [0, 0, 1.5], [3e-39, 0, 0]], np.float32)
    pairs = np.array([[0, 1], [1, 0], [0, 0], [0, 2], [2, 0], [3, 4], [4, 3], [5, 0], [6, 1], [7, 8], [8, 7],
                      [9, 7], [7, 9], [1, 8]], np.int64)
    g = torch.Generator().manual_seed(11)
    rnd = (torch.randn(600, 3, generator=g) * torch.tensor([1e-3, 1.0, 30.0])).numpy().astype(np.float32)
    xg = np.concatenate([pts, rnd]).astype(np.float32)
    ng = xg.shape[0]
    rr = torch.randint(0, ng, (4000,), generator=g).numpy()
    cc = torch.randint(0, ng, (4000,), generator=g).numpy()
    row = np.concatenate([pairs[:, 0], rr]).astype(np.int64)
    col = np.concatenate([pairs[:, 1], cc]).astype(np.int64)
    out["geo_x"], out["geo_row"], out["geo_col"] = xg, row, col
    diff, dist, direction = R.compute_edge_vectors(torch.from_numpy(xg), torch.from_numpy(row), torch.from_numpy(col))
    out["geo_diff"], out["geo_dist"], out["geo_dir"] = diff.numpy(), dist.numpy(), direction.numpy()
    for lmax in (0, 1, 2):
        out[f"geo_Y{lmax}"] = sph(direction, lmax).numpy()


def _ref_module_file(root: str, rel: str, name: str):
    import importlib.util

    spec = importlib.util.spec_from_file_location(name, Path(root) / rel)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def gen_aggregate(root: str, out):
    """EquivariantInterpolate.forward + backward (nn/modules/equivariant_interp.py:58-139) and the
    weighted-sum block of EquivariantPool (nn/modules/equivariant_pool.py:395-420, its three
    formula lines evaluated on the same gathers) + backward, on the CPU."""
    EI = _ref_module_file(root, "geoembodied/nn/modules/equivariant_interp.py", "ref_equivariant_interp")
    g = torch.Generator().manual_seed(21)
    nd, nc = [500, 37, 420], [120, 2, 90]  # a coarse cloud of 2 points pads KNN k=3
    dense = torch.rand(sum(nd), 3, generator=g)
    coarse = torch.rand(sum(nc), 3, generator=g)
    ptr_d = torch.tensor([0] + list(np.cumsum(nd)), dtype=torch.int64)
    ptr_c = torch.tensor([0] + list(np.cumsum(nc)), dtype=torch.int64)
    s = torch.randn(sum(nc), 16, generator=g, requires_grad=True)
    v = torch.randn(sum(nc), 8, 3, generator=g, requires_grad=True)
    t2 = torch.randn(sum(nc), 4, 5, generator=g, requires_grad=True)
    s_skip = torch.randn(sum(nd), 6, generator=g)
    v_skip = torch.randn(sum(nd), 2, 3, generator=g)
    so, vo, to = EI.EquivariantInterpolate(3)(dense, coarse, s, v, ptr_d, ptr_c, s_skip, v_skip, t2, None)
    gs, gv, gt = (torch.randn(t.shape, generator=g) for t in (so, vo, to))
    torch.autograd.backward([so, vo, to], [gs, gv, gt])
    for k, t in dict(dense=dense, coarse=coarse, ptr_d=ptr_d, ptr_c=ptr_c, s=s, v=v, t2=t2, s_skip=s_skip,
                     v_skip=v_skip, s_out=so, v_out=vo, t2_out=to, g_s=gs, g_v=gv, g_t2=gt, grad_s=s.grad,
                     grad_v=v.grad, grad_t2=t2.grad).items():
        out["interp_" + k] = t.detach().numpy()

    # pool block: KNN k=16 of 64 seeds per cloud into clouds of 200 / 9 / 150 points (padding in the
    # 9-point cloud), attention-like weights from a masked softmax
    knn = importlib_module("geoembodied.functional.knn").knn
    npts, nseed = [200, 9, 150], [64, 5, 64]
    pos = torch.rand(sum(npts), 3, generator=g)
    ptr = torch.tensor([0] + list(np.cumsum(npts)), dtype=torch.int64)
    seeds = torch.cat([pos[int(ptr[b]):int(ptr[b]) + nseed[b]] for b in range(3)])
    ptr_s = torch.tensor([0] + list(np.cumsum(nseed)), dtype=torch.int64)
    knn_idx, _ = knn(seeds, pos, ptr_s, ptr, 16)
    valid = knn_idx >= 0
    logits = torch.randn(knn_idx.shape, generator=g).masked_fill(~valid, float("-inf"))
    w = torch.softmax(logits, dim=-1).requires_grad_(True)
    scalars = torch.randn(sum(npts), 32, generator=g, requires_grad=True)
    vectors = torch.randn(sum(npts), 4, 3, generator=g, requires_grad=True)
    safe_idx = knn_idx.clamp(min=0)
    s_out = (w.unsqueeze(-1) * scalars[safe_idx]).sum(dim=1)
    v_out = (w.unsqueeze(-1).unsqueeze(-1) * vectors[safe_idx]).sum(dim=1)
    gs2, gv2 = torch.randn(s_out.shape, generator=g), torch.randn(v_out.shape, generator=g)
    torch.autograd.backward([s_out, v_out], [gs2, gv2])
    for k, t in dict(idx=knn_idx, w=w, scalars=scalars, vectors=vectors, s_out=s_out, v_out=v_out, g_s=gs2,
                     g_v=gv2, grad_s=scalars.grad, grad_v=vectors.grad, grad_w=w.grad).items():
        out["pool_" + k] = t.detach().numpy()


def _stub_data_package():
    """geoembodied.nn's package import reaches geoembodied.data, which the reference tree does not
    ship; two empty stand-in modules let the encoder stage's file import (nothing of them runs)."""
    import types

    if "geoembodied.data" in sys.modules:
        return
    d = types.ModuleType("geoembodied.data")
    b = types.ModuleType("geoembodied.data.batch")
    b.PointCloudBatch = object
    b.to_dense_batch = None
    d.batch = b
    sys.modules["geoembodied.data"] = d
    sys.modules["geoembodied.data.batch"] = b


def _knn_gaps_ok(x: np.ndarray, sizes, k: int) -> bool:
    """the k + 1 nearest of every point (self included) have distinct distances with a relative
    gap above 1e-5, so CPU and GPU distance rounding select and order the same neighbours"""
    o = 0
    for n in sizes:
        p = x[o:o + n].astype(np.float64)
        o += n
        d = np.sort(((p[:, None, :] - p[None, :, :]) ** 2).sum(-1), axis=1)[:, :k + 2]
        if np.any(np.diff(d[:, 1:], axis=1) <= 1e-5 * d[:, 2:]):
            return False
    return True


def gen_hybrid(root: str, out):
    """_EncoderStage._estimate_adaptive_radius / _build_hybrid_graph (nn/modules/
    multi_scale_se3_net.py:99-219) on the CPU, called on a stand-in stage object."""
    import types

    _stub_data_package()
    ms = importlib_module("geoembodied.nn.modules.multi_scale_se3_net")
    stage = types.SimpleNamespace(max_num_neighbors=64, knn_fallback_k=3, radius_multiplier=4.0)
    r, K, kf = 0.1, 64, 3
    for seed in range(700, 800):
        g = torch.Generator().manual_seed(seed)
        clouds = []
        for b in range(3):
            centres = torch.rand(3, 3, generator=g) * 1.5
            cl = centres.repeat_interleave(30, 0) + torch.randn(90, 3, generator=g) * 0.03
            clouds.append(torch.cat([cl, torch.rand(110, 3, generator=g) * 1.5]))
        x = torch.cat(clouds).numpy().astype(np.float32)
        if _radius_safe(x, 3, r, K) and _knn_gaps_ok(x, [200] * 3, kf + 1):
            break
    else:
        raise RuntimeError("no hybrid fixture found")
    pos = torch.from_numpy(x)
    ptr = torch.tensor([0, 200, 400, 600], dtype=torch.int64)
    out["hyb_x"] = x
    out["hyb_meta"] = np.array([K, kf, seed], np.int64)
    out["hyb_r"] = np.array([r], np.float64)
    out["hyb_adaptive_radius"] = np.array([ms._EncoderStage._estimate_adaptive_radius(stage, pos, ptr)], np.float64)
    for tag, batch in (("nobatch", None), ("batch", torch.arange(3).repeat_interleave(200))):
        gr = ms._EncoderStage._build_hybrid_graph(stage, pos, r, ptr, batch)
        for f in ("row", "col", "dist", "col_sorted", "perm", "node_start", "node_end", "avg_degree"):
            out[f"hyb_{tag}_{f}"] = getattr(gr, f).numpy()


def gen_se3(root: str, out):
    """SE3Conv.forward / backward (nn/modules/se3_conv.py:287-545) on the CPU over a graph from the
    reference's SpatialGraph.build: all nine paths (type-2 in and out), and paths 0-4 alone."""
    _stub_data_package()
    se3 = importlib_module("geoembodied.nn.modules.se3_conv")
    SG = _ref_spatial_graph(root)
    g = torch.Generator().manual_seed(31)
    pos = torch.rand(300, 3, generator=g)
    batch = torch.arange(2).repeat_interleave(150)
    graph = SG.build(pos, 0.3, max_num_neighbors=32, batch=batch, num_batch_elements=2)
    out["se3_pos"] = pos.numpy()
    out["se3_row"], out["se3_col"] = graph.row.numpy(), graph.col.numpy()
    for tag, dims in (("full", (16, 8, 24, 6, 4, 3)), ("sv", (16, 8, 24, 6, 0, 0))):
        torch.manual_seed(41)
        conv = se3.SE3Conv(*dims, radius=0.3)
        for k, v in conv.state_dict().items():
            out[f"se3_{tag}_sd_{k}"] = v.numpy()
        s_in = torch.randn(300, dims[0], generator=g, requires_grad=True)
        v_in = torch.randn(300, dims[1], 3, generator=g, requires_grad=True)
        t_in = torch.randn(300, dims[4], 5, generator=g, requires_grad=True) if dims[4] else None
        res = conv(s_in, v_in, graph, type2=t_in) if t_in is not None else conv(s_in, v_in, graph)
        grads = [torch.randn(r.shape, generator=g) for r in res]
        torch.autograd.backward(list(res), grads)
        names = ["s", "v", "t2"]
        for i, r in enumerate(res):
            out[f"se3_{tag}_out_{names[i]}"] = r.detach().numpy()
            out[f"se3_{tag}_gout_{names[i]}"] = grads[i].numpy()
        out[f"se3_{tag}_in_s"], out[f"se3_{tag}_in_v"] = s_in.detach().numpy(), v_in.detach().numpy()
        out[f"se3_{tag}_grad_s"], out[f"se3_{tag}_grad_v"] = s_in.grad.numpy(), v_in.grad.numpy()
        if t_in is not None:
            out[f"se3_{tag}_in_t2"], out[f"se3_{tag}_grad_t2"] = t_in.detach().numpy(), t_in.grad.numpy()
        for k, prm in conv.named_parameters():
            out[f"se3_{tag}_pgrad_{k}"] = prm.grad.numpy()


def importlib_module(name: str):
    import importlib

    return importlib.import_module(name)


def main():
    import importlib.util

    spec = importlib.util.spec_from_file_location("gdl_build_ref",
                                                  Path(__file__).resolve().parents[2] / "oracle" / "build_ref.py")
    build_ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build_ref)
    root = build_ref.reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    if root is None:
        raise SystemExit("usage: make_golden.py REFERENCE_ROOT (or set GDL_REFERENCE_ROOT)")
    root = str(root)
    F, K, R, S = _ref(root)
    torch.set_num_threads(os.cpu_count() or 1)
    out = {}
    gen_fps(F, out)
    gen_knn(K, out, out["fps_c1_idx"])
    gen_radius(R, out)
    gen_segment(S, out, out["knn_c1_idx"])
    np.savez_compressed(HERE / "golden_cpu.npz", **out)
    print("wrote", HERE / "golden_cpu.npz", sum(v.nbytes for v in out.values()) / 1e6, "MB raw")
    graph = {}
    gen_graph(root, R, graph)
    gen_hybrid(root, graph)
    np.savez_compressed(HERE / "golden_graph.npz", **graph)
    print("wrote", HERE / "golden_graph.npz", sum(v.nbytes for v in graph.values()) / 1e6, "MB raw")
    se3 = {}
    gen_se3(root, se3)
    np.savez_compressed(HERE / "golden_se3.npz", **se3)
    print("wrote", HERE / "golden_se3.npz", sum(v.nbytes for v in se3.values()) / 1e6, "MB raw")
    agg = {}
    gen_aggregate(root, agg)
    np.savez_compressed(HERE / "golden_aggregate.npz", **agg)
    print("wrote", HERE / "golden_aggregate.npz", sum(v.nbytes for v in agg.values()) / 1e6, "MB raw")


if __name__ == "__main__":
    main()
