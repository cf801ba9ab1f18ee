"""GPU parity of the fused SE3Conv message aggregation (gdl_se3_aggregate + backward) through
the SE3Conv mirror: against the reference's own fp32 outputs and gradients
(tests/golden/golden_se3.npz) and against the float64 restatement of the reference formulas
(oracle/se3_ref.py, itself pinned to the reference in tests/test_se3_restatement.py).

Floating point, summed in a different order than the reference (per-node channel mixing, then
per-edge products), so the bars are rounding bounds: outputs |ours - f64| <= 1e-5 * (the formula
on absolute values) + 1e-7 per element; gradients max |ours - f64| <= 2e-5 * max |f64| per
tensor. The reference's fp32 results meet the same bars (asserted alongside)."""

import numpy as np
import pytest
import torch

from gdl_b200.se3_conv import SE3Conv
from gdl_b200.spatial_graph import SpatialGraph
from oracle import se3_ref as se3_f64

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = "cuda"
DIMS = {"full": (16, 8, 24, 6, 4, 3), "sv": (16, 8, 24, 6, 0, 0)}


@pytest.fixture(scope="module")
def gs():
    from tests.conftest import ROOT

    return np.load(ROOT / "tests" / "golden" / "golden_se3.npz")


def _f64_grads(sd, dims, pos, row, col, s, v, t2, clouds, cutoff, gouts):
    leaf = {k: t.double().clone().requires_grad_(k != "radial_basis.freqs" and k != "cg_11_2") for k, t in sd.items()}
    si = s.double().clone().requires_grad_(True)
    vi = v.double().clone().requires_grad_(True)
    ti = t2.double().clone().requires_grad_(True) if t2 is not None else None
    outs = se3_f64.se3_forward(leaf, dims, pos, row, col, si, vi, ti, clouds, cutoff)
    outs = outs[:len(gouts)]
    torch.autograd.backward(list(outs), [g.double() for g in gouts])
    grads = {"s": si.grad, "v": vi.grad}
    if ti is not None:
        grads["t2"] = ti.grad
    for k, t in leaf.items():
        if t.requires_grad:
            grads["p:" + k] = t.grad
    return [o.detach() for o in outs], grads


def _check_grad(ours, ref64, other=None):
    tol = 2e-5 * ref64.abs().max().item() + 1e-9
    assert (ours.double() - ref64).abs().max().item() <= tol
    if other is not None:
        assert (other.double() - ref64).abs().max().item() <= tol


@pytest.mark.parametrize("tag", ["full", "sv"])
def test_se3conv_golden(gs, tag):
    dims = DIMS[tag]
    pre = f"se3_{tag}_sd_"
    sd = {k[len(pre):]: torch.from_numpy(gs[k]) for k in gs.files if k.startswith(pre)}
    pos, row, col = (torch.from_numpy(gs[k]) for k in ("se3_pos", "se3_row", "se3_col"))
    s, v = torch.from_numpy(gs[f"se3_{tag}_in_s"]), torch.from_numpy(gs[f"se3_{tag}_in_v"])
    t2 = torch.from_numpy(gs[f"se3_{tag}_in_t2"]) if dims[4] else None
    names = ["s", "v", "t2"] if dims[5] else ["s", "v"]
    gouts = [torch.from_numpy(gs[f"se3_{tag}_gout_{n}"]) for n in names]
    conv = SE3Conv(*dims, radius=0.3).to(DEV)
    conv.load_state_dict({k: t.to(DEV) for k, t in sd.items()})
    batch = torch.arange(2, device=DEV).repeat_interleave(150)
    graph = SpatialGraph.from_edge_index(row.to(DEV), col.to(DEV), pos.to(DEV), 300, batch=batch,
                                         num_batch_elements=2)
    si = s.to(DEV).requires_grad_(True)
    vi = v.to(DEV).requires_grad_(True)
    ti = t2.to(DEV).requires_grad_(True) if t2 is not None else None
    outs = conv(si, vi, graph, type2=ti) if ti is not None else conv(si, vi, graph)
    torch.autograd.backward(list(outs), [g.to(DEV) for g in gouts])
    clouds = [(0, 150), (150, 300)]
    ref64, g64 = _f64_grads(sd, dims, pos, row, col, s, v, t2, clouds, 0.3, gouts)
    bound = se3_f64.se3_forward(sd, dims, pos, row, col, s, v, t2, clouds, 0.3, absolute=True)
    for i, n in enumerate(names):
        ours = outs[i].detach().cpu().double()
        assert torch.all((ours - ref64[i]).abs() <= 1e-5 * bound[i] + 1e-7), n
        golden = torch.from_numpy(gs[f"se3_{tag}_out_{n}"]).double()
        assert torch.all((ours - golden).abs() <= 2e-5 * bound[i] + 2e-7), n
    _check_grad(si.grad.cpu(), g64["s"], torch.from_numpy(gs[f"se3_{tag}_grad_s"]))
    _check_grad(vi.grad.cpu(), g64["v"], torch.from_numpy(gs[f"se3_{tag}_grad_v"]))
    if ti is not None:
        _check_grad(ti.grad.cpu(), g64["t2"], torch.from_numpy(gs[f"se3_{tag}_grad_t2"]))
    for k, prm in conv.named_parameters():
        _check_grad(prm.grad.cpu(), g64["p:" + k], torch.from_numpy(gs[f"se3_{tag}_pgrad_{k}"]))


def test_se3conv_large_random():
    """two clouds of 3000 points, graph from SpatialGraph.build, all nine paths"""
    torch.manual_seed(5)
    dims = (32, 16, 48, 12, 8, 6)
    N = 6000
    pos = torch.rand(N, 3)
    batch = torch.arange(2).repeat_interleave(N // 2)
    graph = SpatialGraph.build(pos.to(DEV), 0.1, max_num_neighbors=32, batch=batch.to(DEV), num_batch_elements=2)
    assert graph.E > 30_000
    conv = SE3Conv(*dims, radius=0.1).to(DEV)
    sd = {k: t.detach().cpu() for k, t in conv.state_dict().items()}
    s, v, t2 = torch.randn(N, 32), torch.randn(N, 16, 3), torch.randn(N, 8, 5)
    si, vi, ti = (t.to(DEV).requires_grad_(True) for t in (s, v, t2))
    outs = conv(si, vi, graph, type2=ti)
    gouts = [torch.randn(o.shape) for o in outs]
    torch.autograd.backward(list(outs), [g.to(DEV) for g in gouts])
    row, col = graph.row.cpu(), graph.col.cpu()
    clouds = [(0, N // 2), (N // 2, N)]
    ref64, g64 = _f64_grads(sd, dims, pos, row, col, s, v, t2, clouds, 0.1, gouts)
    bound = se3_f64.se3_forward(sd, dims, pos, row, col, s, v, t2, clouds, 0.1, absolute=True)
    for i in range(3):
        assert torch.all((outs[i].detach().cpu().double() - ref64[i]).abs() <= 1e-5 * bound[i] + 1e-7)
    _check_grad(si.grad.cpu(), g64["s"])
    _check_grad(vi.grad.cpu(), g64["v"])
    _check_grad(ti.grad.cpu(), g64["t2"])
    for k, prm in conv.named_parameters():
        _check_grad(prm.grad.cpu(), g64["p:" + k])


def test_se3conv_empty_graph_and_mask():
    conv = SE3Conv(4, 2, 5, 3, radius=0.1).to(DEV)
    pos = torch.tensor([[0.0, 0, 0], [5.0, 0, 0]], device=DEV)
    g = SpatialGraph.build(pos, 0.1)
    s_out, v_out = conv(torch.randn(2, 4, device=DEV), torch.randn(2, 2, 3, device=DEV), g)
    assert g.E == 0 and torch.allclose(s_out, conv.scalar_bias.expand(2, 5)) and torch.all(v_out == 0)
    pos = torch.rand(200, 3, device=DEV)
    g = SpatialGraph.build(pos, 0.3)
    mask = torch.rand(200, device=DEV) > 0.3
    s_out, v_out = conv(torch.randn(200, 4, device=DEV), torch.randn(200, 2, 3, device=DEV), g, mask=mask)
    assert torch.all(s_out[~mask] == 0) and torch.all(v_out[~mask] == 0)


def test_backward_degree_division_in_kernel_equals_prescaled():
    """gdl_se3_aggregate_backward divides by the average degree itself (avg_degree given) or takes
    gradients already divided (avg_degree NULL, what SE3Conv passes): both IEEE divisions of the
    same numbers, so every gradient is bit-identical."""
    import ctypes

    from gdl_b200 import _native as nat
    from gdl_b200.se3_conv import _source_csr, cg_11_2_cartesian

    torch.manual_seed(3)
    pos = torch.rand(3000, 3, device=DEV) * 4.0
    batch = torch.repeat_interleave(torch.arange(3, device=DEV), 1000)
    g = SpatialGraph.build(pos, 0.5, max_num_neighbors=32, batch=batch, max_l=2, num_batch_elements=3)
    N, E = g.N, g.E
    cs, cv, ct2 = 20, 7, 5
    widths = [cs, cv, 3 * cv, 3 * cs, 3 * cv, ct2, 5 * ct2, 3 * ct2, cs]
    proj = [torch.randn(N, w, device=DEV) for w in widths]
    R = torch.randn(E, 9, device=DEV)
    cg = cg_11_2_cartesian().to(DEV).contiguous()
    sph = g.Y.contiguous()
    gs, gv, gt = torch.randn(N, cs, device=DEV), torch.randn(N, cv, 3, device=DEV), torch.randn(N, ct2, 5, device=DEV)
    sperm, sstart, send = _source_csr(g)
    st = nat.Se3Paths()
    for i in range(9):
        st.p[i] = proj[i].data_ptr()
        st.r_col[i] = i
    st.cs, st.cv, st.ct2 = cs, cv, ct2
    L = nat.load()

    def run(gs_, gv_, gt_, avg):
        gp = [torch.empty_like(p) for p in proj]
        gR = torch.zeros_like(R)
        arr = (ctypes.c_void_p * 9)(*[t.data_ptr() for t in gp])
        nat.check(L.gdl_se3_aggregate_backward(
            ctypes.byref(st), arr, gR.data_ptr(), gs_.data_ptr(), gv_.data_ptr(), gt_.data_ptr(), R.data_ptr(), 9,
            g.direction.contiguous().data_ptr(), sph.data_ptr(), sph.shape[1], cg.data_ptr(), g.row.data_ptr(),
            g.col.data_ptr(), sperm.data_ptr(), sstart.data_ptr(), send.data_ptr(), avg, N, E,
            nat.stream(torch.device(DEV))), "gdl_se3_aggregate_backward")
        return gp, gR

    deg = g.avg_degree.reshape(N, 1)
    a_gp, a_gR = run(gs, gv, gt, g.avg_degree.data_ptr())
    b_gp, b_gR = run((gs / deg).contiguous(), (gv / deg.unsqueeze(-1)).contiguous(),
                     (gt / deg.unsqueeze(-1)).contiguous(), None)
    assert E > 0 and torch.equal(a_gR, b_gR)
    for x, y in zip(a_gp, b_gp):
        assert torch.equal(x, y)
