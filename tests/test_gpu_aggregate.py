"""GPU parity of the KNN aggregation row (gdl_knn_idw_weights, gdl_knn_weighted_sum and its
backward / weight gradient) through the C ABI: bit-exact against the CPU checker (oracle/),
which tests/test_oracle_aggregate.py pins to the reference's CPU path; the reference fixtures
themselves are met within the fp32-sum bound stated there."""

import numpy as np
import pytest
import torch

from gdl_b200 import csrc
from gdl_b200 import functional as F
from tests.test_oracle_aggregate import close

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = "cuda"


@pytest.fixture(scope="module")
def ga():
    from tests.conftest import ROOT

    return np.load(ROOT / "tests" / "golden" / "golden_aggregate.npz")


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _case(seed, n_src, n_q, k, pad=0.1):
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, n_src, (n_q, k)).astype(np.int64)
    idx[rng.random((n_q, k)) < pad] = -1
    if n_q > 3:
        idx[3, :] = -1          # a row without neighbours
        idx[2, 0] = n_src + 5   # out of range: skipped
    w = rng.random((n_q, k)).astype(np.float32)
    return idx, w


@pytest.mark.parametrize("shape", [(1,), (3,), (5,), (16,), (18,), (64,), (256,), (8, 3), (4, 5)])
@pytest.mark.parametrize("k", [1, 3, 16, 64])
def test_weighted_sum_matches_oracle(oracle, shape, k):
    rng = np.random.default_rng(k * 1000 + int(np.prod(shape)))
    n_src, n_q = 700, 900
    src = rng.standard_normal((n_src,) + shape).astype(np.float32)
    idx, w = _case(k, n_src, n_q, k)
    got = csrc.knn_weighted_sum_cuda(_t(src), _t(idx), _t(w))
    assert got.shape == (n_q,) + shape
    assert np.array_equal(got.cpu().numpy(), oracle.knn_weighted_sum(src, idx, w))
    # backward of two tables at once and the weight gradient
    g1 = rng.standard_normal((n_q,) + shape).astype(np.float32)
    src2 = rng.standard_normal((n_src, 7)).astype(np.float32)
    g2 = rng.standard_normal((n_q, 7)).astype(np.float32)
    gs = csrc.knn_weighted_sum_backward_cuda([_t(g1), _t(g2)], _t(idx), _t(w), [src.shape, src2.shape])
    assert np.array_equal(gs[0].cpu().numpy(), oracle.knn_weighted_sum_backward(g1, idx, w, n_src))
    assert np.array_equal(gs[1].cpu().numpy(), oracle.knn_weighted_sum_backward(g2, idx, w, n_src))
    gw = csrc.knn_weighted_sum_weight_grad_cuda([_t(g1), _t(g2)], [_t(src), _t(src2)], _t(idx))
    assert np.array_equal(gw.cpu().numpy(), oracle.knn_weighted_sum_weight_grad([g1, g2], [src, src2], idx))


def test_idw_weights_match_oracle(oracle):
    rng = np.random.default_rng(4)
    idx, _ = _case(4, 100, 5000, 3, pad=0.2)
    dist = (rng.random((5000, 3)) * 0.01).astype(np.float32)
    dist[::7, 1] = 0.0         # coincident points: clamped at 1e-4
    dist[::11, 2] = 1e30       # KNN padding value
    got = csrc.knn_idw_weights_cuda(_t(idx), _t(dist))
    assert np.array_equal(got.cpu().numpy(), oracle.knn_idw_weights(idx, dist))


def test_interpolate_golden_and_oracle(ga, oracle):
    d, c = _t(ga["interp_dense"]), _t(ga["interp_coarse"])
    pd, pc = _t(ga["interp_ptr_d"]), _t(ga["interp_ptr_c"])
    s = _t(ga["interp_s"]).requires_grad_(True)
    v = _t(ga["interp_v"]).requires_grad_(True)
    t2 = _t(ga["interp_t2"]).requires_grad_(True)
    mod = F.EquivariantInterpolate(3)
    so, vo, to = mod(d, c, s, v, pd, pc, _t(ga["interp_s_skip"]), _t(ga["interp_v_skip"]), t2, None)
    torch.autograd.backward([so, vo, to], [_t(ga["interp_g_s"]), _t(ga["interp_g_v"]), _t(ga["interp_g_t2"])])
    # exact against the checker on this build's own neighbour lists
    idx, dist = F.knn(d, c, pd, pc, 3)
    idx_h, dist_h = idx.cpu().numpy(), dist.cpu().numpy()
    w = oracle.knn_idw_weights(idx_h, dist_h)
    assert np.array_equal(so.detach().cpu().numpy()[:, :16], oracle.knn_weighted_sum(ga["interp_s"], idx_h, w))
    assert np.array_equal(vo.detach().cpu().numpy()[:, :8], oracle.knn_weighted_sum(ga["interp_v"], idx_h, w))
    assert np.array_equal(to.detach().cpu().numpy(), oracle.knn_weighted_sum(ga["interp_t2"], idx_h, w))
    assert np.array_equal(s.grad.cpu().numpy(),
                          oracle.knn_weighted_sum_backward(ga["interp_g_s"][:, :16], idx_h, w, s.shape[0]))
    # the reference fixture within the fp32-sum bound (same neighbour sets: no ties in the inputs)
    assert np.array_equal(idx_h, oracle.knn(ga["interp_dense"], ga["interp_coarse"], ga["interp_ptr_d"],
                                            ga["interp_ptr_c"], 3, dist=oracle.DIST_TORCH)[0])
    for got, f, name in ((so, ga["interp_s"], "s"), (vo, ga["interp_v"], "v"), (to, ga["interp_t2"], "t2")):
        bound = oracle.knn_weighted_sum(np.abs(f), idx_h, np.abs(w))
        g = got.detach().cpu().numpy()
        n = bound.shape[1]
        assert close(g[:, :n], ga[f"interp_{name}_out"][:, :n], bound)
    assert np.array_equal(so.detach().cpu().numpy()[:, 16:], ga["interp_s_skip"])
    for t, name in ((s, "s"), (v, "v"), (t2, "t2")):
        g = ga[f"interp_g_{name}"][:, :t.shape[1]]
        bound = oracle.knn_weighted_sum_backward(np.abs(g), idx_h, np.abs(w), t.shape[0])
        assert close(t.grad.cpu().numpy(), ga[f"interp_grad_{name}"], bound)


def test_pool_weighted_sum_autograd_golden(ga, oracle):
    idx = _t(ga["pool_idx"])
    w = _t(ga["pool_w"]).requires_grad_(True)
    sc = _t(ga["pool_scalars"]).requires_grad_(True)
    vc = _t(ga["pool_vectors"]).requires_grad_(True)
    s_out, v_out = F.knn_weighted_sum(idx, w, sc, vc)
    torch.autograd.backward([s_out, v_out], [_t(ga["pool_g_s"]), _t(ga["pool_g_v"])])
    ih, wh = ga["pool_idx"], ga["pool_w"]
    for got, f, name in ((s_out, ga["pool_scalars"], "s"), (v_out, ga["pool_vectors"], "v")):
        assert np.array_equal(got.detach().cpu().numpy(), oracle.knn_weighted_sum(f, ih, wh))
        assert close(got.detach().cpu().numpy(), ga[f"pool_{name}_out"],
                     oracle.knn_weighted_sum(np.abs(f), ih, np.abs(wh)))
    for t, name in ((sc, "s"), (vc, "v")):
        g = ga[f"pool_g_{name}"]
        assert np.array_equal(t.grad.cpu().numpy(), oracle.knn_weighted_sum_backward(g, ih, wh, t.shape[0]))
        assert close(t.grad.cpu().numpy(), ga[f"pool_grad_{name}"],
                     oracle.knn_weighted_sum_backward(np.abs(g), ih, np.abs(wh), t.shape[0]))
    gw = oracle.knn_weighted_sum_weight_grad([ga["pool_g_s"], ga["pool_g_v"]], [ga["pool_scalars"],
                                                                               ga["pool_vectors"]], ih)
    assert np.array_equal(w.grad.cpu().numpy(), gw)


def test_interpolate_full_size_multiscale(oracle):
    """Config 3's decoder shape: 32 clouds, 2048 dense queries per cloud from 512 coarse points,
    k = 3, 128 scalar + 32 x 3 vector channels; exact against the checker."""
    rng = np.random.default_rng(8)
    B, nd, nc = 32, 2048, 512
    d = rng.random((B * nd, 3)).astype(np.float32)
    c = rng.random((B * nc, 3)).astype(np.float32)
    pd = torch.arange(0, B * nd + 1, nd, dtype=torch.int64)
    pc = torch.arange(0, B * nc + 1, nc, dtype=torch.int64)
    s = rng.standard_normal((B * nc, 128)).astype(np.float32)
    v = rng.standard_normal((B * nc, 32, 3)).astype(np.float32)
    so, vo = F.knn_interpolate(_t(d), _t(c), _t(s), _t(v), pd.to(DEV), pc.to(DEV), 3)
    idx, dist = F.knn(_t(d), _t(c), pd.to(DEV), pc.to(DEV), 3)
    w = oracle.knn_idw_weights(idx.cpu().numpy(), dist.cpu().numpy())
    assert np.array_equal(so.cpu().numpy(), oracle.knn_weighted_sum(s, idx.cpu().numpy(), w))
    assert np.array_equal(vo.cpu().numpy(), oracle.knn_weighted_sum(v, idx.cpu().numpy(), w))


def test_empty_and_degenerate():
    e = torch.empty(0, 3, dtype=torch.int64, device=DEV)
    out = csrc.knn_weighted_sum_cuda(torch.randn(5, 4, device=DEV), e, torch.empty(0, 3, device=DEV))
    assert out.shape == (0, 4)
    k0 = csrc.knn_weighted_sum_cuda(torch.randn(5, 4, device=DEV), torch.empty(6, 0, dtype=torch.int64, device=DEV),
                                    torch.empty(6, 0, device=DEV))
    assert k0.shape == (6, 4) and torch.all(k0 == 0)
    g = csrc.knn_weighted_sum_backward_cuda([torch.randn(6, 4, device=DEV)],
                                            torch.full((6, 2), -1, dtype=torch.int64, device=DEV),
                                            torch.ones(6, 2, device=DEV), [(5, 4)])
    assert torch.all(g[0] == 0)
