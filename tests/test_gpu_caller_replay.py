"""Replay of the reference MultiScaleSE3Net's graph-operator calls on the B200 build.

``tests/golden/golden_caller.npz`` holds every FPS, KNN, radius-graph, CSR-build and
segment-reduce call that one forward and backward of the unchanged reference caller
(``nn/modules/multi_scale_se3_net.py:427``: the encoder stages' hybrid graphs, the pooling
layers' FPS + KNN, the skip fusion's KNN, SE3Conv's aggregation) made, with the arguments it
passed and the reference's results (``tests/golden/make_caller_golden.py``). Each call here
goes, with the same arguments, through

1. the redirected ``geoembodied.csrc`` names -- the module body a maintainer puts in the
   reference's dispatcher (``REDIRECT`` below, the same lines as the integration notes) -- and
   the drop-in ``gdl_b200.functional`` entry points, and
2. the reference's own CUDA kernels built from its sources (``oracle/_ref``), when present,

and the results must agree: bit-exact with the reference kernels (indices, distance bits,
CSR arrays, sums), exact with the recorded CPU results where both paths define the same thing
(FPS with lowest-index ties, neighbour sets, CSR up to the CPU sort's order within a segment),
KNN distances within 1e-5 of the CPU path's torch rounding.
"""

import types

import numpy as np
import pytest
import torch

from tests import caller_calls, ref_cuda

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = "cuda"

# geoembodied/csrc/__init__.py (reference), replacing the JIT loaders
REDIRECT = """
from gdl_b200 import csrc as _b200

def fps_available() -> bool: return _b200.fps_available()
def knn_available() -> bool: return _b200.knn_available()
def segment_reduce_available() -> bool: return _b200.segment_reduce_available()
def get_radius_graph_backend() -> str: return _b200.get_radius_graph_backend()
fps_cuda = _b200.fps_cuda
knn_cuda, knn_self_cuda = _b200.knn_cuda, _b200.knn_self_cuda
radius_graph_cuda = _b200.radius_graph_cuda
sort_and_build_csr_cuda = _b200.sort_and_build_csr_cuda
segment_reduce_sum_cuda = _b200.segment_reduce_sum_cuda
"""

META, CALLS = caller_calls.load()


@pytest.fixture(scope="module")
def redirected():
    ns = types.ModuleType("geoembodied_csrc_redirected")
    exec(compile(REDIRECT, "geoembodied/csrc/__init__.py (redirect)", "exec"), ns.__dict__)
    assert ns.fps_available() and ns.knn_available() and ns.segment_reduce_available()
    assert ns.get_radius_graph_backend() == "cuda"
    return ns


@pytest.fixture(scope="module")
def ref():
    if not ref_cuda.available():
        return None
    return {n: ref_cuda.load(n) for n in ("fps", "knn", "radius_graph", "segment_reduce")}


def _d(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return (t if dtype is None else t.to(dtype)).to(DEV)


def _edge_keys(row, col):
    return np.unique(np.asarray(col, np.int64) * (1 << 32) + np.asarray(row, np.int64))


@pytest.mark.parametrize("c", CALLS, ids=caller_calls.call_id)
def test_replay_call(redirected, ref, c):
    from gdl_b200 import functional as F

    op = c["op"]
    if op == "fps":
        pos, ptr, k = _d(c["pos"]), _d(c["ptr"]), _d(c["k"])
        # the pooling layer's call, as it is written (equivariant_pool.py:261-265)
        got = redirected.fps_cuda(pos, ptr, k)
        low = redirected.fps_cuda(pos, ptr, k, tie_break="lowest_index")
        assert np.array_equal(low.cpu().numpy(), c["out"])  # the reference's CPU fallback
        if ref is not None:
            assert torch.equal(got.cpu(), ref["fps"].fps_cuda(pos, ptr, k).cpu())
        else:
            assert np.array_equal(got.cpu().numpy(), c["out"])
    elif op == "knn":
        q, pq, ps = _d(c["query"]), _d(c["ptr_q"]), _d(c["ptr_s"])
        s = q if c["self"] else _d(c["source"])
        idx, dist = (F.knn_self(q, pq, c["k"]) if c["self"] else F.knn(q, s, pq, ps, c["k"]))
        idx2, dist2 = redirected.knn_cuda(q, s, pq, ps, c["k"])  # functional/knn.py's _knn_dispatch
        assert torch.equal(idx, idx2) and torch.equal(dist.view(torch.int32), dist2.view(torch.int32))
        gi, gd = idx.cpu().numpy(), dist.cpu().numpy()
        ok, nd = caller_calls.knn_difference_explained(gi, gd, c["idx"], c["dist"])
        assert ok and np.array_equal(gi, c["idx"]), nd  # these inputs hold no near-tie
        if ref is not None:
            wi, wd = ref["knn"].knn_cuda(q, s, pq, ps, c["k"])
            assert torch.equal(idx.cpu(), wi.cpu())
            assert torch.equal(dist.cpu().view(torch.int32), wd.cpu().view(torch.int32))
    elif op == "radius_graph":
        x, batch = _d(c["x"]), _d(c["batch"])
        row, col = F.radius_graph(x, c["r"], max_num_neighbors=c["max_num_neighbors"], batch=batch,
                                  loop=c["loop"])
        gr, gc = row.cpu().numpy(), col.cpu().numpy()
        ok, nd = caller_calls.radius_difference_explained(c["x"], c["r"], c["max_num_neighbors"], gr, gc,
                                                          c["row"], c["col"])
        assert ok and nd == 0, nd  # these inputs hold no pair at a rounding edge
        if ref is not None:
            # the reference kernel per cloud (its CUDA path takes equal-size clouds only)
            ptr = caller_calls.ptr_of_batch(c["batch"])
            want = []
            for b in range(len(ptr) - 1):
                a, e = int(ptr[b]), int(ptr[b + 1])
                wr, wc = ref["radius_graph"].radius_graph_cuda_batched(
                    x[a:e].contiguous(), c["r"], c["max_num_neighbors"], torch.empty(0, dtype=torch.bool,
                                                                                      device=DEV),
                    c["loop"], 1, e - a)
                want.append(_edge_keys(wr.cpu().numpy() + a, wc.cpu().numpy() + a))
            assert np.array_equal(_edge_keys(gr, gc), np.sort(np.concatenate(want)))
    elif op == "sort_and_build_csr":
        col = _d(c["col"])
        got = redirected.sort_and_build_csr_cuda(col, c["N"])
        got2 = F.sort_and_build_csr(col, c["N"])
        for a, b in zip(got, got2):
            assert torch.equal(a, b)
        want = [c[n] for n in ("col_sorted", "perm", "node_start", "node_end")]
        assert caller_calls.csr_matches_unordered([t.cpu().numpy() for t in got], want)
        if ref is not None:
            for a, b in zip(got, ref["segment_reduce"].sort_and_build_csr(col, c["N"])):
                assert torch.equal(a.cpu().to(torch.int64), b.cpu().to(torch.int64))
    elif op == "segment_reduce":
        g = torch.Generator().manual_seed(1000 + c["i"])
        msg = torch.randn(*c["shape"], generator=g).to(DEV)
        grad = torch.randn(c["N"], c["shape"][1], generator=g).to(DEV)
        cs, perm = _d(c["col_sorted"], torch.int32), _d(c["perm"], torch.int32)
        ns, ne = _d(c["node_start"], torch.int32), _d(c["node_end"], torch.int32)
        m = msg.clone().requires_grad_(True)
        out = F.segment_reduce(m, cs, perm, ns, ne, c["N"])  # se3_conv.py:521-535
        out.backward(grad)
        out2 = redirected.segment_reduce_sum_cuda(msg, perm, ns, ne, c["N"])
        assert torch.equal(out.detach().view(torch.int32), out2.view(torch.int32))
        want = np.zeros((c["N"], c["shape"][1]))
        mm = msg.cpu().numpy().astype(np.float64)
        np.add.at(want, c["col_sorted"], mm[c["perm"]])
        np.testing.assert_allclose(out.detach().cpu().numpy(), want, rtol=1e-5, atol=1e-5)
        # backward of a sum: each message receives its target's gradient
        gm = np.zeros(c["shape"], np.float32)
        gm[c["perm"]] = grad.cpu().numpy()[c["col_sorted"]]
        assert np.array_equal(m.grad.cpu().numpy(), gm)
        if ref is not None:
            w = ref["segment_reduce"].segment_reduce_sum(msg, perm, ns, ne, c["N"])
            assert torch.equal(out.detach().cpu().view(torch.int32), w.cpu().view(torch.int32))
