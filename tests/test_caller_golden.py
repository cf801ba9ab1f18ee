"""The CPU restatement against the calls the reference's MultiScaleSE3Net made (CPU, no GPU).

Every graph-operator call recorded from one forward and backward of the unchanged caller
(``tests/golden/golden_caller.npz``) goes through the restatement in ``oracle/`` with the
arguments the caller passed, and its result is compared with what the reference returned:
FPS bit-exact (lowest-index ties, the reference's CPU fallback ``csrc/__init__.py:600-660``),
CSR build bit-exact up to the order inside a segment (the reference's CPU sort is unstable), KNN and radius graph equal up to the documented distance rounding of the
reference's torch path (on these inputs: identical neighbour sets and, in the restatement's torch
rounding mode, identical KNN distance bits), segment sums within 1e-5 of a float64 sum.
"""

import numpy as np
import pytest

from tests import caller_calls

META, CALLS = caller_calls.load()


def test_fixture_covers_every_operator():
    ops = {c["op"] for c in CALLS}
    assert ops == {"fps", "knn", "radius_graph", "sort_and_build_csr", "segment_reduce"}
    assert META["sizes"][0] != META["sizes"][1]  # unequal clouds


@pytest.mark.parametrize("c", CALLS, ids=caller_calls.call_id)
def test_restatement_matches_recorded_call(oracle, c):
    op = c["op"]
    if op == "fps":
        got = oracle.fps(c["pos"], c["ptr"], c["k"], tie=oracle.TIE_LOWEST_INDEX, dist=oracle.DIST_TORCH)
        assert np.array_equal(got, c["out"])
    elif op == "knn":
        src = c["query"] if c["self"] else c["source"]
        # the torch rounding of the reference's CPU path: same neighbours, same distance bits
        idx, dist = oracle.knn(c["query"], src, c["ptr_q"], c["ptr_s"], c["k"], dist=oracle.DIST_TORCH)
        assert np.array_equal(idx, c["idx"])
        assert np.array_equal(dist.view(np.uint32), c["dist"].view(np.uint32))
    elif op == "radius_graph":
        ptr = caller_calls.ptr_of_batch(c["batch"])
        row_ptr, src = oracle.radius_graph(c["x"], ptr, c["r"], c["max_num_neighbors"], c["loop"])
        row, col = oracle.csr_to_coo(row_ptr, src)
        ok, nd = caller_calls.radius_difference_explained(c["x"], c["r"], c["max_num_neighbors"], row, col,
                                                          c["row"], c["col"])
        assert ok and nd == 0, nd  # these inputs hold no pair at a rounding edge
    elif op == "sort_and_build_csr":
        got = oracle.sort_and_build_csr(c["col"], c["N"])
        want = [c[n] for n in ("col_sorted", "perm", "node_start", "node_end")]
        assert caller_calls.csr_matches_unordered(got, want)
        # within a segment the restatement keeps edge order (a stable sort)
        cs, pm = np.asarray(got[0]), np.asarray(got[1], np.int64)
        assert np.all((np.diff(cs) > 0) | (np.diff(pm) > 0))
    elif op == "segment_reduce":
        rng = np.random.default_rng(c["i"])
        msg = rng.standard_normal(tuple(c["shape"])).astype(np.float32)
        got = oracle.segment_reduce(msg, c["perm"], c["node_start"], c["node_end"], c["N"])
        want = np.zeros((c["N"], msg.shape[1]))
        np.add.at(want, c["col_sorted"], msg[c["perm"]].astype(np.float64))
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)
