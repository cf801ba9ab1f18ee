"""Allocation-free segment reduce, called through the C ABI.

gdl_segment_reduce_noalloc is for callers that may not allocate device memory while they run:
a CUDA graph captured under a fixed memory plan, plugin or real-time hosts whose enqueue path
forbids cudaMalloc / cudaFree, programs without an allocator for the device. Instead of a
caller workspace it uses a scratch array built into the library. This test checks that it
returns exactly what gdl_segment_reduce (workspace version) returns, on two calls in a row --
the second call must not see what the first left in the shared array -- and that inputs above
its stated limit are refused. The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from gdl_b200 import _native as nat

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

MAX_ROWS = 16320 * 4097  # documented limit of gdl_segment_reduce_noalloc
REDUCE = {"sum": 0, "mean": 1, "max": 2}


def _case(seed):
    """A CSR with short segments, an empty one and two longer than 4096 slots."""
    rng = np.random.default_rng(seed)
    lens = np.concatenate([rng.integers(0, 20, 300), [0, 5000 + seed, 9000], rng.integers(0, 40, 200)])
    rows, C = int(lens.sum()), 24 + 8 * (seed % 2)
    ns = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int32)
    ne = (ns + lens).astype(np.int32)
    perm = rng.permutation(rows).astype(np.int32)
    msg = rng.standard_normal((rows, C)).astype(np.float32)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    return t(msg), t(perm), t(ns), t(ne), len(lens)


def _run(L, fn, msg, perm, ns, ne, N, reduce):
    C = msg.shape[1]
    out = torch.full((N, C), float("nan"), device="cuda")
    arg = torch.full((N, C), -7, dtype=torch.int32, device="cuda") if reduce == "max" else None
    stream = torch.cuda.current_stream().cuda_stream
    common = (msg.data_ptr(), 0, msg.shape[0], C, perm.data_ptr(), ns.data_ptr(), ne.data_ptr(), N, REDUCE[reduce],
              out.data_ptr(), None if arg is None else arg.data_ptr())
    if fn == "noalloc":
        rc = L.gdl_segment_reduce_noalloc(*common, stream)
    else:
        ws = torch.empty(L.gdl_segment_reduce_workspace_size(msg.shape[0], N), dtype=torch.uint8, device="cuda")
        rc = L.gdl_segment_reduce(*common, ws.data_ptr(), ws.numel(), stream)
    assert rc == 0, nat.status_string(rc)
    torch.cuda.synchronize()
    return out, arg


@pytest.mark.parametrize("reduce", ["sum", "max", "mean"])
def test_noalloc_matches_workspace_entry_point(reduce):
    L = nat.load()
    for seed in (1, 2):  # two calls in a row, different inputs
        case = _case(seed)
        want, want_arg = _run(L, "workspace", *case, reduce)
        got, got_arg = _run(L, "noalloc", *case, reduce)
        assert torch.equal(got.view(torch.int32), want.view(torch.int32))  # bit-identical
        if reduce == "max":
            assert torch.equal(got_arg, want_arg)


def test_noalloc_refuses_inputs_above_its_limit():
    L = nat.load()
    rc = L.gdl_segment_reduce_noalloc(None, 0, MAX_ROWS + 1, 4, None, None, None, 1, 0, None, None, None)
    assert rc == 5  # GDL_ERR_OVERFLOW, before any device work
    assert "index range" in nat.status_string(rc)
    _ = ctypes  # the entry point is reached through the ctypes binding of include/gdl_b200.h
