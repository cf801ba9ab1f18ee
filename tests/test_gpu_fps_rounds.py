"""The bucketed FPS kernel's exchange rounds (gdl_fps_round_count), through the C ABI.

The kernel makes its picks in rounds of up to 16: a record that is provably the next pick of the
one-at-a-time chain joins the round. On clouds of duplicated points every minimum is 0 after the
first pick, so no later record qualifies and each round makes exactly one pick; on spread-out
clouds rounds make several. Either way the picks equal the CPU restatement's.
"""

import ctypes

import numpy as np
import pytest
import torch

from gdl_b200 import _native as nat
from gdl_b200 import synthetic

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = "cuda"
MAX_ROUND_PICKS = 16


def _fps_rounds(x, sizes, k):
    L = nat.load()
    ptr = synthetic.ptr_of(sizes)
    B, n, m = len(sizes), x.shape[0], max(sizes)
    kk = np.full(B, k, np.int64)
    xd = torch.from_numpy(x).to(DEV)
    pd, kd = torch.from_numpy(ptr).to(DEV), torch.from_numpy(kk).to(DEV)
    out = torch.empty(B * k, dtype=torch.int64, device=DEV)
    ws = nat.workspace(L.gdl_fps_workspace_size(n, B, m), torch.device(DEV))
    nat.check(L.gdl_fps(xd.data_ptr(), pd.data_ptr(), kd.data_ptr(), B, n, m, 0, out.data_ptr(), None, ws.data_ptr(),
                        ws.numel(), torch.cuda.current_stream().cuda_stream), "fps")
    torch.cuda.synchronize()
    r = ctypes.c_ulonglong(0)
    nat.check(L.gdl_fps_round_count(ws.data_ptr(), n, B, m, ctypes.byref(r)), "gdl_fps_round_count")
    return out.cpu().numpy(), int(r.value), ptr, kk


@pytest.mark.parametrize("sizes", [[30000], [6000, 7000], [131072, 90000]])
def test_rounds_on_spread_clouds(oracle, sizes):
    rng = np.random.default_rng(len(sizes))
    x = (rng.random((sum(sizes), 3), dtype=np.float32) * 2 - 1).astype(np.float32)
    k = 1500
    out, rounds, ptr, kk = _fps_rounds(x, sizes, k)
    want = oracle.fps(x, ptr, kk, tie=oracle.TIE_REFERENCE, dist=oracle.DIST_CUDA)
    assert np.array_equal(out, want)
    assert -(-(k - 1) // MAX_ROUND_PICKS) <= rounds < k - 1


def test_one_pick_per_round_on_duplicates(oracle):
    x = np.zeros((20000, 3), np.float32)
    k = 300
    out, rounds, ptr, kk = _fps_rounds(x, [20000], k)
    assert np.array_equal(out, oracle.fps(x, ptr, kk, tie=oracle.TIE_REFERENCE, dist=oracle.DIST_CUDA))
    assert rounds == k - 1


def test_small_clouds_report_no_rounds():
    L = nat.load()
    r = ctypes.c_ulonglong(7)
    nat.check(L.gdl_fps_round_count(None, 4096, 2, 2048, ctypes.byref(r)), "gdl_fps_round_count")
    assert r.value == 0
