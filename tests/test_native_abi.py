"""CPU checks of the C-ABI library: it loads without a GPU, exports exactly what
include/gdl_b200.h declares, and the host-only size queries behave; the Python layer
refuses CPU tensors (no CPU fallback)."""

import re
from pathlib import Path

import pytest
import torch

from gdl_b200 import _native as nat

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "gdl_b200.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(gdl_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not nat.LIB_PATH.exists():
        from gdl_b200 import build

        build.build()
    return nat.load()


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = declared()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(nat.PROTOTYPES), "ctypes prototypes must mirror the header"


def test_host_only_queries(lib):
    assert lib.gdl_version() >= 100
    assert lib.gdl_status_string(0) == b"ok"
    assert lib.gdl_status_string(2) == b"workspace too small"
    assert lib.gdl_fps_workspace_size(1000, 1, 4096) == 0  # registers/shared memory only
    # bucketed clouds: Morton keys, sorted keys and the order (12 B per point) plus radix scratch
    assert lib.gdl_fps_workspace_size(8 * 131072, 8, 131072) >= 12 * 8 * 131072
    assert lib.gdl_fps_workspace_size(10**6, 1, 10**6) >= 4 * 10**6
    w1 = lib.gdl_knn_workspace_size(2048, 4, 16, 8192)
    w2 = lib.gdl_knn_workspace_size(10**6, 64, 1, 16384)
    assert w1 > 0 and w2 > 0
    assert lib.gdl_radius_graph_workspace_size(131072, 8, 64) > 131072 * 64 * 4
    assert lib.gdl_sort_and_build_csr_workspace_size(10**6, 10**5) > 10**6 * 4
    assert lib.gdl_segment_reduce_workspace_size(10**6, 10**5) >= 256


def test_argument_validation_without_gpu(lib):
    # invalid arguments are rejected before any CUDA call
    assert lib.gdl_fps(None, None, None, 1, 10, 10, 7, None, None, None, 0, None) == 1
    assert lib.gdl_fps_ex(None, None, None, 1, 10, 10, 7, None, None, None, 0, None, 0, -1, -1, None) == 1
    assert lib.gdl_segment_reduce(None, 5, 1, 1, None, None, None, 1, 0, None, None, None, 0, None) == 1
    assert lib.gdl_knn(None, None, None, None, 1, 10, 4, 10, None, None, None, 0, None) == 1
    bad = nat.EdgeGeometry(None, None, None, 1, 3)  # harmonics of degree 3 are not provided
    assert lib.gdl_edge_geometry_coo(None, 4, None, None, 2, bad, None) == 1
    assert lib.gdl_cloud_avg_degree(None, None, 3, None, None, 0, None, None, 0, None) == 1
    assert lib.gdl_radius_csr_finish(None, None, 3, 3, None, 0, None, None, None, None, None, None) == 1
    assert lib.gdl_cloud_avg_degree_workspace_size(8) >= 128
    paths = nat.Se3Paths()
    paths.cs, paths.cv, paths.ct2 = 4, 2, 0
    paths.p[0] = 16  # a path switched on without an R column
    paths.r_col[0] = -1
    assert lib.gdl_se3_aggregate(paths, None, 1, None, None, 1, None, None, None, None, None, None, 5, 5, None, None,
                                 None, None) == 1
    assert lib.gdl_se3_aggregate(None, None, 1, None, None, 1, None, None, None, None, None, None, 5, 5, None, None,
                                 None, None) == 1
    assert lib.gdl_hybrid_graph_capacity(1000, 32, 3) == 1000 * (32 + 6)
    assert lib.gdl_hybrid_graph_workspace_size(1000, 32, 3) > 1000 * 38 * 12
    assert lib.gdl_hybrid_graph(None, None, None, None, 10, 32, 3, None, None, None, None, None, None, None, None,
                                None, None, 0, None) == 1
    assert lib.gdl_weight_grad(None, 4, None, 4, 10, 4, 4, 2, None, None, None, 0, None) == 1  # sub 2
    assert lib.gdl_weight_grad(None, 12, None, 12, 10, 4, 4, 3, 16, 16, None, 0, None) == 1  # bias with sub 3
    assert lib.gdl_weight_grad(16, 3, 16, 4, 10, 4, 4, 1, 16, None, None, 0, None) == 1  # lda < M
    assert lib.gdl_weight_grad(16, 4, 16, 4, 10, 4, 4, 1, 16, None, None, 0, None) == 2  # no workspace
    assert lib.gdl_weight_grad_workspace_size(100_000, 9, 64, 1) >= 9 * 64 * 4


def test_cpu_tensors_raise():
    from gdl_b200 import csrc

    x = torch.zeros(4, 3)
    with pytest.raises(nat.GdlError):
        csrc.fps_cuda(x, torch.tensor([0, 4]), torch.tensor([2]))
    with pytest.raises(nat.GdlError):
        csrc.radius_graph_csr(x, 0.5, torch.tensor([0, 4]))
    with pytest.raises(nat.GdlError):
        csrc.segment_reduce_cuda(x, None, torch.zeros(1, dtype=torch.int32), torch.ones(1, dtype=torch.int32), 1)
    e = torch.zeros(2, dtype=torch.int64)
    with pytest.raises(nat.GdlError):
        csrc.edge_geometry_cuda(x, e, e)
    from gdl_b200.spatial_graph import SpatialGraph

    with pytest.raises(nat.GdlError):
        SpatialGraph.build(x, 0.5)
    with pytest.raises(nat.GdlError):  # positions that require grad are refused before any device check
        SpatialGraph.build(x.requires_grad_(True), 0.5)
