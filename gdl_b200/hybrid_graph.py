"""Hybrid radius / KNN graph -- drop-in for the graph builders of the reference's encoder
stage, ``_EncoderStage._estimate_adaptive_radius`` and ``_EncoderStage._build_hybrid_graph``
(geoembodied/nn/modules/multi_scale_se3_net.py:99-219).

``build_hybrid_graph`` runs the radius graph, a self-KNN with k = knn_fallback_k + 1, and one
native pass (gdl_hybrid_graph) that adds both directions of each fallback edge of the nodes with
fewer than knn_fallback_k radius in-edges, deduplicates the union and orders it by (row, col)
exactly as the reference's hash ``unique()`` does -- without the hash, with the segment-reduce
CSR of the result produced alongside instead of a second sort, and with each edge's geometry
written by the kernel that places the edge. The average degree follows
``SpatialGraph.from_edge_index``. One device->host read (the edge
count), where the reference syncs for ``unique()`` and for the isolated-node test.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import _native as nat
from . import csrc
from .spatial_graph import SpatialGraph, _no_grad_positions


def estimate_adaptive_radius(pos: Tensor, ptr: Tensor, radius_multiplier: float) -> float:
    """mean over points of sqrt(clamp(d_nn, 1e-8, 1e20)) * radius_multiplier, d_nn the squared
    distance to the nearest other point of the cloud (knn_self k = 2, column 1) --
    multi_scale_se3_net.py:99-124. One device->host read."""
    with torch.no_grad():
        _, dists = csrc.knn_cuda(pos, pos, ptr, ptr, 2)
        nn_d = dists[:, 1]
        avg = nn_d.clamp(max=1e20).clamp(min=1e-8).sqrt().mean().item()
    return avg * radius_multiplier


def build_hybrid_graph(pos: Tensor, radius: float, ptr: Tensor, batch: Optional[Tensor] = None, *,
                       max_num_neighbors: int = 32, knn_fallback_k: int = 3, max_l: int = 2) -> SpatialGraph:
    """SpatialGraph of the radius graph with symmetric KNN fallback edges
    (multi_scale_se3_net.py:126-219). Clouds come from ``ptr`` (the reference's radius call
    uses ``batch`` when given, ``ptr``'s equal-size blocks otherwise; both name the same
    clouds for a well-formed batch)."""
    _no_grad_positions(pos)
    dev = nat.require_cuda(pos, what="build_hybrid_graph")
    N = pos.shape[0]
    rp, src, _ = csrc.radius_graph_csr(pos, radius, ptr, max_num_neighbors=max_num_neighbors, with_dst=False)
    kf = int(knn_fallback_k)
    knn_idx = csrc.knn_cuda(pos, pos, ptr, ptr, kf + 1)[0] if kf > 0 else None
    h = csrc.hybrid_graph_cuda(rp, src, knn_idx, N, max_num_neighbors, kf, x=pos, max_l=max_l)
    E = int(h["row_ptr"][N].item())
    if E == 0:
        return SpatialGraph._empty(N, dev, max_l)
    row, col = h["row"][:E], h["col"][:E]
    dist, direction, Y = h["dist"][:E], h["direction"][:E], h["sph"][:E]
    B = ptr.numel() - 1
    avg = csrc.cloud_avg_degree_cuda(h["node_start"], h["node_end"], batch=batch,
                                     num_clouds=B if batch is not None else None)
    return SpatialGraph(row=row, col=col, direction=direction, dist=dist, col_sorted=h["col_sorted"][:E],
                        perm=h["perm"][:E], node_start=h["node_start"], node_end=h["node_end"], Y=Y, N=N, E=E,
                        avg_degree=avg)


class HybridGraphBuilder:
    """The two graph methods of the reference's encoder stage under their own names, for a
    stage object that carries max_num_neighbors, knn_fallback_k and radius_multiplier."""

    def __init__(self, max_num_neighbors: int = 32, knn_fallback_k: int = 3, radius_multiplier: float = 4.0):
        self.max_num_neighbors = max_num_neighbors
        self.knn_fallback_k = knn_fallback_k
        self.radius_multiplier = radius_multiplier

    def _estimate_adaptive_radius(self, pos: Tensor, ptr: Tensor) -> float:
        return estimate_adaptive_radius(pos, ptr, self.radius_multiplier)

    def _build_hybrid_graph(self, pos: Tensor, radius: float, ptr: Tensor,
                            batch: Optional[Tensor] = None) -> SpatialGraph:
        return build_hybrid_graph(pos, radius, ptr, batch, max_num_neighbors=self.max_num_neighbors,
                                  knn_fallback_k=self.knn_fallback_k)
