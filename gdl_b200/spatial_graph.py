"""SpatialGraph -- drop-in for ``geoembodied.nn.modules.spatial_graph.SpatialGraph``
(reference: geoembodied/nn/modules/spatial_graph.py:40-246).

Same frozen fields and constructors. ``build`` runs the radius graph with each edge's
geometry (diff, |diff|, direction, real spherical harmonics l <= max_l) written by the kernel
that emits the edge, then one sort-free pass for the CSR fields and the per-cloud average
degree: the reference's compute_edge_vectors gathers, spherical-harmonics kernel, radix sort
and scatter_add passes become two launches after the graph search. Edges come grouped by
destination (ascending), sources ascending within a destination, so ``perm`` is the identity
and ``col_sorted`` equals ``col``; the reference's edge order is its atomic counter's and
carries no meaning. Geometry is computed for positions as constants: positions that require
grad raise (the reference differentiates through torch ops; this build does not).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
from torch import Tensor

from . import _native as nat
from . import csrc
from .functional.radius_graph import _ptr_from_batch


@dataclass(frozen=True)
class SpatialGraph:
    row: Tensor          # [E] int64 source node indices
    col: Tensor          # [E] int64 target node indices
    direction: Tensor    # [E, 3] float32 unit vectors (x[col] - x[row]) / dist
    dist: Tensor         # [E] float32 edge lengths, clamped below at 1e-8
    col_sorted: Tensor   # [E] int32 targets in segment order
    perm: Tensor         # [E] int32 sorted slot -> original edge
    node_start: Tensor   # [N] int32
    node_end: Tensor     # [N] int32
    Y: Tensor            # [E, (max_l+1)^2] float32 spherical harmonics of direction
    N: int
    E: int
    avg_degree: Optional[Tensor] = None  # [N] float32 average degree of the node's cloud

    @staticmethod
    def build(pos: Tensor, radius: float, max_num_neighbors: int = 32, mask: Optional[Tensor] = None,
              batch: Optional[Tensor] = None, max_l: int = 2,
              num_batch_elements: Optional[int] = None) -> "SpatialGraph":
        """Radius graph + geometry + CSR + average degree (spatial_graph.py:88-167).

        One device->host read (the edge count), like the reference's ``row.shape[0]``; a
        ``batch`` vector costs one more (whether it is sorted) and, without
        ``num_batch_elements``, another (the cloud count); its offsets are built on the device."""
        _no_grad_positions(pos)
        N = pos.shape[0]
        dev = nat.require_cuda(pos, what="SpatialGraph.build")
        if batch is not None:
            batch = batch.to(device=dev, dtype=torch.int64)
            if N > 1 and not bool((batch[1:] >= batch[:-1]).all()):
                return SpatialGraph._build_unsorted(pos, radius, max_num_neighbors, mask, batch, max_l,
                                                    num_batch_elements)
            ptr = _ptr_from_batch(batch, num_batch_elements)
        else:
            B = num_batch_elements if num_batch_elements is not None else 1
            ptr = torch.arange(B + 1, dtype=torch.int64) * (N // B)
        out = csrc.radius_graph_geometry_csr(pos, radius, ptr, max_num_neighbors=max_num_neighbors, mask=mask,
                                             max_l=max_l)
        cs, pm, ns, ne, avg = csrc.radius_csr_finish(out["row_ptr"], out["dst"], N,
                                                     ptr=out["ptr"] if batch is not None else None)
        E = int(out["row_ptr"][N].item())
        if E == 0:
            return SpatialGraph._empty(N, dev, max_l)
        return SpatialGraph(row=out["src"][:E], col=out["dst"][:E], direction=out["direction"][:E],
                            dist=out["dist"][:E], col_sorted=cs[:E], perm=pm[:E], node_start=ns, node_end=ne,
                            Y=out["sph"][:E], N=N, E=E, avg_degree=avg)

    @staticmethod
    def _build_unsorted(pos, radius, max_num_neighbors, mask, batch, max_l, num_batch_elements):
        from .functional.radius_graph import radius_graph
        row, col = radius_graph(pos, radius, max_num_neighbors=max_num_neighbors, batch=batch, mask=mask,
                                num_batch_elements=num_batch_elements)
        return SpatialGraph.from_edge_index(row, col, pos, pos.shape[0], max_l=max_l, batch=batch,
                                            num_batch_elements=num_batch_elements)

    @staticmethod
    def _empty(N: int, device: torch.device, max_l: int = 2) -> "SpatialGraph":
        """Graph without edges (spatial_graph.py:169-186)."""
        num_sh = (max_l + 1) ** 2
        return SpatialGraph(
            row=torch.empty(0, dtype=torch.long, device=device),
            col=torch.empty(0, dtype=torch.long, device=device),
            direction=torch.empty(0, 3, device=device),
            dist=torch.empty(0, device=device),
            col_sorted=torch.empty(0, dtype=torch.int32, device=device),
            perm=torch.empty(0, dtype=torch.int32, device=device),
            node_start=torch.zeros(N, dtype=torch.int32, device=device),
            node_end=torch.zeros(N, dtype=torch.int32, device=device),
            Y=torch.empty(0, num_sh, device=device),
            N=N,
            E=0,
            avg_degree=torch.ones(N, device=device),
        )

    @staticmethod
    def from_edge_index(row: Tensor, col: Tensor, pos: Tensor, N: int, max_l: int = 2,
                        batch: Optional[Tensor] = None,
                        num_batch_elements: Optional[int] = None) -> "SpatialGraph":
        """SpatialGraph of given (row, col) edges (spatial_graph.py:188-246): geometry of the
        COO edges, the stable CSR sort and the per-cloud average degree, on the GPU."""
        _no_grad_positions(pos)
        dev = nat.require_cuda(pos, row, col, what="SpatialGraph.from_edge_index")
        E = row.shape[0]
        if E == 0:
            return SpatialGraph._empty(N, dev, max_l)
        _, dist, direction, Y = csrc.edge_geometry_cuda(pos, row, col, max_l=max_l, with_diff=False)
        col_sorted, perm, node_start, node_end = csrc.sort_and_build_csr_cuda(col, N)
        avg = csrc.cloud_avg_degree_cuda(node_start, node_end, batch=batch, num_clouds=num_batch_elements)
        return SpatialGraph(row=row, col=col, direction=direction, dist=dist, col_sorted=col_sorted, perm=perm,
                            node_start=node_start, node_end=node_end, Y=Y, N=N, E=E, avg_degree=avg)


def _no_grad_positions(pos: Tensor) -> None:
    if pos.requires_grad and torch.is_grad_enabled():
        raise nat.GdlError("SpatialGraph: edge geometry is computed for constant positions; "
                           "pass pos.detach() (positions that require grad are not supported)")
