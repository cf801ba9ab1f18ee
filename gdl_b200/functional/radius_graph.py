"""Radius graph -- drop-in for ``geoembodied.functional.radius_graph``
(reference: geoembodied/functional/radius_graph.py:19-105, 338-358)."""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from .. import _native as nat
from .. import csrc


def _ptr_from_batch(batch_sorted: Tensor, B: Optional[int]) -> Tensor:
    """CSR offsets of a sorted batch vector, built on the device (searchsorted); only when the
    cloud count B is not given is it read from the device (one synchronisation)."""
    if B is None:
        B = int(batch_sorted[-1].item()) + 1 if batch_sorted.numel() else 0
    marks = torch.arange(int(B) + 1, dtype=torch.int64, device=batch_sorted.device)
    return torch.searchsorted(batch_sorted, marks)


def radius_graph_csr(x: Tensor, r: float, ptr: Tensor, *, max_num_neighbors: int = 32, loop: bool = False,
                     mask: Optional[Tensor] = None):
    """Edges of packed clouds as a destination CSR (row_ptr [N+1], src, dst); the first
    row_ptr[N] entries of src/dst are valid. No host synchronisation (pass ``ptr`` as a
    CPU tensor to let small clouds use the fused kernels)."""
    return csrc.radius_graph_csr(x, r, ptr, max_num_neighbors=max_num_neighbors, loop=loop, mask=mask)


def radius_graph(x: Tensor, r: float, *, max_num_neighbors: int = 32, batch: Optional[Tensor] = None,
                 loop: bool = False, mask: Optional[Tensor] = None,
                 num_batch_elements: Optional[int] = None) -> Tuple[Tensor, Tensor]:
    """(row, col) int64 with ||x[row] - x[col]|| < r; row = source (neighbour), col = target.

    Each target keeps its bucket(max_num_neighbors) in {16, 32, 64} nearest in-radius
    points of its own cloud, selected exactly as the reference CUDA kernel does. Clouds come
    from ``batch`` (any sizes, any order), else ``num_batch_elements`` equal-size clouds,
    else one cloud. Edges are grouped by target, sources ascending.
    """
    N = x.shape[0]
    if batch is not None:
        # clouds in any order: a stable sort by cloud on the device (no host read), offsets by
        # searchsorted; the only synchronisations are the edge count below (the output's size)
        # and, without num_batch_elements, the cloud count
        batch = batch.to(torch.int64)
        order = torch.argsort(batch, stable=True)
        xb = x[order]
        mb = mask if mask is None else mask[order]
        ptr = _ptr_from_batch(batch[order], num_batch_elements)
    else:
        order, xb, mb = None, x, mask
        B = num_batch_elements if num_batch_elements is not None else 1
        ptr = torch.arange(B + 1, dtype=torch.int64) * (N // B)
    row_ptr, src, dst = csrc.radius_graph_csr(xb, r, ptr, max_num_neighbors=max_num_neighbors, loop=loop, mask=mb)
    E = int(row_ptr[N].item())
    row, col = src[:E], dst[:E]
    if order is not None:
        row, col = order[row], order[col]
    return row, col


def compute_edge_vectors(x: Tensor, row: Tensor, col: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
    """(diff = x[col] - x[row], |diff| clamped at 1e-8, diff / |diff|) of the reference
    (radius_graph.py:338-358), one CUDA kernel over the edges with the reference's CPU
    rounding (gdl_edge_geometry_coo). Positions are constants here: ``x`` that requires grad
    raises (the reference differentiates through torch ops; this build does not)."""
    if x.requires_grad and torch.is_grad_enabled():
        raise nat.GdlError("compute_edge_vectors: positions that require grad are not supported; "
                           "pass x.detach()")
    diff, dist, direction, _ = csrc.edge_geometry_cuda(x, row, col)
    return diff, dist, direction
