"""Weighted KNN aggregation -- the reductions of the reference's KNN consumers without the
[n_query, k, dim] gathers:

* ``knn_weighted_sum(idx, weight, *feats)``: sum_j weight[q, j] * feat[idx[q, j]] for each
  feature table (the "4. Weighted aggregation" block of EquivariantPool,
  nn/modules/equivariant_pool.py:395-420), differentiable w.r.t. the tables and the weights.
* ``knn_idw_weights(idx, dist)``: the inverse-distance weights of EquivariantInterpolate
  (nn/modules/equivariant_interp.py:91-96).
* ``knn_interpolate(...)``: EquivariantInterpolate.forward as a function (KNN, weights, sums,
  skip concatenation; equivariant_interp.py:58-139).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from .. import csrc
from .knn import knn


class KnnWeightedSum(torch.autograd.Function):
    """outs[t][q] = sum_j weight[q, j] * feats[t][idx[q, j]]; one kernel per table forward, one
    shared sorted pair list for the tables' backward."""

    @staticmethod
    def forward(ctx, idx: Tensor, weight: Tensor, *feats: Tensor):
        outs = tuple(csrc.knn_weighted_sum_cuda(f, idx, weight) for f in feats)
        ctx.save_for_backward(idx, weight, *feats)
        ctx.shapes = [tuple(f.shape) for f in feats]
        ctx.dtypes = [f.dtype for f in feats]
        return outs

    @staticmethod
    def backward(ctx, *grads: Tensor):
        idx, weight, *feats = ctx.saved_tensors
        grads = [torch.zeros(idx.shape[0], *shp[1:], device=idx.device) if g is None else g
                 for g, shp in zip(grads, ctx.shapes)]
        g_feats = [None] * len(feats)
        need = [i for i in range(len(feats)) if ctx.needs_input_grad[2 + i]]
        if need:
            res = csrc.knn_weighted_sum_backward_cuda([grads[i] for i in need], idx, weight,
                                                      [ctx.shapes[i] for i in need])
            for i, r in zip(need, res):
                g_feats[i] = r.to(ctx.dtypes[i])
        g_w = None
        if ctx.needs_input_grad[1]:
            g_w = csrc.knn_weighted_sum_weight_grad_cuda(grads, feats, idx).to(weight.dtype)
        return (None, g_w, *g_feats)


def knn_weighted_sum(idx: Tensor, weight: Tensor, *feats: Tensor):
    """Weighted sums of each query's neighbour rows for every feature table given (any trailing
    shape, fp32 out). Returns one tensor for one table, else a tuple."""
    outs = KnnWeightedSum.apply(idx, weight, *feats)
    return outs[0] if len(outs) == 1 else outs


def knn_idw_weights(idx: Tensor, dist: Tensor) -> Tensor:
    return csrc.knn_idw_weights_cuda(idx, dist)


def knn_interpolate(dense_pos: Tensor, coarse_pos: Tensor, s_coarse: Tensor, v_coarse: Tensor, ptr_dense: Tensor,
                    ptr_coarse: Tensor, k_neighbors: int = 3, s_skip: Optional[Tensor] = None,
                    v_skip: Optional[Tensor] = None, t2_coarse: Optional[Tensor] = None,
                    t2_skip: Optional[Tensor] = None) -> Tuple[Tensor, ...]:
    """EquivariantInterpolate.forward (nn/modules/equivariant_interp.py:58-139): KNN of each
    dense point among its cloud's coarse points, inverse-distance weights, weighted sums of
    s [N, C_s], v [N, C_v, 3] (and t2 [N, C_t2, 5]), then the skip concatenations. Rows whose
    neighbours are all padding come out 0, as in the reference."""
    idx, dist = knn(dense_pos, coarse_pos, ptr_dense, ptr_coarse, k_neighbors)
    w = knn_idw_weights(idx, dist)
    feats = [s_coarse, v_coarse] + ([t2_coarse] if t2_coarse is not None else [])
    outs = KnnWeightedSum.apply(idx, w, *feats)
    s_interp, v_interp = outs[0], outs[1]
    if s_skip is not None:
        s_interp = torch.cat([s_interp, s_skip], dim=-1)
    if v_skip is not None:
        v_interp = torch.cat([v_interp, v_skip], dim=1)
    if t2_coarse is not None:
        t2_interp = outs[2]
        if t2_skip is not None:
            t2_interp = torch.cat([t2_interp, t2_skip], dim=1)
        return s_interp, v_interp, t2_interp
    return s_interp, v_interp


class EquivariantInterpolate(torch.nn.Module):
    """Drop-in for geoembodied.nn.modules.equivariant_interp.EquivariantInterpolate (no
    parameters; same forward signature and outputs)."""

    def __init__(self, k_neighbors: int = 3) -> None:
        super().__init__()
        self.k_neighbors = k_neighbors

    def forward(self, dense_pos, coarse_pos, s_coarse, v_coarse, ptr_dense, ptr_coarse, s_skip=None, v_skip=None,
                t2_coarse=None, t2_skip=None):
        return knn_interpolate(dense_pos, coarse_pos, s_coarse, v_coarse, ptr_dense, ptr_coarse, self.k_neighbors,
                               s_skip, v_skip, t2_coarse, t2_skip)

    def extra_repr(self) -> str:
        return f"k={self.k_neighbors}"
