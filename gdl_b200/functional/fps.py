"""Farthest point sampling -- drop-in for ``geoembodied.functional.fps``
(reference: geoembodied/functional/fps.py:29-162)."""

from __future__ import annotations

import torch
from torch import Tensor

from .. import csrc


def farthest_point_sampling(pos: Tensor, num_samples: int, batch: Tensor = None, ptr: Tensor = None, *,
                            tie_break: str = "reference") -> Tensor:
    """Indices of ``num_samples`` points per cloud chosen by farthest point sampling.

    * ``ptr`` given ([B+1] CSR offsets): k_b = min(n_b, num_samples) picks per cloud, global
      indices in selection order, concatenated (fps.py:84-118).
    * neither given: one cloud; ``num_samples >= N`` returns ``arange(N)`` (fps.py:121-135).
    * ``batch`` given: per cloud as the single-cloud rule, concatenated in cloud order
      (fps.py:68-81); clouds with n_b <= num_samples return their points in index order.
    Seeds at each cloud's first point; ``tie_break`` as in ``csrc.fps_cuda``.
    """
    N = pos.shape[0]
    if ptr is not None:
        ptr_h = ptr.to(torch.int64).cpu()
        k = (ptr_h[1:] - ptr_h[:-1]).clamp(max=num_samples)
        return csrc.fps_cuda(pos, ptr_h, k, tie_break=tie_break)
    if batch is None:
        if num_samples >= N:
            return torch.arange(N, device=pos.device)
        return csrc.fps_cuda(pos, torch.tensor([0, N]), torch.tensor([num_samples]), tie_break=tie_break)
    # legacy batch vector: group points by cloud (stable), sample, map back to global indices
    batch = batch.to(torch.int64)
    order = torch.argsort(batch, stable=True)
    counts = torch.bincount(batch).cpu()
    ptr_h = torch.zeros(counts.numel() + 1, dtype=torch.int64)
    ptr_h[1:] = counts.cumsum(0)
    k = counts.clamp(max=num_samples)
    picks = csrc.fps_cuda(pos[order], ptr_h, k, tie_break=tie_break)
    small = counts <= num_samples
    if bool(small.any()):  # the single-cloud rule returns arange when k >= n
        out_ptr = torch.zeros_like(ptr_h)
        out_ptr[1:] = k.cumsum(0)
        for b in torch.nonzero(small).flatten().tolist():
            picks[int(out_ptr[b]):int(out_ptr[b + 1])] = torch.arange(int(ptr_h[b]), int(ptr_h[b + 1]),
                                                                       device=pos.device)
    return order[picks]
