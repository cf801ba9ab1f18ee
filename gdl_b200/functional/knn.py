"""K-nearest neighbours -- drop-in for ``geoembodied.functional.knn``
(reference: geoembodied/functional/knn.py:31-85)."""

from __future__ import annotations

from typing import Tuple

from torch import Tensor

from ..csrc import knn_cuda as _knn


def knn(query: Tensor, source: Tensor, ptr_q: Tensor, ptr_s: Tensor, k: int) -> Tuple[Tensor, Tensor]:
    """(indices [N_q, k] int64 global into source, -1 padded; squared distances [N_q, k]
    float32, 1e30 padded), nearest first, per cloud of the ptr offsets."""
    return _knn(query, source, ptr_q, ptr_s, k)


def knn_self(pos: Tensor, ptr: Tensor, k: int) -> Tuple[Tensor, Tensor]:
    """KNN of each point within its own cloud; column 0 is the point itself."""
    return _knn(pos, pos, ptr, ptr, k)
