"""Public operators of the B200 build -- the drop-in for ``geoembodied.functional``'s
graph-construction and aggregation entry points."""

from .aggregate import (EquivariantInterpolate, KnnWeightedSum, knn_idw_weights, knn_interpolate,
                        knn_weighted_sum)
from .fps import farthest_point_sampling
from .knn import knn, knn_self
from .radius_graph import compute_edge_vectors, radius_graph, radius_graph_csr
from .segment_reduce import SegmentReduceFunction, segment_reduce, sort_and_build_csr

__all__ = [
    "farthest_point_sampling", "knn", "knn_self", "radius_graph", "radius_graph_csr", "compute_edge_vectors",
    "sort_and_build_csr", "segment_reduce", "SegmentReduceFunction", "knn_weighted_sum", "KnnWeightedSum",
    "knn_idw_weights", "knn_interpolate", "EquivariantInterpolate",
]
