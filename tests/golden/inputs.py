"""Seeded inputs of the golden fixtures (shared by the generator and the tests)."""

import numpy as np

from gdl_b200 import synthetic


def config1_points():
    return synthetic.c1_points()


def config1_segment_inputs():
    """Edge CSR of config 1: 2048 centroids x 16 KNN edges (dst = centroid), msg ~ N(0,1)."""
    col = np.repeat(np.arange(2048, dtype=np.int64), 16)
    return col, synthetic.c1_features()


def config1_grad_out():
    return synthetic.c1_grad_out()
