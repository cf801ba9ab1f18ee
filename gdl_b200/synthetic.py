"""Seeded synthetic point clouds for the five benchmark configurations.

The reference publishes no data set for this path; these generators stand in for the
shapes, sizes and value distributions of its use cases (part segmentation, multiscale
pooling, registration, LiDAR). Everything is drawn on the CPU from
``torch.Generator().manual_seed(seed)`` in float32, so the CPU checker, the CPU baseline
and every GPU see bit-identical inputs.

Configurations (points x clouds, then the pipeline run on them):

* c1  4 x 2048 uniform in [-1,1]^3 -> FPS 512 -> KNN k=16 -> segment sum + max (C=64)
* c2  16 x 2048 on an anisotropically scaled unit sphere -> FPS 512 -> radius graph
      (r=0.2, 32) over the centroids -> segment mean (C=128) fwd + bwd
* c3  32 x 8192 from a 16-component Gaussian mixture -> FPS 2048/512/128 with KNN k=32
      per level -> segment max over bf16 gathered features (C=64/128/256) fwd + bwd
* c4  64 pairs x 16384 from a 32-cluster mixture in a 10 m cube, target = SE(3)
      transform + noise -> KNN k=1 -> segment sum of 6-channel residuals per cloud
* c5  8 x 131072 spinning-LiDAR returns -> FPS 16384 -> radius graph (r=1 m, 64)
      -> segment sum (C=64)
"""

from __future__ import annotations

import math

import numpy as np
import torch


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(int(seed))


def ptr_of(sizes) -> np.ndarray:
    return np.concatenate([[0], np.cumsum(np.asarray(sizes, np.int64))]).astype(np.int64)


# ----------------------------------------------------------------------------- c1
def c1_points(seed: int = 0, B: int = 4, N: int = 2048):
    g = _gen(seed)
    pos = (torch.rand(B * N, 3, generator=g) * 2 - 1).numpy()
    return pos.astype(np.float32), ptr_of([N] * B)


def c1_features(seed: int = 1, E: int = 2048 * 16, C: int = 64):
    return torch.randn(E, C, generator=_gen(seed)).numpy()


def c1_grad_out(seed: int = 2, N: int = 2048, C: int = 64):
    return torch.randn(N, C, generator=_gen(seed)).numpy()


# ----------------------------------------------------------------------------- c2
def c2_points(seed: int = 0, B: int = 16, N: int = 2048):
    g = _gen(seed)
    v = torch.randn(B, N, 3, generator=g)
    v = v / v.norm(dim=-1, keepdim=True)
    v = v + 0.01 * torch.randn(B, N, 3, generator=g)
    scale = 0.5 + torch.rand(B, 1, 3, generator=g)
    pos = (v * scale).reshape(B * N, 3)
    return pos.numpy().astype(np.float32), ptr_of([N] * B)


def c2_features(E: int, seed: int = 1, C: int = 128):
    return torch.randn(E, C, generator=_gen(seed)).numpy()


def c2_grad_out(N: int, seed: int = 2, C: int = 128):
    return torch.randn(N, C, generator=_gen(seed)).numpy()


# ----------------------------------------------------------------------------- c3
def c3_points(seed: int = 0, B: int = 32, N: int = 8192, K: int = 16, sigma: float = 0.1):
    g = _gen(seed)
    centres = torch.rand(B, K, 3, generator=g) * 2 - 1
    comp = torch.randint(0, K, (B, N), generator=g)
    pts = torch.gather(centres, 1, comp[..., None].expand(B, N, 3)) + sigma * torch.randn(B, N, 3, generator=g)
    return pts.reshape(B * N, 3).numpy().astype(np.float32), ptr_of([N] * B)


def c3_level_features(n_rows: int, C: int, seed: int):
    """bf16 features ~N(0,1) as a torch tensor (CPU)."""
    return torch.randn(n_rows, C, generator=_gen(seed)).to(torch.bfloat16)


# ----------------------------------------------------------------------------- c4
def _so3_hat(w):
    x, y, z = w
    return np.array([[0, -z, y], [z, 0, -x], [-y, x, 0]], np.float64)


def se3_exp(xi: np.ndarray) -> np.ndarray:
    """4x4 transform of a twist xi = (rho, phi) (translation part first), float64."""
    rho, phi = np.asarray(xi[:3], np.float64), np.asarray(xi[3:], np.float64)
    th = float(np.linalg.norm(phi))
    W = _so3_hat(phi)
    if th < 1e-8:
        R = np.eye(3) + W
        V = np.eye(3) + 0.5 * W
    else:
        a = math.sin(th) / th
        b = (1 - math.cos(th)) / th**2
        c = (th - math.sin(th)) / th**3
        R = np.eye(3) + a * W + b * W @ W
        V = np.eye(3) + b * W + c * W @ W
    T = np.eye(4)
    T[:3, :3] = R
    T[:3, 3] = V @ rho
    return T


def c4_pairs(seed: int = 0, B: int = 64, N: int = 16384, K: int = 32, cube: float = 10.0, sigma: float = 0.05):
    g = _gen(seed)
    centres = torch.rand(B, K, 3, generator=g) * cube
    comp = torch.randint(0, K, (B, N), generator=g)
    src = torch.gather(centres, 1, comp[..., None].expand(B, N, 3)) + sigma * torch.randn(B, N, 3, generator=g)
    xi = 0.1 * torch.randn(B, 6, generator=g)
    noise = 0.005 * torch.randn(B, N, 3, generator=g)
    src = src.numpy().astype(np.float32)
    tgt = np.empty_like(src)
    for b in range(B):
        T = se3_exp(xi[b].numpy().astype(np.float64))
        tgt[b] = (src[b].astype(np.float64) @ T[:3, :3].T + T[:3, 3]).astype(np.float32)
    tgt = tgt + noise.numpy().astype(np.float32)
    return src.reshape(B * N, 3), tgt.reshape(B * N, 3).astype(np.float32), ptr_of([N] * B)


# ----------------------------------------------------------------------------- c5
def c5_points(seed: int = 0, B: int = 8, N: int = 131072, rings: int = 64):
    g = _gen(seed)
    lo, hi = math.radians(-25.0), math.radians(3.0)
    ring_el = torch.linspace(lo, hi, rings)
    width = (hi - lo) / (rings - 1)
    ring = torch.randint(0, rings, (B, N), generator=g)
    el = ring_el[ring] + (torch.rand(B, N, generator=g) - 0.5) * width
    az = torch.rand(B, N, generator=g) * (2 * math.pi)
    rng = (-20.0 * torch.log1p(-torch.rand(B, N, generator=g))).clamp(1.0, 80.0)
    xyz = torch.stack([rng * torch.cos(el) * torch.cos(az), rng * torch.cos(el) * torch.sin(az), rng * torch.sin(el)], -1)
    xyz = xyz + 0.02 * torch.randn(B, N, 3, generator=g)
    return xyz.reshape(B * N, 3).numpy().astype(np.float32), ptr_of([N] * B)
