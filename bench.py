"""Benchmark of the B200 point-cloud graph pipeline (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5] [--impl ours|reference]

A step is one pass of a configuration's pipeline over its batch of clouds (seeded synthetic
inputs with the shapes of the reference's use cases; see gdl_b200/synthetic.py):

  c5 (default)  8 clouds x 131072 LiDAR points (the largest configuration): FPS -> 16384
                centroids per cloud, radius graph (r = 1 m, 64) over the centroids, segment sum
                of 64-channel features. Under torchrun the 8 clouds are split over the ranks
                by cloud (strong scaling); a whole batch per rank is measured too (weak_scaling).
  c1            4 clouds x 2048 uniform points: FPS -> 512, KNN k=16, segment sum and max
                (64 channels).
  c2            16 clouds x 2048 points: FPS -> 512 centroids per cloud, radius graph
                (r = 0.2, 32 neighbours) over the centroids, segment mean of 128-channel
                features over that graph, forward and backward.
  c3            32 GMM clouds x 8192 points: FPS chain 8192 -> 2048 -> 512 -> 128, KNN k=32
                per level, segment max over gathered bf16 features, forward and backward.
  c4            64 source/target pairs x 16384 points: KNN k=1, residual segment sum.
  c2c           (auxiliary) one SE3Conv layer (scalar, vector and type-2 channels), forward and
                backward, over c2's centroid graph: per-node channel mixing + the fused
                message / segment-reduce kernel.
  c3i           (auxiliary) c3's clouds: the decoder's KNN k=3 inverse-distance interpolation
                128 -> 512 -> 2048 -> 8192 of scalar + vector features, forward and backward.
  c5g           (auxiliary) c5's clouds: radius graph r = 1 m, 64 over all points, segment sum.
  c5h           (auxiliary) c5 with the reference encoder's hybrid graph (radius graph + symmetric
                KNN-3 fallback, deduplicated, with edge geometry) over the FPS centroids.
  c5s           (auxiliary) c5's clouds: SpatialGraph.build -- radius graph r = 1 m, 64 over all
                points with each edge's distance, direction and l <= 2 spherical harmonics, the
                CSR fields and the per-cloud average degree.
  seg           (auxiliary) segment reduce alone: 65536 segments x 32 rows x 64 f32 channels, sum
                and max, forward and backward (the metric's segment-reduce GB/s).

value : input points per second with inputs resident in HBM, timed with CUDA events on the
        launching stream, L2 flushed (256 MiB write) between steps, max over ranks.
e2e   : the same through the public Python API (gdl_b200.functional / csrc) with inputs
        copied from pinned host memory and the result copied back inside each timed step.
roofline : the dominant stage against its bound -- HBM (measured copy bandwidth), FP32 (the
        packed-FMA throughput measured in the same run) or, for FPS, the per-pick latency of
        the same kernel on duplicated points (its exchange chain alone).
per_config : at N=1, configurations 1-4 measured the same way in the same run.
--impl reference times the reference algorithm's CPU implementation (the C restatement
in oracle/, all host threads) on the same configuration.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from gdl_b200 import _native as nat  # noqa: E402
from gdl_b200 import csrc, synthetic  # noqa: E402
from gdl_b200 import functional as F  # noqa: E402
from gdl_b200.spatial_graph import SpatialGraph  # noqa: E402

L2_FLUSH_BYTES = 256 << 20
FPS_BUCKETED_LAUNCHES = 1 + 1 + 13 + 1  # clouds > 4096 points: box, Morton keys, radix sort, FPS


# ----------------------------------------------------------------------------- configs
class C2:
    cpu_fraction = 1.0
    cpu_sample = "full steps"
    points_per_step = property(lambda self: self.B * self.N)
    name = "c2"
    metric = "points/sec (FPS 512 + radius graph r=0.2 k=32 + segment mean C=128 fwd+bwd), config 2"
    B, N, K, R, NN, C = 16, 2048, 512, 0.2, 32, 128

    def _host_init(self, seed, pin=True):
        pos, ptr = synthetic.c2_points(seed=seed, B=self.B, N=self.N)
        self.n_points = pos.shape[0]
        self.nc = self.B * self.K
        g = torch.Generator().manual_seed(seed + 1)
        feat = torch.randn(self.nc, self.C, generator=g)
        self._gout_h = torch.randn(self.nc, self.C, generator=g).numpy()
        self.ptr_h = torch.from_numpy(ptr)
        self.k_h = torch.full((self.B,), self.K, dtype=torch.int64)
        self.cptr_h = torch.arange(0, self.nc + 1, self.K, dtype=torch.int64)
        self.pos_h = torch.from_numpy(pos)
        self.feat_h = feat
        if pin:  # pinned host copies for the end-to-end leg
            self.pos_h, self.feat_h = self.pos_h.pin_memory(), self.feat_h.pin_memory()

    def __init__(self, dev, seed):
        self.dev = dev
        self._host_init(seed)
        # device-resident inputs
        self.pos = self.pos_h.to(dev)
        self.feat = self.feat_h.to(dev)
        self.gout = torch.from_numpy(self._gout_h).to(dev)
        self.ptr = self.ptr_h.to(dev)
        self.k = self.k_h.to(dev)
        self.cptr = self.cptr_h.to(dev)
        self.cap = self.nc * self.NN
        L = nat.load()
        self.L = L
        self.idx = torch.empty(self.nc, dtype=torch.int64, device=dev)
        self.row_ptr = torch.empty(self.nc + 1, dtype=torch.int64, device=dev)
        self.src = torch.zeros(self.cap, dtype=torch.int64, device=dev)
        self.dst = torch.zeros(self.cap, dtype=torch.int64, device=dev)
        self.out = torch.empty(self.nc, self.C, dtype=torch.float32, device=dev)
        self.gmsg = torch.empty(self.cap, self.C, dtype=torch.float32, device=dev)
        self.ws_fps = nat.workspace(L.gdl_fps_workspace_size(self.n_points, self.B, self.N), dev)
        self.ws_rad = nat.workspace(L.gdl_radius_graph_workspace_size(self.nc, self.B, self.NN), dev)
        self.ws_seg = nat.workspace(L.gdl_segment_reduce_workspace_size(self.cap, self.nc), dev)

        # static intermediates, so that every stage can be captured as its own CUDA graph
        self.cent = torch.empty(self.nc, 3, dtype=torch.float32, device=dev)  # written by FPS
        self.row_ptr32 = torch.zeros(self.nc + 1, dtype=torch.int32, device=dev)
        self.ns, self.ne = self.row_ptr32[:-1], self.row_ptr32[1:]
        self.src32 = torch.zeros(self.cap, dtype=torch.int32, device=dev)

    # kernels of this library launched per step (fps 1; radius graph 2 (fused per-cloud kernel
    # + compaction); segment fwd 2 + bwd 2)
    launches_per_step = 1 + 2 + 2 + 2

    def _s(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def stage_fps(self):
        nat.check(self.L.gdl_fps(self.pos.data_ptr(), self.ptr.data_ptr(), self.k.data_ptr(), self.B, self.n_points,
                                 self.N, 0, self.idx.data_ptr(), self.cent.data_ptr(), self.ws_fps.data_ptr(),
                                 self.ws_fps.numel(), self._s()), "fps")

    def stage_radius(self):
        nat.check(self.L.gdl_radius_graph(self.cent.data_ptr(), self.cptr.data_ptr(), self.B, self.nc, self.K, self.R,
                                          self.NN, 0, None, self.row_ptr.data_ptr(), self.src.data_ptr(),
                                          self.dst.data_ptr(), self.row_ptr32.data_ptr(), self.src32.data_ptr(),
                                          self.ws_rad.data_ptr(), self.ws_rad.numel(), self._s()), "radius")

    def stage_seg_fwd(self):
        # messages = source-point features gathered through the CSR (perm = src), mean per destination
        nat.check(self.L.gdl_segment_reduce(self.feat.data_ptr(), 0, self.nc, self.C, self.src32.data_ptr(),
                                            self.ns.data_ptr(), self.ne.data_ptr(), self.nc, 1, self.out.data_ptr(),
                                            None, self.ws_seg.data_ptr(), self.ws_seg.numel(), self._s()),
                  "segment mean")

    def stage_seg_bwd(self):
        # gradient w.r.t. the per-edge messages (slot-indexed rows)
        nat.check(self.L.gdl_segment_reduce_backward(self.gout.data_ptr(), None, 0, None, None, self.cap, self.C, None,
                                                     self.ns.data_ptr(), self.ne.data_ptr(), self.nc, 1,
                                                     self.gmsg.data_ptr(), self.ws_seg.data_ptr(),
                                                     self.ws_seg.numel(), self._s()), "segment mean bwd")

    def stage_list(self):
        return [("fps", self.stage_fps), ("radius_graph", self.stage_radius),
                ("segment_mean_fwd", self.stage_seg_fwd), ("segment_mean_bwd", self.stage_seg_bwd)]

    def fps_chain_picks(self):
        return self.K

    def fps_chain_rounds(self):
        return fps_rounds(self.ws_fps, self.n_points, self.B, self.N, self.K)

    def step(self):
        for _, fn in self.stage_list():
            fn()
        return self.out

    def edges(self):
        return int(self.row_ptr[-1].item())

    def stage_bytes(self, E):
        """algorithmic bytes per launch of each stage"""
        nc, C = self.nc, self.C
        return {
            "fps": 12 * self.n_points + 8 * nc,  # coordinates read once, indices written
            "radius_graph": 12 * nc + 16 * E + 8 * (nc + 1),  # points in, (src, dst) i64 + row_ptr out
            # messages are node features gathered through src32: the node table once, not E rows
            "segment_mean_fwd": 4 * nc * C + 4 * nc * C + 4 * (E + 2 * nc),
            "segment_mean_bwd": 4 * nc * C + 4 * E * C + 4 * 2 * nc,
        }

    def e2e_step(self):
        """Public API, host buffers in and out. The feature upload runs on a second stream while
        FPS and the radius graph run, and the result's download while the backward runs."""
        main = torch.cuda.current_stream(self.dev)
        if not hasattr(self, "_copy_stream"):
            self._copy_stream = torch.cuda.Stream(self.dev)
            self._host_out = torch.empty(self.nc, self.C, dtype=torch.float32).pin_memory()
        cs = self._copy_stream
        cs.wait_stream(main)  # the previous step's readers of the feature buffer are done
        pos = self.pos_h.to(self.dev, non_blocking=True)
        with torch.cuda.stream(cs):
            feat = self.feat_h.to(self.dev, non_blocking=True)
        idx, cent = csrc.fps_cuda(pos, self.ptr_h, self.k_h, return_pos=True)
        row_ptr, src, _, rp32, src32 = csrc.radius_graph_csr(cent, self.R, self.cptr_h, max_num_neighbors=self.NN,
                                                             int32_csr=True)
        ns, ne = rp32[:-1], rp32[1:]
        main.wait_stream(cs)
        feat.record_stream(main)
        out = csrc.segment_reduce_cuda(feat, src32, ns, ne, self.nc, "mean")
        cs.wait_stream(main)
        with torch.cuda.stream(cs):
            self._host_out.copy_(out, non_blocking=True)
        out.record_stream(cs)
        g = csrc.segment_reduce_backward_cuda(self.gout, self.gmsg, None, None, None, ns, ne, self.nc, "mean",
                                              grad_msg=self.gmsg)
        main.synchronize()
        cs.synchronize()
        del g
        return self._host_out

    e2e_h2d = property(lambda self: self.pos_h.numel() * 4 + self.feat_h.numel() * 4)
    e2e_d2h = property(lambda self: self.nc * self.C * 4)

    def cpu_step(self, O):
        pos = self.pos_h.numpy()
        idx = O.fps(pos, self.ptr_h.numpy(), self.k_h.numpy(), dist=O.DIST_CUDA)
        cent = pos[idx]
        rp, src = O.radius_graph(cent, self.cptr_h.numpy(), self.R, self.NN, dist=O.DIST_CUDA)
        ns, ne = rp[:-1].astype(np.int32), rp[1:].astype(np.int32)
        out = O.segment_reduce(self.feat_h.numpy(), src.astype(np.int32), ns, ne, self.nc, "mean")
        O.segment_reduce_backward(self._gout_h, np.zeros((len(src), self.C), np.float32), out, None, ns, ne,
                                  self.nc, "mean")
        return out


def _csr_uniform(nq, k, dev):
    """CSR of `nq` destinations with `k` consecutive slots each (a KNN graph)."""
    ns = (torch.arange(nq, dtype=torch.int32, device=dev) * k).contiguous()
    return ns, (ns + k).contiguous()


class C1:
    """4 clouds x 2048 uniform points: FPS 512 -> KNN k=16 -> segment sum + max (C=64)."""
    cpu_fraction = 1.0
    cpu_sample = "full steps"
    points_per_step = property(lambda self: self.B * self.N)
    name = "c1"
    metric = "points/sec (FPS 512 + KNN k=16 + segment sum and max C=64), config 1"
    B, N, K, KNN, C = 4, 2048, 512, 16, 64
    launches_per_step = 1 + 3 + 2 + 2  # fps; knn tiles + fast + merge (+ exact replay); 2 x segment (short + long)

    def _host_init(self, seed, pin=True):
        pos, ptr = synthetic.c1_points(seed=seed, B=self.B, N=self.N)
        self.n_points = pos.shape[0]
        self.nq = self.B * self.K
        self.pos_h = torch.from_numpy(pos)
        self.ptr_h = torch.from_numpy(ptr)
        self.k_h = torch.full((self.B,), self.K, dtype=torch.int64)
        self.pq_h = torch.arange(0, self.nq + 1, self.K, dtype=torch.int64)
        self.msg_h = torch.from_numpy(synthetic.c1_features(seed=seed + 1, E=self.nq * self.KNN, C=self.C))
        if pin:
            self.pos_h, self.msg_h = self.pos_h.pin_memory(), self.msg_h.pin_memory()

    def __init__(self, dev, seed):
        self.dev = dev
        self._host_init(seed)
        self.pos, self.ptr, self.k, self.pq = (t.to(dev) for t in (self.pos_h, self.ptr_h, self.k_h, self.pq_h))
        self.msg = self.msg_h.to(dev)
        L = self.L = nat.load()
        self.idx = torch.empty(self.nq, dtype=torch.int64, device=dev)
        self.cent = torch.empty(self.nq, 3, device=dev)
        self.nidx = torch.empty(self.nq, self.KNN, dtype=torch.int64, device=dev)
        self.ndist = torch.empty(self.nq, self.KNN, device=dev)
        self.ns, self.ne = _csr_uniform(self.nq, self.KNN, dev)
        self.out_sum = torch.empty(self.nq, self.C, device=dev)
        self.out_max = torch.empty(self.nq, self.C, device=dev)
        self.arg = torch.empty(self.nq, self.C, dtype=torch.int32, device=dev)
        self.ws_fps = nat.workspace(L.gdl_fps_workspace_size(self.n_points, self.B, self.N), dev)
        self.ws_knn = nat.workspace(L.gdl_knn_workspace_size(self.nq, self.B, self.KNN, self.N), dev)
        self.ws_seg = nat.workspace(L.gdl_segment_reduce_workspace_size(self.nq * self.KNN, self.nq), dev)

    def _s(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def stage_fps(self):
        nat.check(self.L.gdl_fps(self.pos.data_ptr(), self.ptr.data_ptr(), self.k.data_ptr(), self.B, self.n_points,
                                 self.N, 0, self.idx.data_ptr(), self.cent.data_ptr(), self.ws_fps.data_ptr(),
                                 self.ws_fps.numel(), self._s()), "fps")

    def stage_knn(self):
        nat.check(self.L.gdl_knn(self.cent.data_ptr(), self.pos.data_ptr(), self.pq.data_ptr(), self.ptr.data_ptr(),
                                 self.B, self.nq, self.KNN, self.N, self.nidx.data_ptr(), self.ndist.data_ptr(),
                                 self.ws_knn.data_ptr(), self.ws_knn.numel(), self._s()), "knn")

    def _seg(self, red, out, arg):
        nat.check(self.L.gdl_segment_reduce(self.msg.data_ptr(), 0, self.nq * self.KNN, self.C, None,
                                            self.ns.data_ptr(), self.ne.data_ptr(), self.nq, red, out.data_ptr(),
                                            nat.ptr(arg), self.ws_seg.data_ptr(), self.ws_seg.numel(), self._s()),
                  "segment")

    def stage_list(self):
        return [("fps", self.stage_fps), ("knn", self.stage_knn),
                ("segment_sum", lambda: self._seg(0, self.out_sum, None)),
                ("segment_max", lambda: self._seg(2, self.out_max, self.arg))]

    def fps_chain_picks(self):
        return self.K

    def fps_chain_rounds(self):
        return fps_rounds(self.ws_fps, self.n_points, self.B, self.N, self.K)

    def knn_pairs(self):
        return self.B * self.K * self.N

    def knn_evaluated(self):
        return knn_distances(self.ws_knn, self.nq, self.B, self.KNN, self.N)

    def step(self):
        for _, fn in self.stage_list():
            fn()

    def edges(self):
        return self.nq * self.KNN

    def stage_bytes(self, E):
        nq, C = self.nq, self.C
        return {"fps": 12 * self.n_points + 20 * nq,
                "knn": 12 * (nq + self.n_points) + 12 * nq * self.KNN,
                "segment_sum": 4 * E * C + 4 * nq * C + 8 * nq,
                "segment_max": 4 * E * C + 8 * nq * C + 8 * nq}

    def e2e_step(self):
        pos = self.pos_h.to(self.dev, non_blocking=True)
        msg = self.msg_h.to(self.dev, non_blocking=True)
        idx, cent = csrc.fps_cuda(pos, self.ptr_h, self.k_h, return_pos=True)
        nidx, _ = F.knn(cent, pos, self.pq, self.ptr, self.KNN)
        s_ = csrc.segment_reduce_cuda(msg, None, self.ns, self.ne, self.nq, "sum")
        m_ = csrc.segment_reduce_cuda(msg, None, self.ns, self.ne, self.nq, "max")
        host = [t.to("cpu", non_blocking=True) for t in (nidx, s_, m_)]
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    e2e_h2d = property(lambda self: self.pos_h.numel() * 4 + self.msg_h.numel() * 4)
    e2e_d2h = property(lambda self: self.nq * self.KNN * 8 + 2 * self.nq * self.C * 4)

    def cpu_step(self, O):
        pos = self.pos_h.numpy()
        idx = O.fps(pos, self.ptr_h.numpy(), self.k_h.numpy(), dist=O.DIST_CUDA)
        O.knn(pos[idx], pos, self.pq_h.numpy(), self.ptr_h.numpy(), self.KNN, dist=O.DIST_CUDA)
        ns = (np.arange(self.nq) * self.KNN).astype(np.int32)
        O.segment_reduce(self.msg_h.numpy(), None, ns, ns + self.KNN, self.nq, "sum")
        O.segment_reduce(self.msg_h.numpy(), None, ns, ns + self.KNN, self.nq, "max")


class C3:
    """32 GMM clouds x 8192 points: FPS chain 8192 -> 2048 -> 512 -> 128, KNN k=32 of each
    level's centroids into the previous level's points, segment max over the gathered bf16
    features of those points (C = 64 / 128 / 256, fp32 compare), forward and backward."""
    name = "c3"
    metric = ("points/sec (FPS chain 8192->2048->512->128 + KNN k=32 per level + bf16 segment max fwd+bwd), "
              "config 3")
    B, N, KNN = 32, 8192, 32
    LEVELS = (2048, 512, 128)
    CH = (64, 128, 256)
    # per level: fps 1; knn tiles + pad + fast + merge + exact replay 5; gather 1; segment max fwd 2
    # (short + long pass) and bwd 2
    # fps: level 0 bucketed, levels 1-2 one CTA kernel each; per level: knn tiles + pad + fast +
    # merge + exact replay 5; gather 1; segment max fwd 2 (short + long pass) and bwd 2
    launches_per_step = FPS_BUCKETED_LAUNCHES + 2 + 3 * (5 + 1 + 2 + 2)
    points_per_step = property(lambda self: self.B * self.N)

    def _sizes(self):
        return (self.N,) + self.LEVELS

    def _host_init(self, seed, pin=True):
        pos, ptr = synthetic.c3_points(seed=seed, B=self.B, N=self.N)
        sz = self._sizes()
        self.pos_h = torch.from_numpy(pos)
        self.lptr_h = [torch.arange(0, self.B * n + 1, n, dtype=torch.int64) for n in sz]
        self.k_h = [torch.full((self.B,), n, dtype=torch.int64) for n in self.LEVELS]
        # features of the points each level's KNN searches (levels 0, 1, 2)
        self.feat_h = [synthetic.c3_level_features(self.B * sz[l], self.CH[l], seed + 1 + l) for l in range(3)]
        g = torch.Generator().manual_seed(seed + 7)
        self.gout_h = [torch.randn(self.B * self.LEVELS[l], self.CH[l], generator=g) for l in range(3)]
        if pin:
            self.pos_h = self.pos_h.pin_memory()
            self.feat_h = [f.pin_memory() for f in self.feat_h]

    def __init__(self, dev, seed):
        self.dev = dev
        self._host_init(seed)
        L = self.L = nat.load()
        sz = self._sizes()
        self.pos = self.pos_h.to(dev)
        self.lptr = [t.to(dev) for t in self.lptr_h]
        self.k = [t.to(dev) for t in self.k_h]
        self.feat = [t.to(dev) for t in self.feat_h]
        self.gout = [t.to(dev) for t in self.gout_h]
        nq = [self.B * n for n in self.LEVELS]
        self.nq = nq
        self.idx = [torch.empty(n, dtype=torch.int64, device=dev) for n in nq]
        self.cent = [torch.empty(n, 3, device=dev) for n in nq]
        self.nidx = [torch.empty(n, self.KNN, dtype=torch.int64, device=dev) for n in nq]
        self.ndist = [torch.empty(n, self.KNN, device=dev) for n in nq]
        self.csr = [_csr_uniform(n, self.KNN, dev) for n in nq]
        self.msg = [torch.empty(nq[l] * self.KNN, self.CH[l], dtype=torch.bfloat16, device=dev) for l in range(3)]
        self.gmsg = [torch.empty_like(m) for m in self.msg]
        self.out = [torch.empty(nq[l], self.CH[l], device=dev) for l in range(3)]
        self.arg = [torch.empty(nq[l], self.CH[l], dtype=torch.int32, device=dev) for l in range(3)]
        self.ws_fps = [nat.workspace(L.gdl_fps_workspace_size(self.B * sz[l], self.B, sz[l]), dev) for l in range(3)]
        self.ws_knn = [nat.workspace(L.gdl_knn_workspace_size(nq[l], self.B, self.KNN, sz[l]), dev) for l in range(3)]
        self.ws_seg = [nat.workspace(L.gdl_segment_reduce_workspace_size(nq[l] * self.KNN, nq[l]), dev)
                       for l in range(3)]

    def _s(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def _src(self, l):
        return self.pos if l == 0 else self.cent[l - 1]

    def stage_fps(self):
        sz = self._sizes()
        for l in range(3):
            ws = self.ws_fps[l]
            nat.check(self.L.gdl_fps(self._src(l).data_ptr(), self.lptr[l].data_ptr(), self.k[l].data_ptr(), self.B,
                                     self.B * sz[l], sz[l], 0, self.idx[l].data_ptr(), self.cent[l].data_ptr(),
                                     ws.data_ptr(), ws.numel(), self._s()), "fps")

    def stage_knn(self):
        sz = self._sizes()
        for l in range(3):
            ws = self.ws_knn[l]
            nat.check(self.L.gdl_knn(self.cent[l].data_ptr(), self._src(l).data_ptr(), self.lptr[l + 1].data_ptr(),
                                     self.lptr[l].data_ptr(), self.B, self.nq[l], self.KNN, sz[l],
                                     self.nidx[l].data_ptr(), self.ndist[l].data_ptr(), ws.data_ptr(), ws.numel(),
                                     self._s()), "knn")

    def stage_gather(self):  # msg = feats[knn_idx], materialised
        for l in range(3):
            f = self.feat[l]
            nat.check(self.L.gdl_gather_rows(f.data_ptr(), f.shape[0], f.shape[1] * 2, self.nidx[l].data_ptr(),
                                             self.msg[l].shape[0], self.msg[l].data_ptr(), self._s()), "gather")

    def stage_seg_fwd(self):
        for l in range(3):
            ns, ne = self.csr[l]
            ws = self.ws_seg[l]
            nat.check(self.L.gdl_segment_reduce(self.msg[l].data_ptr(), 1, self.msg[l].shape[0], self.CH[l], None,
                                                ns.data_ptr(), ne.data_ptr(), self.nq[l], 2, self.out[l].data_ptr(),
                                                self.arg[l].data_ptr(), ws.data_ptr(), ws.numel(), self._s()),
                      "segment max")

    def stage_seg_bwd(self):
        for l in range(3):
            ns, ne = self.csr[l]
            ws = self.ws_seg[l]
            nat.check(self.L.gdl_segment_reduce_backward(self.gout[l].data_ptr(), self.msg[l].data_ptr(), 1,
                                                         self.out[l].data_ptr(), self.arg[l].data_ptr(),
                                                         self.msg[l].shape[0], self.CH[l], None, ns.data_ptr(),
                                                         ne.data_ptr(), self.nq[l], 2, self.gmsg[l].data_ptr(),
                                                         ws.data_ptr(), ws.numel(), self._s()), "segment max bwd")

    def stage_list(self):
        return [("fps_chain", self.stage_fps), ("knn", self.stage_knn), ("gather", self.stage_gather),
                ("segment_max_fwd", self.stage_seg_fwd), ("segment_max_bwd", self.stage_seg_bwd)]

    def fps_chain_picks(self):
        return sum(self.LEVELS)

    def fps_chain_rounds(self):
        sz = self._sizes()
        return sum(fps_rounds(self.ws_fps[l], self.B * sz[l], self.B, sz[l], self.LEVELS[l]) for l in range(3))

    def knn_pairs(self):
        sz = self._sizes()
        return sum(self.B * self.LEVELS[l] * sz[l] for l in range(3))

    def knn_evaluated(self):
        sz = self._sizes()
        return sum(knn_distances(self.ws_knn[l], self.nq[l], self.B, self.KNN, sz[l]) for l in range(3))

    def step(self):
        for _, fn in self.stage_list():
            fn()

    def edges(self):
        return sum(n * self.KNN for n in self.nq)

    def stage_bytes(self, E):
        sz, K = self._sizes(), self.KNN
        nsrc = [self.B * n for n in sz]
        return {
            "fps_chain": sum(12 * nsrc[l] + 20 * self.nq[l] for l in range(3)),
            "knn": sum(12 * (self.nq[l] + nsrc[l]) + 12 * self.nq[l] * K for l in range(3)),
            "gather": sum(4 * self.nq[l] * K * self.CH[l] + 8 * self.nq[l] * K for l in range(3)),
            # bf16 messages in; fp32 max + int32 arg out; 8 bytes of offsets per segment
            "segment_max_fwd": sum(2 * self.nq[l] * K * self.CH[l] + 8 * self.nq[l] * (self.CH[l] + 1)
                                   for l in range(3)),
            # fp32 grad_out + int32 arg in; bf16 grad for every message slot out
            "segment_max_bwd": sum(8 * self.nq[l] * (self.CH[l] + 1) + 2 * self.nq[l] * K * self.CH[l]
                                   for l in range(3)),
        }

    def e2e_step(self):
        pos = self.pos_h.to(self.dev, non_blocking=True)
        feats = [f.to(self.dev, non_blocking=True) for f in self.feat_h]
        src, outs = pos, []
        for l in range(3):
            _, cent = csrc.fps_cuda(src, self.lptr_h[l], self.k_h[l], return_pos=True)
            nidx, _ = csrc.knn_cuda(cent, src, self.lptr_h[l + 1], self.lptr_h[l], self.KNN)
            msg = csrc.gather_rows(feats[l], nidx)
            ns, ne = self.csr[l]
            out, arg = csrc.segment_reduce_cuda(msg, None, ns, ne, self.nq[l], "max", with_arg=True)
            csrc.segment_reduce_backward_cuda(self.gout[l], msg, out, arg, None, ns, ne, self.nq[l], "max",
                                              grad_msg=self.gmsg[l])
            outs.append(out.to("cpu", non_blocking=True))
            src = cent
        torch.cuda.current_stream(self.dev).synchronize()
        return outs

    e2e_h2d = property(lambda self: self.pos_h.numel() * 4 + sum(f.numel() * 2 for f in self.feat_h))
    e2e_d2h = property(lambda self: sum(self.nq[l] * self.CH[l] * 4 for l in range(3)))

    cpu_clouds = 1
    cpu_fraction = 1 / 32
    cpu_sample = "1 of 32 clouds (FPS chain, KNN per level, bf16 segment max fwd+bwd) per sample, scaled x32"

    def cpu_step(self, O):
        sz = self._sizes()
        src = self.pos_h.numpy()[: self.N]
        for l in range(3):
            n, m = sz[l], self.LEVELS[l]
            idx = O.fps(src, [0, n], [m], dist=O.DIST_CUDA)
            cent = src[idx]
            nidx, _ = O.knn(cent, src, [0, m], [0, n], self.KNN, dist=O.DIST_CUDA)
            bits = self.feat_h[l][:n].view(torch.int16).numpy().view(np.uint16)
            msg = bits[nidx.reshape(-1)]
            ns = (np.arange(m) * self.KNN).astype(np.int32)
            out = O.segment_reduce(msg, None, ns, ns + self.KNN, m, "max")
            O.segment_reduce_backward(self.gout_h[l][:m].numpy(), msg, out, None, ns, ns + self.KNN, m, "max")
            src = cent


class C3I:
    """Auxiliary KNN-aggregation workload (the reference's EquivariantInterpolate decoder pass,
    nn/modules/equivariant_interp.py:58-139, on config 3's clouds): the FPS hierarchy
    8192 -> 2048 -> 512 -> 128 of 32 GMM clouds is built once; a step upsamples 128 -> 512 ->
    2048 -> 8192 per cloud: KNN k = 3 of the dense points among the coarse ones, inverse-distance
    weights, weighted sums of C scalar and C/4 x 3 vector channels (C = 256 / 128 / 64), and the
    backward to the coarse features."""
    name = "c3i"
    metric = ("points/sec (KNN k=3 + inverse-distance interpolation of scalar+vector features, fwd+bwd, "
              "128->512->2048->8192), config 3 clouds")
    B, N, KNN = 32, 8192, 3
    SIZES = (8192, 2048, 512, 128)
    CH = (64, 128, 256)  # channels of the coarse level of each step (dense level l <- coarse l + 1)
    # per step l: knn 5; idw 1 + two weighted sums; backward: keys 1 + radix + offsets 1 + 2 tables
    points_per_step = property(lambda self: self.B * self.N)
    cpu_fraction = 1 / 32
    cpu_sample = "the three interpolation steps (KNN, weights, sums, backward) of 1 of 32 clouds, scaled x32"

    @staticmethod
    def _radix_launches(n_src):
        bits = 1
        while bits < 32 and (1 << bits) <= n_src:
            bits += 1
        return 1 + 4 * ((bits + 7) // 8)

    @property
    def launches_per_step(self):
        n = 0
        for l in range(3):
            n += 5 + 3 + 1 + self._radix_launches(self.B * self.SIZES[l + 1]) + 1 + 2
        return n

    def knn_pairs(self):  # dense level l's points against coarse level l + 1's
        return sum(self.B * self.SIZES[l] * self.SIZES[l + 1] for l in range(3))

    def knn_evaluated(self):
        return sum(knn_distances(self.ws_knn[l], self.B * self.SIZES[l], self.B, self.KNN, self.SIZES[l + 1])
                   for l in range(3))

    def _host_init(self, seed, pin=True):
        pos, ptr = synthetic.c3_points(seed=seed, B=self.B, N=self.N)
        self.pos_h = torch.from_numpy(pos)
        self.lptr_h = [torch.arange(0, self.B * n + 1, n, dtype=torch.int64) for n in self.SIZES]
        g = torch.Generator().manual_seed(seed + 3)
        self.s_h = [torch.randn(self.B * self.SIZES[l + 1], self.CH[l], generator=g) for l in range(3)]
        self.v_h = [torch.randn(self.B * self.SIZES[l + 1], self.CH[l] // 4, 3, generator=g) for l in range(3)]
        self.gs_h = [torch.randn(self.B * self.SIZES[l], self.CH[l], generator=g) for l in range(3)]
        self.gv_h = [torch.randn(self.B * self.SIZES[l], self.CH[l] // 4, 3, generator=g) for l in range(3)]
        if pin:
            self.pos_h = self.pos_h.pin_memory()

    def _levels(self, dev):
        """positions of every level: FPS chain on the device (setup, untimed)."""
        lv = [self.pos_h.to(dev)]
        for l in range(3):
            idx, cent = csrc.fps_cuda(lv[-1], self.lptr_h[l], torch.full((self.B,), self.SIZES[l + 1]),
                                      return_pos=True)
            lv.append(cent)
        return lv

    def __init__(self, dev, seed):
        self.dev = dev
        self._host_init(seed)
        L = self.L = nat.load()
        self.lv = self._levels(dev)
        self.lptr = [t.to(dev) for t in self.lptr_h]
        self.s = [t.to(dev) for t in self.s_h]
        self.v = [t.to(dev) for t in self.v_h]
        self.gs = [t.to(dev) for t in self.gs_h]
        self.gv = [t.to(dev) for t in self.gv_h]
        nq = [self.B * self.SIZES[l] for l in range(3)]
        self.nq = nq
        self.idx = [torch.empty(n, self.KNN, dtype=torch.int64, device=dev) for n in nq]
        self.dist = [torch.empty(n, self.KNN, device=dev) for n in nq]
        self.w = [torch.empty(n, self.KNN, device=dev) for n in nq]
        self.so = [torch.empty(nq[l], self.CH[l], device=dev) for l in range(3)]
        self.vo = [torch.empty(nq[l], self.CH[l] // 4, 3, device=dev) for l in range(3)]
        self.gsrc_s = [torch.empty_like(t) for t in self.s]
        self.gsrc_v = [torch.empty_like(t) for t in self.v]
        self.ws_knn = [nat.workspace(L.gdl_knn_workspace_size(nq[l], self.B, self.KNN, self.SIZES[l + 1]), dev)
                       for l in range(3)]
        self.ws_bwd = [nat.workspace(L.gdl_knn_weighted_sum_backward_workspace_size(nq[l], self.KNN,
                                                                                   self.B * self.SIZES[l + 1]), dev)
                       for l in range(3)]
        self._ptrs = []
        for l in range(3):
            go = (ctypes.c_void_p * 2)(self.gs[l].data_ptr(), self.gv[l].data_ptr())
            gsrc = (ctypes.c_void_p * 2)(self.gsrc_s[l].data_ptr(), self.gsrc_v[l].data_ptr())
            dims = (ctypes.c_int64 * 2)(self.CH[l], 3 * (self.CH[l] // 4))
            self._ptrs.append((go, gsrc, dims))

    def _s(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def stage_knn(self):
        for l in range(3):
            ws = self.ws_knn[l]
            nat.check(self.L.gdl_knn(self.lv[l].data_ptr(), self.lv[l + 1].data_ptr(), self.lptr[l].data_ptr(),
                                     self.lptr[l + 1].data_ptr(), self.B, self.nq[l], self.KNN, self.SIZES[l + 1],
                                     self.idx[l].data_ptr(), self.dist[l].data_ptr(), ws.data_ptr(), ws.numel(),
                                     self._s()), "knn")

    def stage_fwd(self):
        for l in range(3):
            n, k = self.nq[l], self.KNN
            nat.check(self.L.gdl_knn_idw_weights(self.idx[l].data_ptr(), self.dist[l].data_ptr(), n, k,
                                                 self.w[l].data_ptr(), self._s()), "idw")
            for src, out, dim in ((self.s[l], self.so[l], self.CH[l]), (self.v[l], self.vo[l], 3 * (self.CH[l] // 4))):
                nat.check(self.L.gdl_knn_weighted_sum(src.data_ptr(), src.shape[0], dim, self.idx[l].data_ptr(),
                                                      self.w[l].data_ptr(), n, k, out.data_ptr(), self._s()), "wsum")

    def stage_bwd(self):
        for l in range(3):
            go, gsrc, dims = self._ptrs[l]
            ws = self.ws_bwd[l]
            nat.check(self.L.gdl_knn_weighted_sum_backward(go, gsrc, dims, 2, self.idx[l].data_ptr(),
                                                           self.w[l].data_ptr(), self.nq[l], self.KNN,
                                                           self.s[l].shape[0], ws.data_ptr(), ws.numel(), self._s()),
                      "wsum bwd")

    def stage_list(self):
        return [("knn", self.stage_knn), ("interp_fwd", self.stage_fwd), ("interp_bwd", self.stage_bwd)]

    def step(self):
        for _, fn in self.stage_list():
            fn()

    def edges(self):
        return sum(n * self.KNN for n in self.nq)

    def stage_bytes(self, E):
        k = self.KNN
        b = {"knn": 0, "interp_fwd": 0, "interp_bwd": 0}
        for l in range(3):
            nq, nc, D = self.nq[l], self.B * self.SIZES[l + 1], self.CH[l] + 3 * (self.CH[l] // 4)
            b["knn"] += 12 * (nq + nc) + 12 * nq * k
            # idx + dist in, weights out; per table idx + weights in, coarse rows once, output rows
            b["interp_fwd"] += 12 * nq * k + 4 * nq * k + 2 * 12 * nq * k + 4 * nc * D + 4 * nq * D
            # idx in, sorted pairs (keys + positions), per table grad rows in once, grad_src out
            b["interp_bwd"] += 8 * nq * k + 16 * nq * k + 4 * nq * D + 4 * nc * D
        return b

    def e2e_step(self):
        pos = self.pos_h.to(self.dev, non_blocking=True)
        lv = [pos] + self.lv[1:]  # coarse levels come from the encoder; dense points are this step's input
        outs = []
        for l in range(3):
            s = self.s[l].detach().requires_grad_(True)
            v = self.v[l].detach().requires_grad_(True)
            so, vo = F.knn_interpolate(lv[l], lv[l + 1], s, v, self.lptr[l], self.lptr[l + 1], self.KNN)
            torch.autograd.backward([so, vo], [self.gs[l], self.gv[l]])
            outs.append(so)
        host = outs[-1].to("cpu", non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    e2e_h2d = property(lambda self: self.pos_h.numel() * 4)
    e2e_d2h = property(lambda self: self.nq[2] * self.CH[2] * 4)

    def cpu_step(self, O):
        if not hasattr(self, "_cpu_levels"):
            pos = self.pos_h.numpy()[:self.N]
            lv = [pos]
            for l in range(3):
                idx = O.fps(lv[-1], [0, lv[-1].shape[0]], [self.SIZES[l + 1]], dist=O.DIST_CUDA)
                lv.append(lv[-1][idx])
            self._cpu_levels = lv
        lv = self._cpu_levels
        for l in range(3):
            nd, nc = self.SIZES[l], self.SIZES[l + 1]
            idx, dist = O.knn(lv[l], lv[l + 1], [0, nd], [0, nc], self.KNN, dist=O.DIST_CUDA)
            w = O.knn_idw_weights(idx, dist)
            s, v = self.s_h[l].numpy()[:nc], self.v_h[l].numpy()[:nc]
            O.knn_weighted_sum(s, idx, w)
            O.knn_weighted_sum(v, idx, w)
            O.knn_weighted_sum_backward(self.gs_h[l].numpy()[:nd], idx, w, nc)
            O.knn_weighted_sum_backward(self.gv_h[l].numpy()[:nd], idx, w, nc)


class C2C:
    """Auxiliary SE3Conv-layer workload (the reference's SE3Conv, nn/modules/se3_conv.py:287-545, on
    config 2's graph): 16 clouds x 2048 points -> FPS 512 -> SpatialGraph.build (r = 0.2, 32) over
    the 8192 centroids (built once); a step is one SE3Conv(128, 32 -> 128, 32; type-2 16 -> 16)
    forward and backward through autograd: per-node channel mixing (cuBLAS), the radial MLP, the
    fused message + segment-reduce kernel and its backward. Eager launches (autograd)."""
    name = "c2c"
    metric = ("centroids/sec (SE3Conv 128s+32v+16t2 -> 128s+32v+16t2, forward + backward, over the config-2 "
              "centroid radius graph)")
    B, N, K, R, NN = 16, 2048, 512, 0.2, 32
    DIMS = (128, 32, 128, 32, 16, 16)
    capture = False
    launches_per_step = 3  # fused forward, grad of R, grad of the projections (source grouping cached)
    cpu_fraction = 1.0
    cpu_sample = ("full steps: the reference layer's formulas in torch fp32 on the CPU (oracle/se3_ref.py), forward "
                  "and backward through autograd")
    points_per_step = property(lambda self: self.B * self.K)

    def _host_init(self, seed, pin=True):
        pos, ptr = synthetic.c2_points(seed=seed, B=self.B, N=self.N)
        self.pos_h, self.ptr_h = torch.from_numpy(pos), torch.from_numpy(ptr)
        g = torch.Generator().manual_seed(seed + 5)
        n = self.B * self.K
        cs, cv, _, _, ct, _ = self.DIMS
        self.s_h, self.v_h, self.t_h = (torch.randn(n, cs, generator=g), torch.randn(n, cv, 3, generator=g),
                                        torch.randn(n, ct, 5, generator=g))

    def __init__(self, dev, seed):
        from gdl_b200.se3_conv import SE3Conv
        self.dev = dev
        self._host_init(seed)
        idx, cent = csrc.fps_cuda(self.pos_h.to(dev), self.ptr_h, torch.full((self.B,), self.K), return_pos=True)
        batch = torch.arange(self.B, device=dev).repeat_interleave(self.K)
        self.graph = SpatialGraph.build(cent, self.R, max_num_neighbors=self.NN, batch=batch,
                                        num_batch_elements=self.B)
        torch.manual_seed(seed + 6)
        self.conv = SE3Conv(*self.DIMS, radius=self.R).to(dev)
        self.s = self.s_h.to(dev).requires_grad_(True)
        self.v = self.v_h.to(dev).requires_grad_(True)
        self.t = self.t_h.to(dev).requires_grad_(True)
        outs = self.conv(self.s, self.v, self.graph, type2=self.t)
        g = torch.Generator(device=dev).manual_seed(seed + 7)
        self.gouts = [torch.randn(o.shape, device=dev, generator=g) for o in outs]

    def stage_layer(self):
        outs = self.conv(self.s, self.v, self.graph, type2=self.t)
        torch.autograd.backward(list(outs), self.gouts)

    def stage_list(self):
        return [("se3conv_fwd_bwd", self.stage_layer)]

    def step(self):
        self.stage_layer()

    def edges(self):
        return self.graph.E

    def stage_bytes(self, E):
        n = self.B * self.K
        cs, cv, _, _, ct, _ = self.DIMS
        proj = cs + cv + 3 * cv + 3 * cs + 3 * cv + ct + 5 * ct + 3 * ct + cs  # floats per node, nine tables
        out = cs + 3 * cv + 5 * ct
        # fused kernels: per edge R (9) + direction (3) + harmonics (9) floats + slot/edge indices, in the
        # forward and twice in the backward; node tables read and their gradients written once; outputs
        # and their gradients once
        return {"se3conv_fwd_bwd": 3 * E * (4 * 21 + 12) + 4 * n * proj * 3 + 4 * n * out * 3}

    def e2e_step(self):
        s = self.s_h.pin_memory().to(self.dev, non_blocking=True).requires_grad_(True)
        v = self.v_h.pin_memory().to(self.dev, non_blocking=True).requires_grad_(True)
        t = self.t_h.pin_memory().to(self.dev, non_blocking=True).requires_grad_(True)
        outs = self.conv(s, v, self.graph, type2=t)
        torch.autograd.backward(list(outs), self.gouts)
        host = s.grad.to("cpu", non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    e2e_h2d = property(lambda self: 4 * (self.s_h.numel() + self.v_h.numel() + self.t_h.numel()))
    e2e_d2h = property(lambda self: 4 * self.s_h.numel())

    def cpu_step(self, O):
        from oracle import se3_ref
        if not hasattr(self, "_cpu_graph"):
            pos = self.pos_h.numpy()
            idx = O.fps(pos, self.ptr_h.numpy(), np.full(self.B, self.K), dist=O.DIST_CUDA)
            cent = pos[idx]
            rp, src = O.radius_graph(cent, np.arange(0, self.B * self.K + 1, self.K), self.R, self.NN,
                                     dist=O.DIST_CUDA)
            row, col = O.csr_to_coo(rp, src)
            torch.manual_seed(6)
            sd = {}
            cs_i, cv_i, cs_o, cv_o, ct_i, ct_o = self.DIMS
            for name, (o, i) in dict(w_ss=(cs_o, cs_i), w_sv=(cv_o, cs_i), w_vv_scalar=(cv_o, cv_i),
                                     w_vs=(cs_o, cv_i), w_vv_cross=(cv_o, cv_i), w_st2=(ct_o, cs_i),
                                     w_t2t2=(ct_o, ct_i), w_vt2=(ct_o, cv_i), w_t2s=(cs_o, ct_i)).items():
                sd[name + ".weight"] = torch.randn(o, i) / i ** 0.5
            sd["radial_basis.freqs"] = torch.arange(1, 17).float() * np.pi / self.R
            sd["radial_basis.mlp.0.weight"], sd["radial_basis.mlp.0.bias"] = torch.randn(64, 16) / 4, torch.zeros(64)
            sd["radial_basis.mlp.2.weight"], sd["radial_basis.mlp.2.bias"] = torch.randn(9, 64) / 8, torch.zeros(9)
            sd["scalar_bias"] = torch.zeros(cs_o)
            self._cpu_graph = (torch.from_numpy(cent), torch.from_numpy(row), torch.from_numpy(col), sd)
        cent, row, col, sd = self._cpu_graph
        clouds = [(b * self.K, (b + 1) * self.K) for b in range(self.B)]
        leaf = {k: t.clone().requires_grad_(k.endswith("weight") or k.endswith("bias")) for k, t in sd.items()}
        s, v, t = (x.clone().requires_grad_(True) for x in (self.s_h, self.v_h, self.t_h))
        outs = se3_ref.se3_forward(leaf, self.DIMS, cent, row, col, s, v, t, clouds, self.R, dtype=torch.float32)
        torch.autograd.backward(list(outs), [torch.ones_like(o) for o in outs])


class C4:
    """64 source/target pairs x 16384 points: KNN k=1 target->source, 6-channel residual
    features, segment sum per cloud (64 segments x 16384 rows)."""
    name = "c4"
    metric = "points/sec (KNN k=1 target->source + residual segment sum C=6), config 4"
    B, N, KNN, C = 64, 16384, 1, 6
    launches_per_step = 3 + 2  # knn tiles + fast (+ exact replay); segment short + long

    def _host_init(self, seed, pin=True):
        src, tgt, ptr = synthetic.c4_pairs(seed=seed, B=self.B, N=self.N)
        self.n = src.shape[0]
        self.src_h, self.tgt_h = torch.from_numpy(src), torch.from_numpy(tgt)
        if pin:
            self.src_h, self.tgt_h = self.src_h.pin_memory(), self.tgt_h.pin_memory()
        self.ptr_h = torch.from_numpy(ptr)

    def __init__(self, dev, seed):
        self.dev = dev
        self._host_init(seed)
        self.src, self.tgt, self.ptr = self.src_h.to(dev), self.tgt_h.to(dev), self.ptr_h.to(dev)
        L = self.L = nat.load()
        self.nidx = torch.empty(self.n, 1, dtype=torch.int64, device=dev)
        self.ndist = torch.empty(self.n, 1, device=dev)
        self.feat = torch.empty(self.n, self.C, device=dev)
        self.ns = (torch.arange(self.B, dtype=torch.int32, device=dev) * self.N).contiguous()
        self.ne = (self.ns + self.N).contiguous()
        self.out = torch.empty(self.B, self.C, device=dev)
        self.ws_knn = nat.workspace(L.gdl_knn_workspace_size(self.n, self.B, 1, self.N), dev)
        self.ws_seg = nat.workspace(L.gdl_segment_reduce_workspace_size(self.n, self.B), dev)

    def _s(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def stage_knn(self):
        nat.check(self.L.gdl_knn(self.tgt.data_ptr(), self.src.data_ptr(), self.ptr.data_ptr(), self.ptr.data_ptr(),
                                 self.B, self.n, 1, self.N, self.nidx.data_ptr(), self.ndist.data_ptr(),
                                 self.ws_knn.data_ptr(), self.ws_knn.numel(), self._s()), "knn")

    def stage_residual(self):  # [t - s_nn, s_nn x (t - s_nn)] (torch elementwise, 2 kernels)
        s_nn = self.src.index_select(0, self.nidx.view(-1))
        d = self.tgt - s_nn
        torch.cat([d, torch.cross(s_nn, d, dim=1)], dim=1, out=self.feat)

    def stage_seg(self):
        nat.check(self.L.gdl_segment_reduce(self.feat.data_ptr(), 0, self.n, self.C, None, self.ns.data_ptr(),
                                            self.ne.data_ptr(), self.B, 0, self.out.data_ptr(), None,
                                            self.ws_seg.data_ptr(), self.ws_seg.numel(), self._s()), "segment")

    def stage_list(self):
        return [("knn", self.stage_knn), ("residual", self.stage_residual), ("segment_sum", self.stage_seg)]

    def knn_pairs(self):
        return self.B * self.N * self.N

    def knn_evaluated(self):
        return knn_distances(self.ws_knn, self.n, self.B, 1, self.N)

    def step(self):
        for _, fn in self.stage_list():
            fn()

    def edges(self):
        return self.n

    def stage_bytes(self, E):
        return {"knn": 12 * 2 * self.n + 12 * self.n, "residual": 12 * 3 * self.n + 24 * self.n,
                "segment_sum": 4 * self.n * self.C + 4 * self.B * self.C + 8 * self.B}

    def e2e_step(self):
        src = self.src_h.to(self.dev, non_blocking=True)
        tgt = self.tgt_h.to(self.dev, non_blocking=True)
        idx, _ = F.knn(tgt, src, self.ptr, self.ptr, 1)
        s_nn = src[idx.view(-1)]
        d = tgt - s_nn
        feat = torch.cat([d, torch.cross(s_nn, d, dim=1)], dim=1)
        out = csrc.segment_reduce_cuda(feat, None, self.ns, self.ne, self.B, "sum")
        host = out.to("cpu", non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    e2e_h2d = property(lambda self: 2 * self.n * 12)
    e2e_d2h = property(lambda self: self.B * self.C * 4)

    cpu_clouds = 2  # the CPU sample: 2 of the 64 pairs, scaled to the full batch
    cpu_fraction = 2 / 64
    cpu_sample = "2 of 64 cloud pairs (KNN + residual segment sum) per sample, scaled x32"
    points_per_step = property(lambda self: 2 * self.B * self.N)  # source + target points

    def cpu_step(self, O):
        m = self.cpu_clouds * self.N
        src, tgt = self.src_h.numpy()[:m], self.tgt_h.numpy()[:m]
        ptr = np.arange(0, m + 1, self.N)
        idx, _ = O.knn(tgt, src, ptr, ptr, 1, dist=O.DIST_CUDA)
        s_nn = src[idx[:, 0]]
        d = tgt - s_nn
        feat = np.concatenate([d, np.cross(s_nn, d)], 1).astype(np.float32)
        ns = (np.arange(self.cpu_clouds) * self.N).astype(np.int32)
        O.segment_reduce(feat, None, ns, ns + self.N, self.cpu_clouds, "sum")


class C5:
    """8 LiDAR clouds x 131072 points: FPS 16384 -> radius graph r=1 m, 64 -> segment sum C=64."""
    points_per_step = property(lambda self: self.B * self.N)
    name = "c5"
    metric = "points/sec (FPS 16384 + radius graph r=1 k=64 + segment sum C=64), config 5"
    B, N, K, R, NN, C = 8, 131072, 16384, 1.0, 64, 64
    launches_per_step = FPS_BUCKETED_LAUNCHES + 25 + 2

    shardable = True  # the batch of clouds can be split over ranks (strong scaling)

    def _clouds(self, seed, clouds):
        """This rank's clouds [c0, c1) of the seeded 8-cloud batch (all of it by default)."""
        c0, c1 = clouds if clouds is not None else (0, type(self).B)
        pos, _ = synthetic.c5_points(seed=seed, B=type(self).B, N=self.N)
        self.B = c1 - c0
        return pos[c0 * self.N:c1 * self.N].copy(), synthetic.ptr_of([self.N] * self.B), (c0, c1)

    def _host_init(self, seed, pin=True, clouds=None):
        pos, ptr, (c0, c1) = self._clouds(seed, clouds)
        self.n_points = pos.shape[0]
        self.nc = self.B * self.K
        self.pos_h = torch.from_numpy(pos)
        self.ptr_h = torch.from_numpy(ptr)
        self.k_h = torch.full((self.B,), self.K, dtype=torch.int64)
        self.cptr_h = torch.arange(0, self.nc + 1, self.K, dtype=torch.int64)
        g = torch.Generator().manual_seed(seed + 1)
        self.feat_h = torch.randn(type(self).B * self.K, self.C, generator=g)[c0 * self.K:c1 * self.K].contiguous()
        if pin:
            self.pos_h, self.feat_h = self.pos_h.pin_memory(), self.feat_h.pin_memory()

    def __init__(self, dev, seed, clouds=None):
        self.dev = dev
        self._host_init(seed, clouds=clouds)
        self.pos, self.ptr, self.k, self.cptr = (t.to(dev) for t in (self.pos_h, self.ptr_h, self.k_h, self.cptr_h))
        self.feat = self.feat_h.to(dev)
        self.cap = self.nc * self.NN
        L = self.L = nat.load()
        self.idx = torch.empty(self.nc, dtype=torch.int64, device=dev)
        self.cent = torch.empty(self.nc, 3, device=dev)
        self.row_ptr = torch.empty(self.nc + 1, dtype=torch.int64, device=dev)
        self.src = torch.zeros(self.cap, dtype=torch.int64, device=dev)
        self.row_ptr32 = torch.zeros(self.nc + 1, dtype=torch.int32, device=dev)
        self.ns, self.ne = self.row_ptr32[:-1], self.row_ptr32[1:]
        self.src32 = torch.zeros(self.cap, dtype=torch.int32, device=dev)
        self.out = torch.empty(self.nc, self.C, device=dev)
        self.ws_fps = nat.workspace(L.gdl_fps_workspace_size(self.n_points, self.B, self.N), dev)
        self.ws_rad = nat.workspace(L.gdl_radius_graph_workspace_size(self.nc, self.B, self.NN), dev)
        self.ws_seg = nat.workspace(L.gdl_segment_reduce_workspace_size(self.cap, self.nc), dev)

    def _s(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def stage_fps(self):
        nat.check(self.L.gdl_fps(self.pos.data_ptr(), self.ptr.data_ptr(), self.k.data_ptr(), self.B, self.n_points,
                                 self.N, 0, self.idx.data_ptr(), self.cent.data_ptr(), self.ws_fps.data_ptr(),
                                 self.ws_fps.numel(), self._s()), "fps")

    def stage_radius(self):
        nat.check(self.L.gdl_radius_graph(self.cent.data_ptr(), self.cptr.data_ptr(), self.B, self.nc, self.K, self.R,
                                          self.NN, 0, None, self.row_ptr.data_ptr(), self.src.data_ptr(), None,
                                          self.row_ptr32.data_ptr(), self.src32.data_ptr(), self.ws_rad.data_ptr(),
                                          self.ws_rad.numel(), self._s()), "radius")

    def stage_seg(self):
        nat.check(self.L.gdl_segment_reduce(self.feat.data_ptr(), 0, self.nc, self.C, self.src32.data_ptr(),
                                            self.ns.data_ptr(), self.ne.data_ptr(), self.nc, 0, self.out.data_ptr(),
                                            None, self.ws_seg.data_ptr(), self.ws_seg.numel(), self._s()), "segment")

    def stage_list(self):
        return [("fps", self.stage_fps), ("radius_graph", self.stage_radius), ("segment_sum", self.stage_seg)]

    def fps_chain_picks(self):
        return self.K

    def fps_chain_rounds(self):
        return fps_rounds(self.ws_fps, self.n_points, self.B, self.N, self.K)

    def knn_pairs(self):  # the hybrid graph's self-KNN over the centroids
        return self.B * self.K * self.K

    def knn_evaluated(self):
        return knn_distances(self.ws_knn, self.nc, self.B, self.KF + 1, self.K)

    def step(self):
        for _, fn in self.stage_list():
            fn()

    def edges(self):
        return int(self.row_ptr[-1].item())

    def stage_bytes(self, E):
        nc, C = self.nc, self.C
        # the segment sum gathers node features through src32: the node table is read once
        return {"fps": 12 * self.n_points + 20 * nc, "radius_graph": 12 * nc + 12 * E + 12 * (nc + 1),
                "segment_sum": 4 * min(E, nc) * C + 4 * nc * C + 4 * (E + 2 * nc)}

    def e2e_step(self):
        # the features are needed only by the last stage: their copy runs on a side stream while
        # FPS runs (copy engine and SMs in parallel); the segment sum waits for it
        main = torch.cuda.current_stream(self.dev)
        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream(self.dev)
        pos = self.pos_h.to(self.dev, non_blocking=True)
        self._copy_stream.wait_stream(main)  # after the positions: FPS needs them first
        with torch.cuda.stream(self._copy_stream):
            feat = self.feat_h.to(self.dev, non_blocking=True)
        idx, cent = csrc.fps_cuda(pos, self.ptr_h, self.k_h, return_pos=True)
        row_ptr, src, _, rp32, src32 = csrc.radius_graph_csr(cent, self.R, self.cptr_h, max_num_neighbors=self.NN,
                                                             int32_csr=True)
        main.wait_stream(self._copy_stream)
        feat.record_stream(main)
        out = csrc.segment_reduce_cuda(feat, src32, rp32[:-1], rp32[1:], self.nc, "sum")
        host = out.to("cpu", non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    e2e_h2d = property(lambda self: self.pos_h.numel() * 4 + self.feat_h.numel() * 4)
    e2e_d2h = property(lambda self: self.nc * self.C * 4)

    cpu_clouds = 1      # the CPU sample: one cloud, first 256 FPS picks, scaled to the full step
    cpu_picks = 256
    cpu_fraction = (256 / 16384) / 8
    cpu_sample = ("FPS of 256 of 16384 picks on 1 of 8 clouds per sample, scaled x512 (FPS dominates this step; "
                  "every pick scans the whole cloud, so its cost is the same for every pick)")

    def cpu_step(self, O):
        pos = self.pos_h.numpy()[:self.N]
        O.fps(pos, [0, self.N], [self.cpu_picks], dist=O.DIST_CUDA)


class C5G(C5):
    """Auxiliary LiDAR graph-build workload (not one of the reference's configurations): config 5's
    clouds, radius graph r = 1 m, 64 neighbours over ALL 131072 points of each cloud, segment sum of
    64-channel point features over it. In config 5 proper the graph is built over the 16384 FPS
    centroids, which FPS leaves >= 1.75 m apart, so r = 1 m gives no edge there."""
    name = "c5g"
    metric = "points/sec (radius graph r=1 k=64 over all points + segment sum C=64), config 5 clouds"
    launches_per_step = 25 + 2

    def _host_init(self, seed, pin=True, clouds=None):
        pos, ptr, (c0, c1) = self._clouds(seed, clouds)
        self.n_points = pos.shape[0]
        self.nc = self.n_points
        self.pos_h = torch.from_numpy(pos)
        self.ptr_h = torch.from_numpy(ptr)
        g = torch.Generator().manual_seed(seed + 1)
        self.feat_h = torch.randn(type(self).B * self.N, self.C, generator=g)[c0 * self.N:c1 * self.N].contiguous()
        if pin:
            self.pos_h, self.feat_h = self.pos_h.pin_memory(), self.feat_h.pin_memory()

    def __init__(self, dev, seed, clouds=None):
        self.dev = dev
        self._host_init(seed, clouds=clouds)
        self.pos, self.ptr = self.pos_h.to(dev), self.ptr_h.to(dev)
        self.feat = self.feat_h.to(dev)
        self.cap = self.nc * self.NN
        L = self.L = nat.load()
        self.row_ptr = torch.empty(self.nc + 1, dtype=torch.int64, device=dev)
        self.src = torch.zeros(self.cap, dtype=torch.int64, device=dev)
        self.row_ptr32 = torch.zeros(self.nc + 1, dtype=torch.int32, device=dev)
        self.ns, self.ne = self.row_ptr32[:-1], self.row_ptr32[1:]
        self.src32 = torch.zeros(self.cap, dtype=torch.int32, device=dev)
        self.out = torch.empty(self.nc, self.C, device=dev)
        self.ws_rad = nat.workspace(L.gdl_radius_graph_workspace_size(self.nc, self.B, self.NN), dev)
        self.ws_seg = nat.workspace(L.gdl_segment_reduce_workspace_size(self.cap, self.nc), dev)

    def stage_radius(self):
        nat.check(self.L.gdl_radius_graph(self.pos.data_ptr(), self.ptr.data_ptr(), self.B, self.nc, self.N, self.R,
                                          self.NN, 0, None, self.row_ptr.data_ptr(), self.src.data_ptr(), None,
                                          self.row_ptr32.data_ptr(), self.src32.data_ptr(), self.ws_rad.data_ptr(),
                                          self.ws_rad.numel(), self._s()), "radius")

    def stage_list(self):
        return [("radius_graph", self.stage_radius), ("segment_sum", self.stage_seg)]

    def stage_bytes(self, E):
        nc, C = self.nc, self.C
        return {"radius_graph": 12 * nc + 12 * E + 12 * (nc + 1),
                "segment_sum": 4 * min(E, nc) * C + 4 * nc * C + 4 * (E + 2 * nc)}

    def e2e_step(self):
        pos = self.pos_h.to(self.dev, non_blocking=True)
        feat = self.feat_h.to(self.dev, non_blocking=True)
        row_ptr, src, _, rp32, src32 = csrc.radius_graph_csr(pos, self.R, self.ptr_h, max_num_neighbors=self.NN,
                                                             int32_csr=True)
        out = csrc.segment_reduce_cuda(feat, src32, rp32[:-1], rp32[1:], self.nc, "sum")
        host = out.to("cpu", non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    e2e_d2h = property(lambda self: self.nc * self.C * 4)
    cpu_fraction = 1 / 8
    cpu_sample = "radius graph + segment sum of 1 of 8 clouds per sample, scaled x8"

    def cpu_step(self, O):
        pos = self.pos_h.numpy()[:self.N]
        rp, src = O.radius_graph(pos, np.array([0, self.N]), self.R, self.NN, dist=O.DIST_CUDA)
        O.segment_reduce(self.feat_h.numpy()[:self.N], src.astype(np.int32), rp[:-1].astype(np.int32),
                         rp[1:].astype(np.int32), self.N, "sum")


class C5H(C5):
    """Config 5 with the reference encoder's hybrid graph in place of the plain radius graph
    (_EncoderStage._build_hybrid_graph, nn/modules/multi_scale_se3_net.py:126-219): FPS 16384 per
    LiDAR cloud, radius graph r = 1 m / 64 over the centroids (empty: FPS leaves them >= 1.75 m
    apart), self-KNN k = 4, both directions of the 3 nearest for every node with fewer than 3
    radius in-edges, deduplicated in (row, col) order with its CSR and each edge's distance,
    direction and l <= 2 harmonics, the per-node average degree, and the segment sum of
    64-channel features over the resulting graph."""
    name = "c5h"
    metric = ("points/sec (FPS 16384 + hybrid radius r=1 k=64 / KNN-3 fallback graph with edge geometry + "
              "segment sum C=64), config 5")
    KF = 3
    MAX_L = 2

    @property
    def launches_per_step(self):
        bits = 1
        while bits < 32 and (1 << bits) <= self.nc:
            bits += 1
        radix = 1 + 4 * ((bits + 7) // 8)
        # fps 1; radius (general path) 25 - 2 segment launches of C5's count; knn 5; hybrid: count,
        # scan 3, fill, unique, scan 3, emit, radix, order; avg degree 2; segment 2
        return FPS_BUCKETED_LAUNCHES + 23 + 5 + (1 + 3 + 1 + 1 + 3 + 1 + radix + 1) + 2 + 2

    def __init__(self, dev, seed, clouds=None):
        super().__init__(dev, seed, clouds)
        L = self.L
        nc = self.nc
        self.cap_h = int(L.gdl_hybrid_graph_capacity(nc, self.NN, self.KF))
        i64, i32 = dict(dtype=torch.int64, device=dev), dict(dtype=torch.int32, device=dev)
        f = dict(dtype=torch.float32, device=dev)
        self.knn_idx = torch.empty(nc, self.KF + 1, **i64)
        self.knn_d = torch.empty(nc, self.KF + 1, **f)
        self.h_rp = torch.empty(nc + 1, **i64)
        self.h_row, self.h_col = torch.empty(self.cap_h, **i64), torch.empty(self.cap_h, **i64)
        self.h_cs, self.h_perm = torch.empty(self.cap_h, **i32), torch.empty(self.cap_h, **i32)
        self.h_src = torch.empty(self.cap_h, **i32)
        self.h_ns, self.h_ne = torch.empty(nc, **i32), torch.empty(nc, **i32)
        self.dist = torch.empty(self.cap_h, **f)
        self.direction = torch.empty(self.cap_h, 3, **f)
        self.sph = torch.empty(self.cap_h, (self.MAX_L + 1) ** 2, **f)
        self.avg = torch.empty(nc, **f)
        self.geom = nat.EdgeGeometry(None, self.dist.data_ptr(), self.direction.data_ptr(), self.sph.data_ptr(),
                                     self.MAX_L)
        self.ws_knn = nat.workspace(L.gdl_knn_workspace_size(nc, self.B, self.KF + 1, self.K), dev)
        self.ws_h = nat.workspace(L.gdl_hybrid_graph_workspace_size(nc, self.NN, self.KF), dev)
        self.ws_avg = nat.workspace(L.gdl_cloud_avg_degree_workspace_size(self.B), dev)
        self.ws_seg_h = nat.workspace(L.gdl_segment_reduce_workspace_size(self.cap_h, nc), dev)

    def stage_knn(self):
        nat.check(self.L.gdl_knn(self.cent.data_ptr(), self.cent.data_ptr(), self.cptr.data_ptr(), self.cptr.data_ptr(),
                                 self.B, self.nc, self.KF + 1, self.K, self.knn_idx.data_ptr(), self.knn_d.data_ptr(),
                                 self.ws_knn.data_ptr(), self.ws_knn.numel(), self._s()), "knn")

    def stage_hybrid(self):
        nat.check(self.L.gdl_hybrid_graph(self.cent.data_ptr(), self.row_ptr.data_ptr(), self.src.data_ptr(),
                                          self.knn_idx.data_ptr(), self.nc, self.NN, self.KF, self.h_rp.data_ptr(),
                                          self.h_row.data_ptr(), self.h_col.data_ptr(), self.h_cs.data_ptr(),
                                          self.h_perm.data_ptr(), self.h_src.data_ptr(), self.h_ns.data_ptr(),
                                          self.h_ne.data_ptr(), ctypes.byref(self.geom), self.ws_h.data_ptr(),
                                          self.ws_h.numel(), self._s()), "hybrid")
        nat.check(self.L.gdl_cloud_avg_degree(self.h_ns.data_ptr(), self.h_ne.data_ptr(), self.nc, None,
                                              self.cptr.data_ptr(), self.B, self.avg.data_ptr(),
                                              self.ws_avg.data_ptr(), self.ws_avg.numel(), self._s()), "avg degree")

    def stage_seg(self):
        nat.check(self.L.gdl_segment_reduce(self.feat.data_ptr(), 0, self.nc, self.C, self.h_src.data_ptr(),
                                            self.h_ns.data_ptr(), self.h_ne.data_ptr(), self.nc, 0, self.out.data_ptr(),
                                            None, self.ws_seg_h.data_ptr(), self.ws_seg_h.numel(), self._s()),
                  "segment")

    def stage_list(self):
        return [("fps", self.stage_fps), ("radius_graph", self.stage_radius), ("knn", self.stage_knn),
                ("hybrid_graph", self.stage_hybrid), ("segment_sum", self.stage_seg)]

    def edges(self):
        return int(self.h_rp[-1].item())

    def stage_bytes(self, E):
        nc, C = self.nc, self.C
        b = super().stage_bytes(E)
        k = self.KF + 1
        b["knn"] = 12 * 2 * nc + 12 * nc * k
        # radius CSR + knn in; per edge (row, col) i64 + col_sorted, perm, src_sorted i32 + dist,
        # direction, 9 harmonics out; node start/end + average degree
        b["hybrid_graph"] = 8 * (nc + 1) + 8 * nc * k + E * (16 + 12 + 52) + 20 * nc
        b["segment_sum"] = 4 * min(E, nc) * C + 4 * nc * C + 4 * (E + 2 * nc)
        return b

    def e2e_step(self):
        from gdl_b200.hybrid_graph import build_hybrid_graph
        pos = self.pos_h.to(self.dev, non_blocking=True)
        feat = self.feat_h.to(self.dev, non_blocking=True)
        idx, cent = csrc.fps_cuda(pos, self.ptr_h, self.k_h, return_pos=True)
        g = build_hybrid_graph(cent, self.R, self.cptr_h, max_num_neighbors=self.NN, knn_fallback_k=self.KF)
        src_of_slot = g.row[g.perm.long()].to(torch.int32)
        out = csrc.segment_reduce_cuda(feat, src_of_slot, g.node_start, g.node_end, self.nc, "sum")
        host = out.to("cpu", non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    cpu_clouds = 1
    cpu_picks = 2048
    cpu_fraction = (2048 / 16384) / 8
    cpu_sample = ("FPS of 2048 of 16384 picks on 1 of 8 clouds per sample, scaled x64 (FPS dominates this step; "
                  "the hybrid graph of those centroids runs in the same sample)")

    def cpu_step(self, O):
        pos = self.pos_h.numpy()[:self.N]
        idx = O.fps(pos, [0, self.N], [self.cpu_picks], dist=O.DIST_CUDA)
        cent = pos[idx]
        n = cent.shape[0]
        rp, src = O.radius_graph(cent, np.array([0, n]), self.R, self.NN, dist=O.DIST_CUDA)
        knn_idx, _ = O.knn(cent, cent, [0, n], [0, n], self.KF + 1, dist=O.DIST_CUDA)
        row, col = O.hybrid_graph(rp, src, knn_idx, self.KF)
        O.edge_geometry(cent, row, col, max_l=self.MAX_L)
        O.sort_and_build_csr(col, n)


class C5S(C5G):
    """Auxiliary graph-geometry workload (the reference's SpatialGraph.build, nn/modules/
    spatial_graph.py:88-167, on config 5's clouds): radius graph r = 1 m, 64 neighbours over all
    131072 points of each cloud with every edge's distance, direction and l <= 2 spherical
    harmonics written by the emission kernel, then the sort-free CSR fields and each cloud's
    average degree."""
    name = "c5s"
    metric = ("points/sec (SpatialGraph.build: radius graph r=1 k=64 + edge dist/direction/spherical "
              "harmonics l<=2 + CSR + avg degree), config 5 clouds")
    launches_per_step = 25 + 1
    MAX_L = 2

    def __init__(self, dev, seed, clouds=None):
        super().__init__(dev, seed, clouds)
        f = dict(dtype=torch.float32, device=dev)
        self.dst = torch.zeros(self.cap, dtype=torch.int64, device=dev)
        self.dist = torch.empty(self.cap, **f)
        self.direction = torch.empty(self.cap, 3, **f)
        self.sph = torch.empty(self.cap, (self.MAX_L + 1) ** 2, **f)
        self.geom = nat.EdgeGeometry(None, self.dist.data_ptr(), self.direction.data_ptr(), self.sph.data_ptr(),
                                     self.MAX_L)
        i32 = dict(dtype=torch.int32, device=dev)
        self.col_sorted, self.perm = torch.empty(self.cap, **i32), torch.empty(self.cap, **i32)
        self.node_start, self.node_end = torch.empty(self.nc, **i32), torch.empty(self.nc, **i32)
        self.avg = torch.empty(self.nc, **f)
        self.batch_h = torch.arange(self.B).repeat_interleave(self.N)
        self.feat_h = torch.empty(0)  # no features in this workload

    def stage_radius_geometry(self):
        nat.check(self.L.gdl_radius_graph_geometry(self.pos.data_ptr(), self.ptr.data_ptr(), self.B, self.nc, self.N,
                                                   self.R, self.NN, 0, None, self.row_ptr.data_ptr(),
                                                   self.src.data_ptr(), self.dst.data_ptr(),
                                                   self.row_ptr32.data_ptr(), self.src32.data_ptr(),
                                                   ctypes.byref(self.geom), self.ws_rad.data_ptr(),
                                                   self.ws_rad.numel(), self._s()), "radius geometry")

    def stage_finish(self):
        nat.check(self.L.gdl_radius_csr_finish(self.row_ptr.data_ptr(), self.dst.data_ptr(), self.nc, self.cap,
                                               self.ptr.data_ptr(), self.B, self.col_sorted.data_ptr(),
                                               self.perm.data_ptr(), self.node_start.data_ptr(),
                                               self.node_end.data_ptr(), self.avg.data_ptr(), self._s()),
                  "csr finish")

    def stage_list(self):
        return [("radius_geometry", self.stage_radius_geometry), ("csr_finish", self.stage_finish)]

    def stage_bytes(self, E):
        nc = self.nc
        # points in; per edge src/dst i64 + src32 + dist + direction + 9 harmonics out; row pointers
        geo = 12 * nc + E * (8 + 8 + 4 + 4 + 12 + 4 * (self.MAX_L + 1) ** 2) + 12 * (nc + 1)
        # row_ptr + dst in; col_sorted + perm out; node_start/end + avg degree out
        return {"radius_geometry": geo, "csr_finish": 8 * (nc + 1) + 8 * E + 8 * E + 12 * nc}

    def e2e_step(self):
        pos = self.pos_h.to(self.dev, non_blocking=True)
        batch = self.batch_h.to(self.dev, non_blocking=True)
        g = SpatialGraph.build(pos, self.R, max_num_neighbors=self.NN, batch=batch, max_l=self.MAX_L,
                               num_batch_elements=self.B)
        host = g.avg_degree.to("cpu", non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    e2e_h2d = property(lambda self: self.pos_h.numel() * 4 + self.batch_h.numel() * 8)
    e2e_d2h = property(lambda self: self.nc * 4 + 8 * (self.B + 1) + 8)  # avg degree + cloud sizes + edge count
    cpu_fraction = 1 / 8
    cpu_sample = "radius graph + edge geometry + CSR + avg degree of 1 of 8 clouds per sample, scaled x8"

    def cpu_step(self, O):
        pos = self.pos_h.numpy()[:self.N]
        rp, src = O.radius_graph(pos, np.array([0, self.N]), self.R, self.NN, dist=O.DIST_CUDA)
        row, col = O.csr_to_coo(rp, src)
        O.edge_geometry(pos, row, col, max_l=self.MAX_L)
        _, _, ns, ne = O.sort_and_build_csr(col, self.N)
        O.cloud_avg_degree(ns, ne)


class SEG:
    """Auxiliary segment-reduce workload (the metric's "segment-reduce HBM GB/s"): 65536 segments x
    32 rows of 64-channel f32 messages (2.1 M rows, 537 MB), read directly (no gather); a step is the
    sum and max forward and their backward (the max's tie-splitting gradient)."""
    name = "seg"
    metric = "points/sec (segment sum + max fwd + bwd, 65536 segments x 32 rows x 64 f32 channels)"
    B, N, DEG, C = 65536, 32, 32, 64
    launches_per_step = 2 + 2 + 2 + 3  # fwd (short + long) x 2; bwd sum 2; bwd max 2 + tie fix-up
    points_per_step = property(lambda self: self.B * self.DEG)  # rows reduced per step
    cpu_fraction = 1 / 64
    cpu_sample = "1024 of 65536 segments (sum and max, forward and backward) per sample, scaled x64"

    def _host_init(self, seed, pin=True):
        g = torch.Generator().manual_seed(seed)
        self.rows = self.B * self.DEG
        self.msg_h = torch.randn(self.rows, self.C, generator=g)
        self.gout_h = torch.randn(self.B, self.C, generator=g)
        if pin:
            self.msg_h = self.msg_h.pin_memory()

    def __init__(self, dev, seed):
        self.dev = dev
        self._host_init(seed)
        self.msg = self.msg_h.to(dev)
        self.gout = self.gout_h.to(dev)
        self.ns, self.ne = _csr_uniform(self.B, self.DEG, dev)
        self.out_sum = torch.empty(self.B, self.C, device=dev)
        self.out_max = torch.empty(self.B, self.C, device=dev)
        self.arg = torch.empty(self.B, self.C, dtype=torch.int32, device=dev)
        self.g_sum = torch.empty_like(self.msg)
        self.g_max = torch.empty_like(self.msg)
        self.L = nat.load()
        self.ws = nat.workspace(self.L.gdl_segment_reduce_workspace_size(self.rows, self.B), dev)

    def _s(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def _fwd(self, red, out, arg):
        nat.check(self.L.gdl_segment_reduce(self.msg.data_ptr(), 0, self.rows, self.C, None, self.ns.data_ptr(),
                                            self.ne.data_ptr(), self.B, red, out.data_ptr(), nat.ptr(arg),
                                            self.ws.data_ptr(), self.ws.numel(), self._s()), "segment fwd")

    def _bwd(self, red, out, arg, g):
        nat.check(self.L.gdl_segment_reduce_backward(self.gout.data_ptr(), self.msg.data_ptr(), 0, nat.ptr(out),
                                                     nat.ptr(arg), self.rows, self.C, None, self.ns.data_ptr(),
                                                     self.ne.data_ptr(), self.B, red, g.data_ptr(),
                                                     self.ws.data_ptr(), self.ws.numel(), self._s()), "segment bwd")

    def stage_list(self):
        return [("segment_sum_fwd", lambda: self._fwd(0, self.out_sum, None)),
                ("segment_max_fwd", lambda: self._fwd(2, self.out_max, self.arg)),
                ("segment_sum_bwd", lambda: self._bwd(0, None, None, self.g_sum)),
                ("segment_max_bwd", lambda: self._bwd(2, self.out_max, self.arg, self.g_max))]

    def step(self):
        for _, fn in self.stage_list():
            fn()

    def edges(self):
        return self.rows

    def stage_bytes(self, E):
        rows, B, C = self.rows, self.B, self.C
        idx = 8 * B  # node start / end
        return {"segment_sum_fwd": 4 * rows * C + 4 * B * C + idx,
                "segment_max_fwd": 4 * rows * C + 8 * B * C + idx,  # + the int32 arg
                "segment_sum_bwd": 4 * B * C + 4 * rows * C + idx,
                "segment_max_bwd": 8 * B * C + 4 * rows * C + idx}  # grad_out + arg in

    def e2e_step(self):
        msg = self.msg_h.to(self.dev, non_blocking=True)
        s_ = csrc.segment_reduce_cuda(msg, None, self.ns, self.ne, self.B, "sum")
        m_, a_ = csrc.segment_reduce_cuda(msg, None, self.ns, self.ne, self.B, "max", with_arg=True)
        host = [t.to("cpu", non_blocking=True) for t in (s_, m_)]
        torch.cuda.current_stream(self.dev).synchronize()
        return host

    e2e_h2d = property(lambda self: self.rows * self.C * 4)
    e2e_d2h = property(lambda self: 2 * self.B * self.C * 4)

    def cpu_step(self, O):
        m = 1024
        msg = self.msg_h.numpy()[: m * self.DEG]
        ns = (np.arange(m) * self.DEG).astype(np.int32)
        out = O.segment_reduce(msg, None, ns, ns + self.DEG, m, "sum")
        mx = O.segment_reduce(msg, None, ns, ns + self.DEG, m, "max")
        O.segment_reduce_backward(self.gout_h.numpy()[:m], msg, out, None, ns, ns + self.DEG, m, "sum")
        O.segment_reduce_backward(self.gout_h.numpy()[:m], msg, mx, None, ns, ns + self.DEG, m, "max")


CONFIGS = {"c1": C1, "c2": C2, "c2c": C2C, "c3": C3, "c3i": C3I, "c4": C4, "c5": C5, "c5g": C5G, "c5h": C5H, "c5s": C5S,
           "seg": SEG}



# ----------------------------------------------------------------------------- helpers
class ClockSampler:
    """NVML samples (every 10 ms) of this GPU's SM clock and throttle reasons while the
    timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, gpu_index: int, period_s: float = 0.01):
        self.idx, self.period = gpu_index, period_s
        self.sm, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()

    def _sample(self, nv, h):
        self.sm.append(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        for name, bit in self.REASONS.items():
            if r & bit:
                self.reasons.add(name)

    def _run(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self._sample(nv, h)
            while not self._stop.wait(self.period):
                self._sample(nv, h)
            self._sample(nv, h)
        except Exception as e:  # no NVML: report nothing rather than guess
            self.error = repr(e)

    def __enter__(self):
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()
        time.sleep(0.02)
        return self

    def __exit__(self, *a):
        self._stop.set()
        self.thread.join(timeout=5)

    def summary(self):
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.sm)}


ROOFLINE_NOTES = {
    "fps": "FPS is a serial chain of picks per cloud. The bucketed kernel makes them in exchange rounds "
           "of up to 16 exact picks (about 6 on LiDAR clouds); its bound is the latency of those "
           "rounds: `peak` is the time per pick of a chain with this run's exchange rounds and nothing "
           "to update (the per-round time of the same kernel and launch shape on clouds of duplicated "
           "points, where every round makes one pick, times `exchange_rounds`, per pick); the rest of "
           "`achieved` is the bucket updates. HBM is irrelevant (the points are read once).",
    "fps_chain": "see fps: the three levels' chains run back to back (the two small levels one pick per "
                 "exchange); `peak` uses the chain's mean per-round time on duplicated points",
    "knn": "the distance scan runs on the FP32 pipe (8 flops per evaluated distance, packed fp32x2); "
           "`peak` is the packed-FMA throughput measured in this run (gdl_fp32_peak); `achieved` counts "
           "the distances the kernels evaluated (gdl_knn_distance_count): clouds of 4097-32767 sources "
           "skip source blocks by an exact bound, so that is fewer than the brute-force pairs "
           "(brute_force_equivalent_tflops is the rate of a scan that evaluates all of them).",
    "se3conv_fwd_bwd": "a whole layer step through eager autograd (cuBLAS projection GEMMs, the radial MLP, "
                       "the fused message kernels and their backward) over a 43.9 K-edge graph: launch-bound; "
                       "the bytes are those of the fused kernels only.",
    "radius_geometry": "dominated by the radius search (candidate scan in L1/L2, not HBM); the geometry "
                       "emission's own DRAM figures are in profiles/geometry_aggregation_kernels.md.",
    "radius_graph": "the radius search scans candidate cells from L1/L2; its algorithmic HBM bytes (points, "
                    "edges) are small next to the candidate work.",
}

STAGE_BOUND = {"fps": "latency", "fps_chain": "latency", "knn": "fp32"}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(config, stage):
    """DRAM bytes per launch of `stage` measured by ncu for `config` (profiles/ncu_traffic.json)."""
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(config, {}).get(stage)


def fps_rounds(ws, n_points, B, max_cloud_points, picks):
    """Exchange rounds of the last FPS call on this workspace for its longest cloud: the bucketed
    kernel's counter (gdl_fps_round_count), or one round per pick for clouds of <= 4096 points."""
    L = nat.load()
    out = ctypes.c_ulonglong(0)
    nat.check(L.gdl_fps_round_count(ws.data_ptr(), n_points, B, max_cloud_points, ctypes.byref(out)),
              "gdl_fps_round_count")
    return int(out.value) if out.value else max(picks - 1, 0)


def knn_distances(ws, n_q, B, k, max_src):
    """Distances the last gdl_knn call with workspace `ws` evaluated (gdl_knn_distance_count)."""
    out = ctypes.c_ulonglong(0)
    nat.check(nat.load().gdl_knn_distance_count(ws.data_ptr(), n_q, B, k, max_src, ctypes.byref(out)),
              "knn distance count")
    return int(out.value)


def fp32_peaks(dev):
    """FP32 FMA throughput of this GPU in TFLOP/s, scalar and packed (gdl_fp32_peak, every SM busy)."""
    L = nat.load()
    blocks, iters = 8 * 148, 4096
    out = torch.empty(blocks * 256, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    res = {}
    for packed in (0, 1):
        best = None
        for _ in range(4):
            ev[0].record()
            nat.check(L.gdl_fp32_peak(out.data_ptr(), iters, packed, blocks, st), "fp32 peak")
            ev[1].record()
            ev[1].synchronize()
            t = ev[0].elapsed_time(ev[1])
            best = t if best is None else min(best, t)
        res["fp32x2" if packed else "fp32"] = L.gdl_fp32_peak_flops(iters, packed, blocks) / (best / 1000) / 1e12
    return res


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ----------------------------------------------------------------------------- arms
def config_of(cfg_cls, n_gpus):
    """The workload description both arms print (identical for the same configuration and N)."""
    strong = getattr(cfg_cls, "shardable", False)
    return {"workload": f"{cfg_cls.name}: {cfg_cls.B} clouds x {cfg_cls.N} points" + ("" if strong else " per GPU"),
            "clouds": cfg_cls.B, "points_per_cloud": cfg_cls.N, "l2": "flushed between steps (256 MiB write)",
            "parallelism": (f"the {cfg_cls.B} clouds sharded by cloud over {n_gpus} GPU(s), no collective in a step"
                            if strong else f"one batch per GPU on {n_gpus} GPU(s), no collective in a step")}


def run_reference_arm(args, cfg_cls):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import oracle as O

    O.lib()
    threads = O.num_threads()
    cfg = cfg_cls.__new__(cfg_cls)
    cfg._host_init(0, pin=False)
    for _ in range(args.warmup):
        cfg.cpu_step(O)
    t = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cfg.cpu_step(O)
        t.append(time.perf_counter() - t0)
    ms = 1000 * sum(t) / len(t) / cfg.cpu_fraction
    value = cfg.points_per_step / (ms / 1000)
    line = {"metric": cfg_cls.metric, "value": value, "unit": "points/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if getattr(cfg_cls, "shardable", False) else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": config_of(cfg_cls, args.gpus),
            "cpu_baseline": {"value": value, "unit": "points/s", "cores": threads, "kind": "port",
                             "sample": f"each step: {cfg.cpu_sample}, on the C restatement of the reference "
                                       f"algorithm (oracle/)"},
            "e2e": {"value": value, "unit": "points/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def cpu_baseline(cfg, seconds=10.0):
    """The C restatement on all host threads, on a bounded sample of the step, scaled to a step."""
    from oracle import oracle as O

    O.lib()
    cfg.cpu_step(O)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        cfg.cpu_step(O)
        n += 1
        if time.perf_counter() - t0 > seconds or n >= 50:
            break
    dt = (time.perf_counter() - t0) / n / cfg.cpu_fraction
    return {"value": cfg.points_per_step / dt, "unit": "points/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} samples of {cfg.name} on the C restatement: {cfg.cpu_sample} "
                      f"({dt * 1000:.1f} ms per full step)"}


class Timed:
    """A configuration's stages, each captured as one CUDA graph (eager if capture fails), timed
    with CUDA events on the launching stream; L2 flushed by a 256 MiB write before each step."""

    def __init__(self, cfg, dev, eager=False):
        self.cfg, self.dev = cfg, dev
        self.stages = cfg.stage_list()
        self.flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.runners = [fn for _, fn in self.stages]
        self.launch = "eager"
        if not eager and getattr(cfg, "capture", True):
            try:
                graphs = []
                for _, fn in self.stages:
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        fn()
                    graphs.append(g)
                self.runners = [g.replay for g in graphs]
                self.graphs = graphs
                self.launch = "one CUDA graph per stage"
            except Exception as e:  # keep going eagerly, say so in the line
                print(f"[bench] graph capture failed, eager launches: {e!r}", file=sys.stderr)
            torch.cuda.synchronize(dev)

    def run(self, steps, barrier=None):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(self.stages) + 1)]
        step_ms, acc = [], [0.0] * len(self.stages)
        if barrier:
            barrier()
        for _ in range(steps):
            self.flush.zero_()
            ev[0].record()
            for i, run in enumerate(self.runners):
                run()
                ev[i + 1].record()
            ev[-1].synchronize()
            step_ms.append(ev[0].elapsed_time(ev[-1]))
            for i in range(len(self.stages)):
                acc[i] += ev[i].elapsed_time(ev[i + 1])
        if barrier:
            barrier()
        return sum(step_ms), {name: acc[i] / steps for i, (name, _) in enumerate(self.stages)}

    def stage_time(self, name, reps=3):
        """Best-of-`reps` device time of one stage's runner (after one warm replay)."""
        i = [n for n, _ in self.stages].index(name)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        self.runners[i]()
        best = None
        for _ in range(reps):
            self.flush.zero_()
            ev[0].record()
            self.runners[i]()
            ev[1].record()
            ev[1].synchronize()
            t = ev[0].elapsed_time(ev[1])
            best = t if best is None else min(best, t)
        return best


def fps_floor_ms(timed, stage):
    """The FPS stage on clouds of duplicated points (every coordinate 0): after the first pick no
    minimum changes, so the bucketed kernel skips every update and only its exchange chain runs."""
    cfg = timed.cfg
    saved = cfg.pos.clone()
    cfg.pos.zero_()
    try:
        return timed.stage_time(stage)
    finally:
        cfg.pos.copy_(saved)
        torch.cuda.synchronize(timed.dev)


def roofline_of(cfg, timed, stage_ms, E, peaks):
    """Roofline object of the configuration's dominant stage (the largest device time)."""
    hbm, hbm_kind = measured_peak()
    dom = max(stage_ms, key=stage_ms.get)
    bound = STAGE_BOUND.get(dom, "hbm")
    r = {"kernel": dom, "bound": bound, "note": ROOFLINE_NOTES.get(dom, "")}
    if bound == "latency":
        # The FPS chain is a sequence of exchange rounds (up to 16 exact picks each in the bucketed
        # kernel, one in the small-cloud kernel); its floor is the same number of rounds with
        # nothing to update: the time per round of the stage on duplicated points (one pick per
        # round there) times this run's round count.
        picks = cfg.fps_chain_picks()
        timed.stage_time(dom)
        rounds = cfg.fps_chain_rounds()
        floor = fps_floor_ms(timed, dom)
        dup_rounds = cfg.fps_chain_rounds()
        floor_round_us = 1000 * floor / max(dup_rounds, 1)
        ach, pk = 1000 * stage_ms[dom] / picks, floor_round_us * rounds / picks
        r.update({"unit": "us/pick", "achieved": ach, "peak": pk, "frac": pk / ach,
                  "picks_per_cloud_chain": picks, "exchange_rounds": rounds,
                  "picks_per_round": picks / max(rounds, 1), "floor_us_per_round": floor_round_us,
                  "peak_source": ("measured in this run: the exchange-only time per round (the same stage on "
                                  "duplicated points, one pick per round) x this run's exchange rounds"),
                  "traffic": ncu_traffic(cfg.name, dom)})
    elif bound == "fp32":
        pairs = cfg.knn_pairs()
        evaluated = cfg.knn_evaluated() if hasattr(cfg, "knn_evaluated") else pairs
        ach = 8 * evaluated / (stage_ms[dom] / 1000) / 1e12
        pk = peaks.get("fp32x2")
        r.update({"unit": "TFLOP/s", "achieved": ach, "peak": pk, "frac": ach / pk if pk else None,
                  "distances_evaluated": evaluated, "brute_force_pairs": pairs,
                  "brute_force_equivalent_tflops": 8 * pairs / (stage_ms[dom] / 1000) / 1e12,
                  "peak_source": "measured in this run (gdl_fp32_peak, packed fp32x2 FMA)",
                  "traffic": ncu_traffic(cfg.name, dom),
                  "hbm_gbs": cfg.stage_bytes(E)[dom] / (stage_ms[dom] / 1000) / 1e9})
    else:
        algo = cfg.stage_bytes(E)[dom]
        ach = algo / (stage_ms[dom] / 1000) / 1e9
        r.update({"unit": "GB/s", "achieved": ach, "peak": hbm, "frac": ach / hbm,
                  "algorithmic_bytes_per_launch": algo, "traffic": ncu_traffic(cfg.name, dom),
                  "peak_source": (f"{hbm_kind} (MEASURED_PEAKS.json hbm_gbs)" if hbm_kind == "measured"
                                  else "fallback 6.65 TB/s")})
    return r


def e2e_ms_of(cfg, steps, barrier=None):
    for _ in range(2):
        cfg.e2e_step()
    if barrier:
        barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        cfg.e2e_step()
    return 1000 * (time.perf_counter() - t0) / steps


def per_config_line(name, dev, args, peaks):
    """One other configuration, measured the same way (steps of its pipeline, HBM-resident inputs)."""
    cfg = CONFIGS[name](dev, seed=0)
    for _ in range(3):
        cfg.step()
    torch.cuda.synchronize(dev)
    timed = Timed(cfg, dev, args.eager)
    steps = args.per_config_steps
    total, stage_ms = timed.run(steps)
    E = cfg.edges()
    out = {"value": cfg.points_per_step * steps / (total / 1000), "unit": "points/s",
           "ms_per_step": total / steps, "steps": steps, "stage_ms": stage_ms,
           "workload": f"{cfg.name}: {cfg.B} clouds x {cfg.N} points", "launch": timed.launch,
           "roofline": roofline_of(cfg, timed, stage_ms, E, peaks)}
    if not args.no_e2e:
        ms = e2e_ms_of(cfg, max(3, min(steps, 10)))
        out["e2e"] = {"value": cfg.points_per_step / (ms / 1000), "unit": "points/s",
                      "h2d_bytes_per_step": cfg.e2e_h2d, "d2h_bytes_per_step": cfg.e2e_d2h}
    if not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(cfg, seconds=min(args.cpu_seconds, 3.0))
    del timed
    return out


def run_ours(args, cfg_cls):
    ws, rank, local = dist_env()
    if ws > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(dev)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(*vals):
        t = torch.tensor([float(v) for v in vals], dtype=torch.float64, device=dev)
        if ws > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return [float(x) for x in t]

    peaks = fp32_peaks(dev)
    # Strong scaling where the batch shards by cloud (8 clouds
    # over up to 8 GPUs): every rank builds the same seeded batch and keeps its own clouds. Other
    # configurations run a full batch per rank (weak scaling).
    strong = getattr(cfg_cls, "shardable", False)
    if strong:
        from gdl_b200.sharding import shard_clouds

        if ws > cfg_cls.B:
            raise SystemExit(f"{cfg_cls.name} has {cfg_cls.B} clouds: at most {cfg_cls.B} ranks")
        c0, c1 = shard_clouds([cfg_cls.N * getattr(cfg_cls, "K", 1)] * cfg_cls.B, ws, rank)
        if args.clouds:  # a smaller batch (the first clouds), e.g. for a profiler capture
            c0, c1 = min(c0, args.clouds), min(c1, args.clouds)
        cfg = cfg_cls(dev, seed=0, clouds=(c0, c1))
        global_points = (min(cfg_cls.B, args.clouds) if args.clouds else cfg_cls.B) * cfg_cls.N
    else:
        cfg = cfg_cls(dev, seed=1000 * rank)
        global_points = ws * cfg.points_per_step
    for _ in range(max(args.warmup, 3)):
        cfg.step()
    torch.cuda.synchronize(dev)
    timed = Timed(cfg, dev, args.eager)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        total_ms, stage_ms = timed.run(args.steps, barrier)
    E = cfg.edges()
    launch = timed.launch
    roof = roofline_of(cfg, timed, stage_ms, E, peaks) if rank == 0 else None

    e2e_ms = None
    if not args.no_e2e:
        e2e_ms = e2e_ms_of(cfg, max(3, min(args.steps, 50)), barrier)
    total_ms, e2e_max = max_over_ranks(total_ms, e2e_ms or 0.0)
    value = global_points * args.steps / (total_ms / 1000)

    weak = None
    if strong and ws > 1:  # the same configuration with a whole batch per rank, for comparison
        del timed
        wcfg = cfg_cls(dev, seed=1000 * rank)
        for _ in range(3):
            wcfg.step()
        wt = Timed(wcfg, dev, args.eager)
        wsteps = max(3, min(args.steps, 20))
        wms, _ = wt.run(wsteps, barrier)
        (wms,) = max_over_ranks(wms)
        weak = {"value": ws * wcfg.points_per_step * wsteps / (wms / 1000), "unit": "points/s",
                "ms_per_step": wms / wsteps, "clouds_per_gpu": wcfg.B}
        del wt, wcfg

    if rank == 0:
        line = {
            "metric": cfg.metric, "value": value, "unit": "points/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config_of(cfg_cls, ws),
            "run": {"clouds_rank0": cfg.B, "edges_rank0": E, "launch": launch},
            "stage_ms": stage_ms,
            "roofline": roof,
            "peaks": {"fp32_tflops": peaks.get("fp32"), "fp32x2_tflops": peaks.get("fp32x2"),
                      "hbm_gbs": measured_peak()[0]},
            "gpu_launches": cfg.launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        if strong:
            line["note"] = ("strong scaling: the 8-cloud batch is split over the ranks; each cloud's FPS is a "
                            "serial chain of 16384 picks on one thread-block cluster, so a rank's time is bounded "
                            "below by one cloud's chain (fps_bucket_kernel) however few clouds it holds")
        if weak:
            line["weak_scaling"] = weak
        if e2e_ms is not None:
            line["e2e"] = {"value": global_points / (e2e_max / 1000), "unit": "points/s",
                           "h2d_bytes_per_step": cfg.e2e_h2d, "d2h_bytes_per_step": cfg.e2e_d2h}
        if not args.no_cpu_baseline and ws == 1:
            line["cpu_baseline"] = cpu_baseline(cfg, seconds=args.cpu_seconds)
        if ws == 1 and not args.no_per_config:
            del timed
            line["per_config"] = {n: per_config_line(n, dev, args, peaks) for n in args.per_config.split(",") if n}
        print(json.dumps(line), flush=True)
    timed = None
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c5", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--eager", action="store_true", help="launch kernels one by one instead of a CUDA graph")
    ap.add_argument("--per-config", default="c1,c2,c3,c4",
                    help="other configurations measured in the same run (N=1 only), in the line's per_config")
    ap.add_argument("--per-config-steps", type=int, default=30)
    ap.add_argument("--no-per-config", action="store_true")
    ap.add_argument("--clouds", type=int, default=0,
                    help="LiDAR configurations (c5*): only the first N clouds of the batch (profiling; 0 = all)")
    args = ap.parse_args()
    cfg_cls = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference_arm(args, cfg_cls)
    return run_ours(args, cfg_cls)


if __name__ == "__main__":
    sys.exit(main())
