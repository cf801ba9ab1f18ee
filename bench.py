"""Benchmark of the B200 point-cloud graph pipeline (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A step is one pass of a configuration's pipeline over its batch of clouds (seeded synthetic
inputs with the shapes of the reference's use cases; see gdl_b200/synthetic.py):

  c2 (default)  16 clouds x 2048 points: FPS -> 512 centroids per cloud, radius graph
                (r = 0.2, 32 neighbours) over the centroids, segment mean of 128-channel
                features over that graph, forward and backward.
  c5            8 clouds x 131072 LiDAR points: FPS -> 16384, radius graph (r = 1 m, 64),
                segment sum of 64-channel features.

value : input points per second with inputs resident in HBM, timed with CUDA events on the
        launching stream, L2 flushed (256 MiB write) between steps, max over ranks.
e2e   : the same through the public Python API (gdl_b200.functional / csrc) with inputs
        copied from pinned host memory and the result copied back inside each timed step.
Under torchrun each rank processes its own batch (weak scaling, no collective in a step).
--impl reference times the reference algorithm's CPU implementation (the C restatement
in oracle/, all host threads) on the same configuration.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
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

L2_FLUSH_BYTES = 256 << 20


# ----------------------------------------------------------------------------- configs
class C2:
    name = "c2"
    metric = "points/sec (FPS 512 + radius graph r=0.2 k=32 + segment mean C=128 fwd+bwd), config 2"
    B, N, K, R, NN, C = 16, 2048, 512, 0.2, 32, 128

    def __init__(self, dev, seed):
        self.dev = dev
        pos, ptr = synthetic.c2_points(seed=seed, B=self.B, N=self.N)
        self.n_points = pos.shape[0]
        self.nc = self.B * self.K
        g = torch.Generator().manual_seed(seed + 1)
        feat = torch.randn(self.nc, self.C, generator=g)
        gout = torch.randn(self.nc, self.C, generator=g)
        self.ptr_h = torch.from_numpy(ptr)
        self.k_h = torch.full((self.B,), self.K, dtype=torch.int64)
        self.cptr_h = torch.arange(0, self.nc + 1, self.K, dtype=torch.int64)
        # host copies (pinned) for the end-to-end leg
        self.pos_h = torch.from_numpy(pos).pin_memory()
        self.feat_h = feat.pin_memory()
        # device-resident inputs
        self.pos = self.pos_h.to(dev)
        self.feat = self.feat_h.to(dev)
        self.gout = gout.to(dev)
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
        self.ws_fps = nat.workspace(L.gdl_fps_workspace_size(self.n_points, self.N), dev)
        self.ws_rad = nat.workspace(L.gdl_radius_graph_workspace_size(self.nc, self.B, self.NN), dev)
        self.ws_seg = nat.workspace(L.gdl_segment_reduce_workspace_size(self.cap, self.nc), dev)

    # kernels of this library launched per step (fps 1; radius 25: grid, keys, radix sort
    # 1 + 4 x 4, gather, query, scan 3, compact; segment fwd 2 + bwd 2)
    launches_per_step = 1 + 25 + 2 + 2

    def step(self, ev=None):
        L, s = self.L, torch.cuda.current_stream(self.dev).cuda_stream
        rec = (lambda i: ev[i].record()) if ev else (lambda i: None)
        rec(0)
        nat.check(L.gdl_fps(self.pos.data_ptr(), self.ptr.data_ptr(), self.k.data_ptr(), self.B, self.n_points,
                            self.N, 0, self.idx.data_ptr(), self.ws_fps.data_ptr(), self.ws_fps.numel(), s), "fps")
        rec(1)
        cent = self.pos.index_select(0, self.idx)
        rec(2)
        nat.check(L.gdl_radius_graph(cent.data_ptr(), self.cptr.data_ptr(), self.B, self.nc, self.R, self.NN, 0, None,
                                     self.row_ptr.data_ptr(), self.src.data_ptr(), self.dst.data_ptr(),
                                     self.ws_rad.data_ptr(), self.ws_rad.numel(), s), "radius")
        rec(3)
        ns = self.row_ptr[:-1].to(torch.int32)
        ne = self.row_ptr[1:].to(torch.int32)
        src32 = self.src.to(torch.int32)
        rec(4)
        # messages = source-point features gathered by the CSR (perm = src), mean per destination
        nat.check(L.gdl_segment_reduce(self.feat.data_ptr(), 0, self.nc, self.C, src32.data_ptr(), ns.data_ptr(),
                                       ne.data_ptr(), self.nc, 1, self.out.data_ptr(), None, self.ws_seg.data_ptr(),
                                       self.ws_seg.numel(), s), "segment mean")
        rec(5)
        # gradient w.r.t. the per-edge messages (slot-indexed rows)
        nat.check(L.gdl_segment_reduce_backward(self.gout.data_ptr(), None, 0, None, None, self.cap, self.C, None,
                                                ns.data_ptr(), ne.data_ptr(), self.nc, 1, self.gmsg.data_ptr(),
                                                self.ws_seg.data_ptr(), self.ws_seg.numel(), s), "segment mean bwd")
        rec(6)
        return self.out

    stages = {"fps": (0, 1), "radius_graph": (2, 3), "segment_mean_fwd": (4, 5), "segment_mean_bwd": (5, 6)}

    def stage_bytes(self, E):
        """algorithmic bytes per launch of each stage"""
        nc, C = self.nc, self.C
        return {
            "fps": 12 * self.n_points + 8 * nc,  # coordinates read once, indices written
            "radius_graph": 12 * nc + 16 * E + 8 * (nc + 1),  # points in, (src, dst) i64 + row_ptr out
            "segment_mean_fwd": 4 * E * C + 4 * nc * C + 4 * (E + 2 * nc),
            "segment_mean_bwd": 4 * nc * C + 4 * E * C + 4 * 2 * nc,
        }

    def e2e_step(self):
        """Public API, host buffers in and out."""
        pos = self.pos_h.to(self.dev, non_blocking=True)
        feat = self.feat_h.to(self.dev, non_blocking=True)
        idx = F.farthest_point_sampling(pos, self.K, ptr=self.ptr_h)
        cent = pos[idx]
        row_ptr, src, _ = F.radius_graph_csr(cent, self.R, self.cptr, max_num_neighbors=self.NN)
        ns, ne = row_ptr[:-1], row_ptr[1:]
        out = csrc.segment_reduce_cuda(feat, src, ns, ne, self.nc, "mean")
        g = csrc.segment_reduce_backward_cuda(self.gout, self.gmsg, None, None, None, ns, ne, self.nc, "mean",
                                              grad_msg=self.gmsg)
        host = out.to("cpu", non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        del g
        return host

    e2e_h2d = property(lambda self: self.pos_h.numel() * 4 + self.feat_h.numel() * 4)
    e2e_d2h = property(lambda self: self.nc * self.C * 4)

    def cpu_step(self, O):
        pos = self.pos_h.numpy()
        idx = O.fps(pos, self.ptr_h.numpy(), self.k_h.numpy(), dist=O.DIST_CUDA)
        cent = pos[idx]
        rp, src = O.radius_graph(cent, self.cptr_h.numpy(), self.R, self.NN, dist=O.DIST_CUDA)
        ns, ne = rp[:-1].astype(np.int32), rp[1:].astype(np.int32)
        out = O.segment_reduce(self.feat_h.numpy(), src.astype(np.int32), ns, ne, self.nc, "mean")
        O.segment_reduce_backward(self.gout.cpu().numpy() if not hasattr(self, "_gout_h") else self._gout_h,
                                  np.zeros((len(src), self.C), np.float32), out, None, ns, ne, self.nc, "mean")
        return out


CONFIGS = {"c2": C2}


# ----------------------------------------------------------------------------- helpers
class ClockSampler:
    """nvidia-smi samples (200 ms) of this GPU while the timed region runs."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            if len(r) >= 9:
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(kernel_stage):
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d.get(kernel_stage)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ----------------------------------------------------------------------------- arms
def run_reference_arm(args, cfg_cls):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import oracle as O

    O.lib()
    threads = O.num_threads()
    cfg = cfg_cls.__new__(cfg_cls)
    # host-only setup (no device needed)
    pos, ptr = synthetic.c2_points(seed=0, B=cfg_cls.B, N=cfg_cls.N)
    cfg.pos_h = torch.from_numpy(pos)
    cfg.ptr_h = torch.from_numpy(ptr)
    cfg.k_h = torch.full((cfg_cls.B,), cfg_cls.K, dtype=torch.int64)
    cfg.nc = cfg_cls.B * cfg_cls.K
    cfg.cptr_h = torch.arange(0, cfg.nc + 1, cfg_cls.K, dtype=torch.int64)
    g = torch.Generator().manual_seed(1)
    cfg.feat_h = torch.randn(cfg.nc, cfg_cls.C, generator=g)
    cfg._gout_h = torch.randn(cfg.nc, cfg_cls.C, generator=g).numpy()
    for _ in range(args.warmup):
        cfg.cpu_step(O)
    t = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cfg.cpu_step(O)
        t.append(time.perf_counter() - t0)
    ms = 1000 * sum(t) / len(t)
    pts = cfg_cls.B * cfg_cls.N
    value = pts / (ms / 1000)
    line = {"metric": cfg_cls.metric, "value": value, "unit": "points/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": cfg_cls.name, "clouds": cfg_cls.B, "points_per_cloud": cfg_cls.N},
            "cpu_baseline": {"value": value, "unit": "points/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} full steps of {cfg_cls.name} on the C restatement"},
            "e2e": {"value": value, "unit": "points/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def cpu_baseline(cfg, seconds=10.0):
    from oracle import oracle as O

    O.lib()
    cfg._gout_h = cfg.gout.cpu().numpy()
    cfg.cpu_step(O)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        cfg.cpu_step(O)
        n += 1
        if time.perf_counter() - t0 > seconds or n >= 50:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": cfg.B * cfg.N / dt, "unit": "points/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} full steps of {cfg.name} on the C restatement ({dt * 1000:.1f} ms/step)"}


def run_ours(args, cfg_cls):
    ws, rank, local = dist_env()
    if ws > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local if ws > 1 else 0)
    torch.cuda.set_device(dev)
    cfg = cfg_cls(dev, seed=1000 * rank)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    nev = 7
    for _ in range(max(args.warmup, 3)):
        cfg.step()
    torch.cuda.synchronize(dev)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(args.steps)]
    step_ms = []
    barrier()
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        for i in range(args.steps):
            flush.zero_()
            cfg.step(evs[i])
        torch.cuda.synchronize(dev)
    barrier()
    for e in evs:
        step_ms.append(e[0].elapsed_time(e[-1]))
    total_ms = sum(step_ms)
    stage_ms = {k: sum(e[b].elapsed_time(e[c]) for e in evs) / args.steps for k, (b, c) in cfg.stages.items()}
    E = int(cfg.row_ptr[-1].item())

    # end-to-end through the public API
    for _ in range(2):
        cfg.e2e_step()
    barrier()
    t0 = time.perf_counter()
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(e2e_steps):
        cfg.e2e_step()
    e2e_ms = 1000 * (time.perf_counter() - t0) / e2e_steps

    t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    total_ms, e2e_ms = float(t[0]), float(t[1])
    pts = cfg.B * cfg.N
    value = ws * pts * args.steps / (total_ms / 1000)
    e2e_val = ws * pts / (e2e_ms / 1000)

    line = None
    if rank == 0:
        peak, peak_kind = measured_peak()
        dom = max(stage_ms, key=stage_ms.get)
        algo = cfg.stage_bytes(E)[dom]
        achieved = algo / (stage_ms[dom] / 1000) / 1e9
        line = {
            "metric": cfg.metric, "value": value, "unit": "points/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{cfg.name}: {cfg.B} clouds x {cfg.N} points per rank", "clouds": cfg.B,
                       "points_per_cloud": cfg.N, "edges": E, "l2": "flushed between steps (256 MiB write)",
                       "parallelism": f"clouds sharded over {ws} GPU(s), no collective in a step"},
            "stage_ms": stage_ms,
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": ncu_traffic(dom),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6.65 TB/s",
                         "algorithmic_bytes_per_launch": algo},
            "e2e": {"value": e2e_val, "unit": "points/s", "h2d_bytes_per_step": cfg.e2e_h2d,
                    "d2h_bytes_per_step": cfg.e2e_d2h},
            "gpu_launches": cfg.launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, seconds=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    cfg_cls = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference_arm(args, cfg_cls)
    return run_ours(args, cfg_cls)


if __name__ == "__main__":
    sys.exit(main())
