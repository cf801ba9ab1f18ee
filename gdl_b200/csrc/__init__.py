"""Operator entry points of the B200 build -- the drop-in for ``geoembodied.csrc``.

Same names, arguments, dtypes and return values as the reference dispatcher
(geoembodied/csrc/__init__.py:120-597); every call runs the sm_100a kernels of
libgdl_b200.so on the current CUDA stream. Differences, all deliberate:

* no CPU fallback and no JIT compile step: CPU tensors raise ``GdlError``; the library is
  built once by ``python -m gdl_b200.build``;
* ``fps_cuda`` takes ``tie_break`` ("reference" = bit-identical to the reference kernel,
  "lowest_index" = torch.argmax order);
* ``radius_graph_cuda`` returns the edges grouped by destination with ascending sources (the
  reference's order is that of its atomic counter, i.e. arbitrary) and accepts clouds of any
  sizes through ``radius_graph_csr``;
* segment reduce also offers mean and max (``segment_reduce_cuda``).
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple

import numpy as np
import torch

from .. import _native as nat

__all__ = [
    "gather_rows",
    "get_radius_graph_backend", "radius_graph_cuda", "radius_graph_csr",
    "segment_reduce_available", "sort_and_build_csr_cuda", "segment_reduce_sum_cuda", "segment_reduce_cuda",
    "segment_reduce_backward_cuda", "knn_available", "knn_cuda", "knn_self_cuda", "fps_available", "fps_cuda",
]


def _available() -> bool:
    try:
        nat.load()
    except Exception:
        return False
    return torch.cuda.is_available()


def get_radius_graph_backend() -> str:
    """'cuda' when the B200 library is usable (reference: csrc/__init__.py:120-127)."""
    return "cuda" if _available() else "unavailable"


def segment_reduce_available() -> bool:
    return _available()


def knn_available() -> bool:
    return _available()


def fps_available() -> bool:
    return _available()


# --------------------------------------------------------------------------- FPS
def fps_cuda(pos: torch.Tensor, ptr: torch.Tensor, k_per_batch: torch.Tensor, *,
             tie_break: str = "reference", return_pos: bool = False, status: Optional[torch.Tensor] = None):
    """Farthest point sampling per cloud (reference: csrc/__init__.py:566-597,
    fps_kernel.cu:160-209). Returns int64 global indices, cloud b's picks at offset
    sum_{c<b} k_c; a cloud with k > n yields n indices followed by -1.

    One device->host copy of ``ptr``/``k_per_batch`` sizes the output (the reference
    also synchronises once, fps_kernel.cu:183); pass CPU tensors to avoid it. With
    ``return_pos`` also returns the picked coordinates [total, 3] (written by the kernel).

    ``status``: an int32 CUDA tensor of one element, zeroed by the caller. The large-cloud
    kernel's exchange waits are bounded; if one gives up (never observed), that cloud's
    remaining picks are -2 (coordinates 0) and ``status`` receives GDL_ERR_TIMEOUT (6). The
    call does not read it back (no extra synchronisation); check it when convenient.
    """
    dev = nat.require_cuda(pos, what="fps_cuda")
    pos = pos.contiguous().float()
    host = torch.cat([ptr.reshape(-1).to(torch.int64), k_per_batch.reshape(-1).to(torch.int64)]).cpu()
    B = ptr.numel() - 1
    ptr_h, k_h = host[: B + 1], host[B + 1:]
    total = int(k_h.clamp(min=0).sum()) if B > 0 else 0
    if total <= 0 or pos.shape[0] == 0:
        e = torch.empty(0, dtype=torch.int64, device=dev)
        return (e, torch.empty(0, 3, device=dev)) if return_pos else e
    max_n = int((ptr_h[1:] - ptr_h[:-1]).max())
    ptr_d = nat.to_device(ptr_h, dev) if not ptr.is_cuda else ptr.to(torch.int64).contiguous()
    k_d = nat.to_device(k_h, dev) if not k_per_batch.is_cuda else k_per_batch.to(torch.int64).contiguous()
    out = torch.empty(total, dtype=torch.int64, device=dev)
    opos = torch.empty(total, 3, dtype=torch.float32, device=dev) if return_pos else None
    L = nat.load()
    ws = nat.workspace(L.gdl_fps_workspace_size(pos.shape[0], B, max_n), dev)
    if status is None:
        nat.check(L.gdl_fps(pos.data_ptr(), ptr_d.data_ptr(), k_d.data_ptr(), B, pos.shape[0], max_n,
                            nat.TIE[tie_break], out.data_ptr(), nat.ptr(opos), ws.data_ptr(), ws.numel(),
                            nat.stream(dev)), "gdl_fps")
    else:
        if not (status.is_cuda and status.dtype == torch.int32 and status.numel() >= 1):
            raise nat.GdlError("fps_cuda: status must be an int32 CUDA tensor of at least one element")
        nat.check(L.gdl_fps_ex(pos.data_ptr(), ptr_d.data_ptr(), k_d.data_ptr(), B, pos.shape[0], max_n,
                               nat.TIE[tie_break], out.data_ptr(), nat.ptr(opos), ws.data_ptr(), ws.numel(),
                               status.data_ptr(), 0, -1, -1, nat.stream(dev)), "gdl_fps_ex")
    return (out, opos) if return_pos else out


# --------------------------------------------------------------------------- KNN
def knn_cuda(query: torch.Tensor, source: torch.Tensor, ptr_q: torch.Tensor, ptr_s: torch.Tensor,
             k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Batched brute-force KNN (reference: csrc/__init__.py:376-410, knn_kernel.cu:200-291).

    Returns (indices [N_q, k] int64 global, -1 padded; dists [N_q, k] f32 squared, 1e30
    padded), ordered exactly like the reference kernel (at most 64 real neighbours).
    No host synchronisation.
    """
    dev = nat.require_cuda(query, source, what="knn_cuda")
    query = query.contiguous().float()
    source = source.contiguous().float()
    ptr_s_host = ptr_s.to(torch.int64) if not ptr_s.is_cuda else None
    ptr_q = nat.to_device(ptr_q, dev, torch.int64)
    ptr_s = nat.to_device(ptr_s, dev, torch.int64)
    K = int(k)
    nq = query.shape[0]
    if nq == 0 or K <= 0:
        return (torch.empty(0, K, dtype=torch.int64, device=dev), torch.empty(0, K, dtype=torch.float32, device=dev))
    B = ptr_q.numel() - 1
    if ptr_s.numel() != ptr_q.numel():
        raise nat.GdlError("knn_cuda: ptr_q and ptr_s must have the same length (B+1)")
    idx = torch.empty(nq, K, dtype=torch.int64, device=dev)
    dist = torch.empty(nq, K, dtype=torch.float32, device=dev)
    L = nat.load()
    # largest cloud: exact when ptr_s lives on the host, else the mean (it only sizes the
    # split of each cloud's scan over CTAs; any value is correct)
    if ptr_s_host is not None and B > 0:
        max_src = int((ptr_s_host[1:] - ptr_s_host[:-1]).max())
    else:
        max_src = -(-source.shape[0] // max(B, 1))
    ws = nat.workspace(L.gdl_knn_workspace_size(nq, B, K, max_src), dev)
    nat.check(L.gdl_knn(query.data_ptr(), source.data_ptr() if source.numel() else None, ptr_q.data_ptr(),
                        ptr_s.data_ptr(), B, nq, K, max_src, idx.data_ptr(), dist.data_ptr(), ws.data_ptr(),
                        ws.numel(), nat.stream(dev)), "gdl_knn")
    return idx, dist


def knn_self_cuda(points: torch.Tensor, ptr: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Self-KNN, self included (reference: csrc/__init__.py:413-432)."""
    return knn_cuda(points, points, ptr, ptr, k)


# --------------------------------------------------------------------------- radius graph
def _radius_call(x, r, ptr, max_num_neighbors, loop, mask, with_dst, max_cloud_points, int32_csr, geom):
    dev = nat.require_cuda(x, what="radius_graph")
    x = x.contiguous().float()
    N = x.shape[0]
    if max_cloud_points is None:
        max_cloud_points = int((ptr[1:] - ptr[:-1]).max()) if (not ptr.is_cuda and ptr.numel() > 1) else 0
    ptr = nat.to_device(ptr, dev, torch.int64)
    B = ptr.numel() - 1
    cap_k = 16 if max_num_neighbors <= 16 else 32 if max_num_neighbors <= 32 else 64
    cap = max(N * cap_k, 1)
    row_ptr = torch.empty(N + 1, dtype=torch.int64, device=dev)
    src = torch.empty(cap, dtype=torch.int64, device=dev)
    dst = torch.empty_like(src) if with_dst else None
    rp32 = torch.empty(N + 1, dtype=torch.int32, device=dev) if int32_csr else None
    src32 = torch.empty(cap, dtype=torch.int32, device=dev) if int32_csr else None
    m = None
    if mask is not None and mask.numel() > 0:
        m = nat.to_device(mask, dev)
        m = m.view(torch.uint8) if m.dtype == torch.bool else m.to(torch.uint8)
    L = nat.load()
    ws = nat.workspace(L.gdl_radius_graph_workspace_size(N, B, int(max_num_neighbors)), dev)
    args = (x.data_ptr() if N else None, ptr.data_ptr(), B, N, int(max_cloud_points), float(r), int(max_num_neighbors),
            int(bool(loop)), nat.ptr(m), row_ptr.data_ptr(), src.data_ptr(), nat.ptr(dst), nat.ptr(rp32),
            nat.ptr(src32))
    if geom is None:
        nat.check(L.gdl_radius_graph(*args, ws.data_ptr(), ws.numel(), nat.stream(dev)), "gdl_radius_graph")
    else:
        nat.check(L.gdl_radius_graph_geometry(*args, geom(cap, dev), ws.data_ptr(), ws.numel(), nat.stream(dev)),
                  "gdl_radius_graph_geometry")
    return row_ptr, src, dst, rp32, src32, ptr


def radius_graph_csr(x: torch.Tensor, r: float, ptr: torch.Tensor, *, max_num_neighbors: int = 32,
                     loop: bool = False, mask: Optional[torch.Tensor] = None, with_dst: bool = True,
                     max_cloud_points: Optional[int] = None, int32_csr: bool = False):
    """Radius graph of packed clouds as a destination CSR, without a host sync.

    Returns (row_ptr [N+1] int64, src [cap] int64, dst [cap] int64 or None); the first
    row_ptr[N] entries of src/dst are the edges (row=src=neighbour, col=dst=query),
    grouped by destination with ascending sources. cap = N * bucket(max_num_neighbors).
    ``max_cloud_points`` (taken from ``ptr`` when it is a CPU tensor) lets clouds of up to
    4096 points use the fused one-CTA-per-cloud kernels. ``int32_csr`` appends
    (row_ptr32 [N+1], src32 [cap]) int32 copies, the layout segment_reduce_cuda consumes.
    """
    row_ptr, src, dst, rp32, src32, _ = _radius_call(x, r, ptr, max_num_neighbors, loop, mask, with_dst,
                                                     max_cloud_points, int32_csr, None)
    return (row_ptr, src, dst, rp32, src32) if int32_csr else (row_ptr, src, dst)


class _GeomOut:
    """Per-edge output buffers of the geometry entry points (gdl_edge_geometry)."""

    def __init__(self, max_l: Optional[int], with_diff: bool, with_dist: bool = True, with_dir: bool = True):
        if max_l is not None and max_l not in (0, 1, 2):
            raise ValueError(f"max_l must be 0, 1 or 2, got {max_l}")
        self.max_l, self.with_diff, self.with_dist, self.with_dir = max_l, with_diff, with_dist, with_dir
        self.diff = self.dist = self.direction = self.sph = None
        self._struct = None

    def __call__(self, cap: int, dev):
        f = dict(dtype=torch.float32, device=dev)
        self.diff = torch.empty(cap, 3, **f) if self.with_diff else None
        self.dist = torch.empty(cap, **f) if self.with_dist else None
        self.direction = torch.empty(cap, 3, **f) if self.with_dir else None
        self.sph = torch.empty(cap, (self.max_l + 1) ** 2, **f) if self.max_l is not None else None
        self._struct = nat.EdgeGeometry(nat.ptr(self.diff), nat.ptr(self.dist), nat.ptr(self.direction),
                                        nat.ptr(self.sph), int(self.max_l or 0))
        return ctypes.byref(self._struct)


def radius_graph_geometry_csr(x: torch.Tensor, r: float, ptr: torch.Tensor, *, max_num_neighbors: int = 32,
                              loop: bool = False, mask: Optional[torch.Tensor] = None, max_l: Optional[int] = 2,
                              with_diff: bool = False, max_cloud_points: Optional[int] = None) -> dict:
    """radius_graph_csr plus each edge's geometry, written by the kernel that emits the edge.

    Returns a dict of device tensors, edge slots [0, row_ptr[N]) valid: ``row_ptr`` [N+1],
    ``src``/``dst`` [cap] int64, ``row_ptr32`` [N+1] / ``src32`` [cap] int32, ``dist`` [cap],
    ``direction`` [cap, 3], ``sph`` [cap, (max_l+1)^2] (None when max_l is None), ``diff``
    [cap, 3] (None unless with_diff), and ``ptr`` (int64 on the device). Values follow
    compute_edge_vectors (x[dst] - x[src]) and spherical_harmonics(normalize=False) of the
    reference (functional/radius_graph.py:338-358, kernels/triton_sph_harm.py:200-240)."""
    g = _GeomOut(max_l, with_diff)
    row_ptr, src, dst, rp32, src32, ptr_d = _radius_call(x, r, ptr, max_num_neighbors, loop, mask, True,
                                                         max_cloud_points, True, g)
    return dict(row_ptr=row_ptr, src=src, dst=dst, row_ptr32=rp32, src32=src32, dist=g.dist,
                direction=g.direction, sph=g.sph, diff=g.diff, ptr=ptr_d)


def radius_csr_finish(row_ptr: torch.Tensor, dst: torch.Tensor, N: int, *, ptr: Optional[torch.Tensor] = None,
                      avg_degree: bool = True):
    """SpatialGraph's CSR fields of a destination-grouped radius graph without a sort:
    (col_sorted [cap] i32, perm [cap] i32, node_start [N] i32, node_end [N] i32, avg_degree [N]
    f32 or None); the first row_ptr[N] slots of col_sorted / perm are valid. ``ptr`` (device
    int64) gives the clouds of the average degree, None one cloud."""
    dev = nat.require_cuda(row_ptr, dst, what="radius_csr_finish")
    cap = dst.numel()
    i32 = dict(dtype=torch.int32, device=dev)
    cs, pm = torch.empty(cap, **i32), torch.empty(cap, **i32)
    ns, ne = torch.empty(N, **i32), torch.empty(N, **i32)
    avg = torch.empty(N, dtype=torch.float32, device=dev) if avg_degree else None
    B = 0 if ptr is None else ptr.numel() - 1
    L = nat.load()
    nat.check(L.gdl_radius_csr_finish(row_ptr.data_ptr(), dst.data_ptr(), int(N), cap, nat.ptr(ptr), B,
                                      nat.ptr(cs) if cap else None, nat.ptr(pm) if cap else None,
                                      nat.ptr(ns) if N else None, nat.ptr(ne) if N else None,
                                      nat.ptr(avg) if N else None, nat.stream(dev)), "gdl_radius_csr_finish")
    return cs, pm, ns, ne, avg


def edge_geometry_cuda(x: torch.Tensor, row: torch.Tensor, col: torch.Tensor, *, max_l: Optional[int] = None,
                       with_diff: bool = True, with_dist: bool = True, with_dir: bool = True):
    """(diff, dist, direction, sph) of COO edges row=src -> col=dst (compute_edge_vectors +
    spherical_harmonics(normalize=False) of the reference); entries not requested are None."""
    dev = nat.require_cuda(x, row, col, what="edge_geometry_cuda")
    x = x.contiguous().float()
    row = row.to(torch.int64).contiguous()
    col = col.to(torch.int64).contiguous()
    E = row.numel()
    g = _GeomOut(max_l, with_diff, with_dist, with_dir)
    st = g(E, dev)
    nat.check(nat.load().gdl_edge_geometry_coo(x.data_ptr() if x.numel() else None, x.shape[0],
                                               row.data_ptr() if E else None, col.data_ptr() if E else None, E, st,
                                               nat.stream(dev)), "gdl_edge_geometry_coo")
    return g.diff, g.dist, g.direction, g.sph


def cloud_avg_degree_cuda(node_start: torch.Tensor, node_end: torch.Tensor, *, batch: Optional[torch.Tensor] = None,
                          ptr: Optional[torch.Tensor] = None, num_clouds: Optional[int] = None) -> torch.Tensor:
    """avg_degree [N] of SpatialGraph (nn/modules/spatial_graph.py:131-153): the average degree
    of each node's cloud (clouds from ``batch``, else ``ptr``, else one), clamped at 1."""
    dev = nat.require_cuda(node_start, node_end, what="cloud_avg_degree_cuda")
    N = node_start.numel()
    out = torch.empty(N, dtype=torch.float32, device=dev)
    b = p = None
    B = 0
    if batch is not None:
        b = nat.to_device(batch, dev, torch.int64)
        B = int(num_clouds) if num_clouds is not None else (int(b.max().item()) + 1 if N else 1)
    elif ptr is not None:
        p = nat.to_device(ptr, dev, torch.int64)
        B = p.numel() - 1
    L = nat.load()
    ws = nat.workspace(L.gdl_cloud_avg_degree_workspace_size(max(B, 1)), dev)
    nat.check(L.gdl_cloud_avg_degree(node_start.contiguous().data_ptr() if N else None,
                                     node_end.contiguous().data_ptr() if N else None, N, nat.ptr(b), nat.ptr(p), B,
                                     out.data_ptr() if N else None, ws.data_ptr(), ws.numel(), nat.stream(dev)),
              "gdl_cloud_avg_degree")
    return out


def radius_graph_cuda(x: torch.Tensor, r: float, *, max_num_neighbors: int = 32, loop: bool = False,
                      mask: Optional[torch.Tensor] = None, batch_size: Optional[int] = None,
                      points_per_batch: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(row, col) int64 edges, global indices (reference: csrc/__init__.py:130-186,
    radius_graph_kernel.cu:253-467). Equal-size batches via batch_size/points_per_batch
    like the reference; one device->host read of the edge count."""
    dev = nat.require_cuda(x, what="radius_graph_cuda")
    N = x.shape[0]
    if batch_size is not None and batch_size > 1:
        assert points_per_batch is not None, "points_per_batch required when batch_size > 1"
        ptr = torch.arange(0, batch_size + 1, dtype=torch.int64) * int(points_per_batch)
    else:
        ptr = torch.tensor([0, N], dtype=torch.int64)
    row_ptr, src, dst = radius_graph_csr(x, r, ptr, max_num_neighbors=max_num_neighbors, loop=loop, mask=mask)
    E = int(row_ptr[N].item())
    return src[:E], dst[:E]


# --------------------------------------------------------------------------- segment reduce
def sort_and_build_csr_cuda(col: torch.Tensor, N: int):
    """Stable sort by destination + CSR offsets (reference: csrc/__init__.py:261-277,
    segment_reduce_kernel.cu:100-169). Returns (col_sorted, perm, node_start, node_end) int32."""
    dev = nat.require_cuda(col, what="sort_and_build_csr_cuda")
    col = col.to(torch.int64).contiguous()
    E = col.numel()
    cs = torch.empty(E, dtype=torch.int32, device=dev)
    pm = torch.empty(E, dtype=torch.int32, device=dev)
    ns = torch.empty(N, dtype=torch.int32, device=dev)
    ne = torch.empty(N, dtype=torch.int32, device=dev)
    L = nat.load()
    ws = nat.workspace(L.gdl_sort_and_build_csr_workspace_size(E, N), dev)
    nat.check(L.gdl_sort_and_build_csr(col.data_ptr() if E else None, E, int(N), cs.data_ptr() if E else None,
                                       pm.data_ptr() if E else None, ns.data_ptr() if N else None,
                                       ne.data_ptr() if N else None, ws.data_ptr(), ws.numel(), nat.stream(dev)),
              "gdl_sort_and_build_csr")
    return cs, pm, ns, ne


def segment_reduce_cuda(msg: torch.Tensor, perm: Optional[torch.Tensor], node_start: torch.Tensor,
                        node_end: torch.Tensor, N: int, reduce: str = "sum", *, with_arg: bool = False):
    """out [N, C] float32 = reduce over slots [node_start[n], node_end[n]) of msg[perm[slot]].

    msg float32 or bfloat16 (fp32 accumulation). perm None = identity. For reduce="max"
    and with_arg, also returns arg [N, C] int32 (slot of the unique maximum, -1 if tied).
    """
    dev = nat.require_cuda(msg, node_start, node_end, what="segment_reduce")
    if msg.dtype not in nat.DTYPE:
        msg = msg.float()
    msg = msg.contiguous()
    if msg.dim() == 1:
        msg = msg.unsqueeze(1)
    E, C = msg.shape
    out = torch.empty(N, C, dtype=torch.float32, device=dev)
    arg = torch.empty(N, C, dtype=torch.int32, device=dev) if (reduce == "max" and with_arg) else None
    ns = node_start.to(torch.int32).contiguous()
    ne = node_end.to(torch.int32).contiguous()
    pm = None if perm is None else perm.to(torch.int32).contiguous()
    L = nat.load()
    ws = nat.stream_workspace(L.gdl_segment_reduce_workspace_size(E, N), dev)
    if N > 0 and C > 0:
        nat.check(L.gdl_segment_reduce(msg.data_ptr() if E else None, nat.DTYPE[msg.dtype], E, C, nat.ptr(pm),
                                       ns.data_ptr(), ne.data_ptr(), int(N), nat.REDUCE[reduce], out.data_ptr(),
                                       nat.ptr(arg), ws.data_ptr(), ws.numel(), nat.stream(dev)),
                  "gdl_segment_reduce")
    return (out, arg) if with_arg else out


def segment_reduce_sum_cuda(msg: torch.Tensor, perm: torch.Tensor, node_start: torch.Tensor,
                            node_end: torch.Tensor, N: int) -> torch.Tensor:
    """Deterministic segment sum (reference: csrc/__init__.py:280-302)."""
    return segment_reduce_cuda(msg, perm, node_start, node_end, N, "sum")


def segment_reduce_backward_cuda(grad_out: torch.Tensor, msg: torch.Tensor, out: Optional[torch.Tensor],
                                 arg: Optional[torch.Tensor], perm: Optional[torch.Tensor], node_start: torch.Tensor,
                                 node_end: torch.Tensor, N: int, reduce: str = "sum",
                                 grad_msg: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gradient w.r.t. msg (msg's shape and dtype): grad_msg[perm[j]] for every slot j of every
    segment (the reference's gather + un-permute, functional/segment_reduce.py:142-158).

    Rows that no slot references are zero (or keep ``grad_msg``'s contents when it is given;
    a CSR from sort_and_build_csr references every row exactly once).
    """
    dev = nat.require_cuda(grad_out, node_start, node_end, what="segment_reduce_backward")
    E = msg.shape[0]
    C = grad_out.shape[1] if grad_out.dim() == 2 else 1
    if grad_msg is None:
        grad_msg = torch.zeros(msg.shape, dtype=msg.dtype, device=dev)
    if E == 0 or C == 0 or N == 0:
        return grad_msg
    go = grad_out.float().contiguous()
    m = msg.contiguous()
    pm = None if perm is None else perm.to(torch.int32).contiguous()
    ns = node_start.to(torch.int32).contiguous()
    ne = node_end.to(torch.int32).contiguous()
    L = nat.load()
    ws = nat.workspace(L.gdl_segment_reduce_workspace_size(E, N), dev)
    nat.check(L.gdl_segment_reduce_backward(go.data_ptr(), m.data_ptr(), nat.DTYPE[msg.dtype], nat.ptr(out),
                                            nat.ptr(arg), E, C, nat.ptr(pm), ns.data_ptr(), ne.data_ptr(), int(N),
                                            nat.REDUCE[reduce], grad_msg.data_ptr(), ws.data_ptr(), ws.numel(),
                                            nat.stream(dev)), "gdl_segment_reduce_backward")
    return grad_msg


def gather_rows(src: torch.Tensor, idx: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[i] = src[idx[i]] for a 2-D tensor of any dtype (rows of a multiple of 4 bytes);
    indices outside [0, src.shape[0]) give zero rows. The msg = feats[knn_idx] step of the
    reference's pooling layer (nn/modules/equivariant_pool.py:277-300)."""
    dev = nat.require_cuda(src, idx, what="gather_rows")
    src = src.contiguous()
    idx = idx.reshape(-1).to(torch.int64).contiguous()
    shape = (idx.numel(),) + tuple(src.shape[1:])
    if out is None:
        out = torch.empty(shape, dtype=src.dtype, device=dev)
    elif tuple(out.shape) != shape or out.dtype != src.dtype or not out.is_contiguous():
        raise nat.GdlError("gather_rows: out must be a contiguous tensor of shape [len(idx), *src.shape[1:]]")
    row_bytes = src[0].numel() * src.element_size() if src.shape[0] else int(np.prod(shape[1:])) * src.element_size()
    nat.check(nat.load().gdl_gather_rows(src.data_ptr() if src.numel() else None, src.shape[0], row_bytes,
                                         idx.data_ptr(), idx.numel(), out.data_ptr(), nat.stream(dev)),
              "gdl_gather_rows")
    return out


# --------------------------------------------------------------------------- KNN aggregation
def _rows(t: torch.Tensor) -> torch.Tensor:
    """[n, ...] float32 contiguous viewed as [n, dim]."""
    t = t.contiguous()
    if t.dtype != torch.float32:
        t = t.float()
    return t.reshape(t.shape[0], -1)


def knn_idw_weights_cuda(idx: torch.Tensor, dist: torch.Tensor) -> torch.Tensor:
    """Inverse-distance weights of EquivariantInterpolate (nn/modules/equivariant_interp.py:92-96)
    from KNN output: w = inv / max(sum inv, 1e-8), inv = 1/sqrt(max(dist, 1e-4)), 0 for padding."""
    dev = nat.require_cuda(idx, dist, what="knn_idw_weights_cuda")
    idx = idx.to(torch.int64).contiguous()
    dist = dist.contiguous().float()
    n, k = idx.shape
    w = torch.empty(n, k, dtype=torch.float32, device=dev)
    nat.check(nat.load().gdl_knn_idw_weights(nat.ptr(idx) if w.numel() else None, nat.ptr(dist) if w.numel() else None,
                                             n, k, nat.ptr(w) if w.numel() else None, nat.stream(dev)),
              "gdl_knn_idw_weights")
    return w


def knn_weighted_sum_cuda(src: torch.Tensor, idx: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """out[q] = sum_j weight[q, j] * src[idx[q, j]] over valid neighbours, shape [n_query, *src.shape[1:]]
    (one pass, no [n_query, k, ...] gather)."""
    dev = nat.require_cuda(src, idx, weight, what="knn_weighted_sum_cuda")
    s2 = _rows(src)
    idx = idx.to(torch.int64).contiguous()
    weight = weight.contiguous().float()
    n, k = idx.shape
    out = torch.empty(n, *src.shape[1:], dtype=torch.float32, device=dev)
    dim = s2.shape[1]
    nat.check(nat.load().gdl_knn_weighted_sum(nat.ptr(s2) if s2.numel() else None, s2.shape[0], dim,
                                              nat.ptr(idx) if idx.numel() else None,
                                              nat.ptr(weight) if weight.numel() else None, n, k,
                                              nat.ptr(out) if out.numel() else None, nat.stream(dev)),
              "gdl_knn_weighted_sum")
    return out


def knn_weighted_sum_backward_cuda(grad_outs, idx: torch.Tensor, weight: torch.Tensor, src_shapes):
    """Gradients w.r.t. the source tables of knn_weighted_sum_cuda: one transposed (sorted) pair
    list shared by all tables, deterministic fp32 folds. ``src_shapes``: shapes of the sources."""
    dev = nat.require_cuda(idx, weight, what="knn_weighted_sum_backward_cuda")
    idx = idx.to(torch.int64).contiguous()
    weight = weight.contiguous().float()
    n, k = idx.shape
    n_src = int(src_shapes[0][0]) if src_shapes else 0
    gos = [_rows(g) for g in grad_outs]
    outs = [torch.empty(*shp, dtype=torch.float32, device=dev) for shp in src_shapes]
    o2 = [o.reshape(o.shape[0], -1) for o in outs]
    T = len(gos)
    gop = (ctypes.c_void_p * max(T, 1))(*[g.data_ptr() for g in gos])
    osp = (ctypes.c_void_p * max(T, 1))(*[o.data_ptr() for o in o2])
    dims = (ctypes.c_int64 * max(T, 1))(*[o.shape[1] for o in o2])
    L = nat.load()
    ws = nat.workspace(L.gdl_knn_weighted_sum_backward_workspace_size(n, k, n_src), dev)
    nat.check(L.gdl_knn_weighted_sum_backward(gop, osp, dims, T, nat.ptr(idx) if idx.numel() else None,
                                              nat.ptr(weight) if weight.numel() else None, n, k, n_src,
                                              ws.data_ptr(), ws.numel(), nat.stream(dev)),
              "gdl_knn_weighted_sum_backward")
    return outs


def knn_weighted_sum_weight_grad_cuda(grad_outs, srcs, idx: torch.Tensor) -> torch.Tensor:
    """grad_weight[q, j] = sum over tables of sum_c grad_out[q, c] * src[idx[q, j], c]."""
    dev = nat.require_cuda(idx, what="knn_weighted_sum_weight_grad_cuda")
    idx = idx.to(torch.int64).contiguous()
    n, k = idx.shape
    gw = torch.zeros(n, k, dtype=torch.float32, device=dev)
    L = nat.load()
    for t, (g, s) in enumerate(zip(grad_outs, srcs)):
        g2, s2 = _rows(g), _rows(s)
        nat.check(L.gdl_knn_weighted_sum_weight_grad(nat.ptr(g2) if g2.numel() else None,
                                                     nat.ptr(s2) if s2.numel() else None, s2.shape[0], s2.shape[1],
                                                     nat.ptr(idx) if idx.numel() else None, n, k, int(t > 0),
                                                     nat.ptr(gw) if gw.numel() else None, nat.stream(dev)),
                  "gdl_knn_weighted_sum_weight_grad")
    return gw


# --------------------------------------------------------------------------- weight gradients
def _row_matrix(t: torch.Tensor) -> torch.Tensor:
    """[rows, ...] float32 as a [rows, width] matrix with unit inner stride (a view when possible)."""
    if t.dtype != torch.float32:
        t = t.float()
    t = t.reshape(t.shape[0], math.prod(t.shape[1:]))
    if t.shape[1] > 0 and (t.stride(1) != 1 or t.stride(0) < t.shape[1]):
        t = t.contiguous()
    return t


def weight_grad_cuda(grad_out: torch.Tensor, inp: torch.Tensor, sub: int = 1, col_sum: bool = False):
    """Weight (and bias) gradient of a per-row linear map: grad_out [rows, M, sub] (or [rows, M] for
    sub 1), inp [rows, N, sub] -> (C [M, N] = sum_{r, j} grad_out[r, :, j]^T inp[r, :, j], column sums
    of grad_out [M] or None), deterministic (gdl_weight_grad)."""
    dev = nat.require_cuda(grad_out, inp, what="weight_grad_cuda")
    A, B = _row_matrix(grad_out), _row_matrix(inp)
    rows = A.shape[0]
    M, N = A.shape[1] // sub, B.shape[1] // sub
    C = torch.empty(M, N, dtype=torch.float32, device=dev)
    cs = torch.empty(M, dtype=torch.float32, device=dev) if col_sum else None
    L = nat.load()
    ws = nat.workspace(L.gdl_weight_grad_workspace_size(rows, M, N, sub), dev)
    nat.check(L.gdl_weight_grad(nat.ptr(A) if A.numel() else None, A.stride(0) if A.numel() else M * sub,
                                nat.ptr(B) if B.numel() else None, B.stride(0) if B.numel() else N * sub, rows, M, N,
                                sub, nat.ptr(C) if C.numel() else None, nat.ptr(cs), ws.data_ptr(), ws.numel(),
                                nat.stream(dev)), "gdl_weight_grad")
    return C, cs


# --------------------------------------------------------------------------- hybrid graph
def hybrid_graph_cuda(radius_row_ptr: torch.Tensor, radius_src: torch.Tensor, knn_idx: Optional[torch.Tensor],
                      N: int, max_num_neighbors: int, knn_fallback_k: int, x: Optional[torch.Tensor] = None,
                      max_l: Optional[int] = None) -> dict:
    """Radius edges + symmetric KNN fallback edges for nodes with fewer than knn_fallback_k
    radius in-edges, deduplicated in (row, col) order (multi_scale_se3_net.py:126-219), with
    the CSR of sort_and_build_csr(col) and, when ``x`` is given, each edge's distance and
    direction (+ harmonics up to ``max_l``). Returns device tensors: ``row_ptr`` [N+1] (E at
    [N]), ``row`` / ``col`` [cap] int64, ``col_sorted`` / ``perm`` / ``src_sorted`` [cap] int32,
    ``node_start`` / ``node_end`` [N] int32, ``dist`` / ``direction`` / ``sph`` (or None); the
    first E slots of the edge arrays are valid."""
    dev = nat.require_cuda(radius_row_ptr, radius_src, what="hybrid_graph_cuda")
    L = nat.load()
    kf = int(knn_fallback_k)
    cap = max(int(L.gdl_hybrid_graph_capacity(N, int(max_num_neighbors), kf)), 1)
    knn_idx = None if (knn_idx is None or kf == 0) else knn_idx.to(torch.int64).contiguous()
    i64 = dict(dtype=torch.int64, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    out = dict(row_ptr=torch.empty(N + 1, **i64), row=torch.empty(cap, **i64), col=torch.empty(cap, **i64),
               col_sorted=torch.empty(cap, **i32), perm=torch.empty(cap, **i32), src_sorted=torch.empty(cap, **i32),
               node_start=torch.empty(max(N, 1), **i32), node_end=torch.empty(max(N, 1), **i32))
    g = None
    if x is not None:
        x = x.contiguous().float()
        g = _GeomOut(max_l, False)
        gp = g(cap, dev)
    ws = nat.workspace(L.gdl_hybrid_graph_workspace_size(N, int(max_num_neighbors), kf), dev)
    nat.check(L.gdl_hybrid_graph(nat.ptr(x) if (x is not None and N) else None, radius_row_ptr.data_ptr(),
                                 radius_src.data_ptr(), nat.ptr(knn_idx), N, int(max_num_neighbors), kf,
                                 out["row_ptr"].data_ptr(), out["row"].data_ptr(), out["col"].data_ptr(),
                                 out["col_sorted"].data_ptr(), out["perm"].data_ptr(), out["src_sorted"].data_ptr(),
                                 out["node_start"].data_ptr(), out["node_end"].data_ptr(), gp if g else None,
                                 ws.data_ptr(), ws.numel(), nat.stream(dev)), "gdl_hybrid_graph")
    out["node_start"], out["node_end"] = out["node_start"][:N], out["node_end"][:N]
    out["dist"] = g.dist if g else None
    out["direction"] = g.direction if g else None
    out["sph"] = g.sph if g else None
    return out
