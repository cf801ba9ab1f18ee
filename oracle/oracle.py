"""numpy front end of the CPU parity checker (``oracle/gdl_oracle.c``).

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` leg may import this module; the product
(``gdl_b200``) never does. Each function restates one reference operator; the cited
reference lines are in the C source.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libgdl_oracle.so"

# distance rounding modes (see gdl_oracle.c)
DIST_TORCH = 0
DIST_FMA_ZYX = 1
DIST_FMA_ZXY = 2
DIST_FMA_Z_SUM = 3
DIST_NOFMA_FTZ = 4
DIST_FMA_XYZ = 5
DIST_MODES = {
    "torch": DIST_TORCH,
    "fma_zyx": DIST_FMA_ZYX,
    "fma_zxy": DIST_FMA_ZXY,
    "fma_z_sum": DIST_FMA_Z_SUM,
    "nofma_ftz": DIST_NOFMA_FTZ,
    "fma_xyz": DIST_FMA_XYZ,
}
# Rounding of the reference CUDA kernels' `dx*dx + dy*dy + dz*dz` under nvcc -O3
# --use_fast_math for sm_100a: fma(dz, dz, fma(dx, dx, dy*dy)) with flush-to-zero. Pinned on
# a B200: of the candidate modes only this one reproduces, bit for bit, every distance the
# reference KNN kernel returned (tests/test_gpu_ref_pin.py::test_distance_rounding_pinned).
DIST_CUDA = DIST_FMA_ZXY

TIE_REFERENCE = 0
TIE_LOWEST_INDEX = 1
REDUCE = {"sum": 0, "mean": 1, "max": 2}

_lib = None


def build() -> Path:
    """Compile the oracle library with the committed Makefile (gcc, pthreads)."""
    env = dict(os.environ)
    env.setdefault("CC", "gcc")
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True, env=env)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        i64 = ctypes.c_int64
        i32 = ctypes.c_int
        L.gdl_oracle_fps.argtypes = [P, P, P, i32, i32, i32, P]
        L.gdl_oracle_knn.argtypes = [P, P, P, P, i32, i64, i32, i32, P, P]
        L.gdl_oracle_radius_graph.argtypes = [P, P, i32, ctypes.c_double, i32, i32, P, i32, P, P]
        L.gdl_oracle_radius_graph.restype = i64
        L.gdl_oracle_sort_and_build_csr.argtypes = [P, i64, i64, P, P, P, P]
        L.gdl_oracle_segment_reduce.argtypes = [P, i32, P, P, P, i64, i64, i32, P]
        L.gdl_oracle_segment_reduce_backward.argtypes = [P, P, i32, P, P, P, P, i64, i64, i64, i32, P]
        L.gdl_oracle_fps_priority.argtypes = [i64, i32]
        L.gdl_oracle_fps_priority.restype = ctypes.c_uint32
        L.gdl_oracle_num_threads.restype = i32
        L.gdl_oracle_set_num_threads.argtypes = [i32]
        L.gdl_oracle_radius_grid.argtypes = [P, i64, ctypes.c_float, P, P]
        L.gdl_oracle_edge_geometry.argtypes = [P, i64, P, P, i64, P, P, P, P, i32]
        L.gdl_oracle_cloud_avg_degree.argtypes = [P, P, i64, P, P, i32, P]
        L.gdl_oracle_knn_idw_weights.argtypes = [P, P, i64, i32, P]
        L.gdl_oracle_hybrid_graph.argtypes = [P, P, P, i64, i32, P, P]
        L.gdl_oracle_hybrid_graph.restype = i64
        L.gdl_oracle_knn_weighted_sum.argtypes = [P, i64, i64, P, P, i64, i32, P]
        L.gdl_oracle_knn_weighted_sum_backward.argtypes = [P, i64, P, P, i64, i32, i64, P]
        L.gdl_oracle_knn_weighted_sum_weight_grad.argtypes = [P, P, i64, i64, P, i64, i32, i32, P]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a), dtype=dtype)


def set_num_threads(n: int) -> None:
    lib().gdl_oracle_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().gdl_oracle_num_threads())


def fps(pos, ptr, k_per_cloud, tie=TIE_REFERENCE, dist=DIST_CUDA) -> np.ndarray:
    """Farthest point sampling; global int64 indices laid out by cumsum(k)."""
    pos = _c(pos, np.float32).reshape(-1, 3)
    ptr = _c(ptr, np.int64)
    k = _c(k_per_cloud, np.int64)
    B = ptr.shape[0] - 1
    out = np.full(int(np.clip(k, 0, None).sum()), -1, dtype=np.int64)
    lib().gdl_oracle_fps(_p(pos), _p(ptr), _p(k), B, tie, dist, _p(out))
    return out


def fps_priority(i: int, tie=TIE_REFERENCE) -> int:
    return int(lib().gdl_oracle_fps_priority(int(i), tie))


def knn(query, source, ptr_q, ptr_s, k: int, dist=DIST_CUDA):
    """Brute-force KNN with the reference MinK semantics -> (idx int64, dist f32)."""
    query = _c(query, np.float32).reshape(-1, 3)
    source = _c(source, np.float32).reshape(-1, 3)
    ptr_q = _c(ptr_q, np.int64)
    ptr_s = _c(ptr_s, np.int64)
    nq = query.shape[0]
    kk = max(int(k), 0)
    idx = np.full((nq, kk), -1, dtype=np.int64)
    dd = np.full((nq, kk), 1e30, dtype=np.float32)
    lib().gdl_oracle_knn(_p(query), _p(source), _p(ptr_q), _p(ptr_s), ptr_q.shape[0] - 1, nq, kk, dist,
                         _p(idx), _p(dd))
    return idx, dd


def radius_graph(x, ptr, r: float, max_num_neighbors: int = 32, loop: bool = False, mask=None,
                 dist=DIST_CUDA):
    """Radius graph -> (row_ptr [N+1], src [E]) CSR over destinations, sources ascending."""
    x = _c(x, np.float32).reshape(-1, 3)
    ptr = _c(ptr, np.int64)
    N = int(ptr[-1])
    cap = 16 if max_num_neighbors <= 16 else 32 if max_num_neighbors <= 32 else 64
    row_ptr = np.zeros(N + 1, dtype=np.int64)
    src = np.zeros(max(N * cap, 1), dtype=np.int64)
    m = None if mask is None else _c(mask, np.uint8)
    E = lib().gdl_oracle_radius_graph(_p(x), _p(ptr), ptr.shape[0] - 1, float(r), int(max_num_neighbors),
                                      int(bool(loop)), None if m is None else _p(m), dist, _p(row_ptr), _p(src))
    return row_ptr, src[:E].copy()


def radius_grid(x, r: float):
    """(mins[3] f32, res[3] i32) of the reference's per-cloud cell grid."""
    x = _c(x, np.float32).reshape(-1, 3)
    mins = np.zeros(3, np.float32)
    res = np.zeros(3, np.int32)
    inv = np.float32(1.0) / np.float32(r)
    lib().gdl_oracle_radius_grid(_p(x), x.shape[0], ctypes.c_float(inv), _p(mins), _p(res))
    return mins, res


def csr_to_coo(row_ptr, src):
    """(row=src, col=dst) int64 edge lists of a destination CSR."""
    deg = np.diff(row_ptr)
    col = np.repeat(np.arange(len(deg), dtype=np.int64), deg)
    return np.asarray(src, np.int64), col


def sort_and_build_csr(col, N: int):
    col = _c(col, np.int64)
    E = col.shape[0]
    cs = np.zeros(E, np.int32)
    pm = np.zeros(E, np.int32)
    ns = np.zeros(N, np.int32)
    ne = np.zeros(N, np.int32)
    rc = lib().gdl_oracle_sort_and_build_csr(_p(col), E, N, _p(cs), _p(pm), _p(ns), _p(ne))
    if rc != 0:
        raise ValueError("sort_and_build_csr: destination index out of range")
    return cs, pm, ns, ne


def _msg_args(msg):
    msg = np.ascontiguousarray(msg)
    if msg.dtype == np.float32:
        return msg, 0
    if msg.dtype == np.uint16:  # raw bfloat16 bits
        return msg, 1
    raise TypeError(f"msg must be float32 or bfloat16 bits (uint16), got {msg.dtype}")


def segment_reduce(msg, perm, node_start, node_end, N: int, reduce: str = "sum") -> np.ndarray:
    msg, dt = _msg_args(msg)
    C = msg.shape[1] if msg.ndim == 2 else 1
    out = np.zeros((N, C), np.float32)
    pm = None if perm is None else _c(perm, np.int32)
    ns = _c(node_start, np.int32)
    ne = _c(node_end, np.int32)
    lib().gdl_oracle_segment_reduce(_p(msg), dt, None if pm is None else _p(pm), _p(ns), _p(ne), N, C,
                                    REDUCE[reduce], _p(out))
    return out


def segment_reduce_backward(grad_out, msg, out, perm, node_start, node_end, N: int, reduce: str = "sum"):
    msg, dt = _msg_args(msg)
    E = msg.shape[0]
    C = msg.shape[1] if msg.ndim == 2 else 1
    go = _c(grad_out, np.float32)
    o = _c(out, np.float32)
    gm = np.zeros((E, C), np.uint16 if dt == 1 else np.float32)
    pm = None if perm is None else _c(perm, np.int32)
    lib().gdl_oracle_segment_reduce_backward(_p(go), _p(msg), dt, _p(o), None if pm is None else _p(pm),
                                             _p(_c(node_start, np.int32)), _p(_c(node_end, np.int32)), N, C, E,
                                             REDUCE[reduce], _p(gm))
    return gm


def edge_geometry(x, row, col, max_l=2):
    """(diff [E,3], dist [E], direction [E,3], sph [E,(max_l+1)^2]) of COO edges row -> col."""
    x = _c(x, np.float32)
    row = _c(row, np.int64)
    col = _c(col, np.int64)
    E = row.shape[0]
    diff = np.zeros((E, 3), np.float32)
    dist = np.zeros(E, np.float32)
    dire = np.zeros((E, 3), np.float32)
    sph = np.zeros((E, (max_l + 1) ** 2), np.float32)
    lib().gdl_oracle_edge_geometry(_p(x), x.shape[0], _p(row), _p(col), E, _p(diff), _p(dist), _p(dire), _p(sph),
                                   int(max_l))
    return diff, dist, dire, sph


def cloud_avg_degree(node_start, node_end, batch=None, ptr=None, num_clouds=None) -> np.ndarray:
    ns = _c(node_start, np.int32)
    ne = _c(node_end, np.int32)
    n = ns.shape[0]
    b = None if batch is None else _c(batch, np.int64)
    p = None if ptr is None else _c(ptr, np.int64)
    if b is not None:
        B = int(num_clouds) if num_clouds is not None else (int(b.max()) + 1 if n else 1)
    elif p is not None:
        B = p.shape[0] - 1
    else:
        B = 1
    out = np.zeros(n, np.float32)
    lib().gdl_oracle_cloud_avg_degree(_p(ns), _p(ne), n, None if b is None else _p(b), None if p is None else _p(p),
                                      B, _p(out))
    return out


def hybrid_graph(row_ptr, src, knn_idx, kf: int):
    """(row, col) int64 of the radius + KNN-fallback union, ordered by (row, col)."""
    rp = _c(row_ptr, np.int64)
    src = _c(src, np.int64)
    n = rp.shape[0] - 1
    knn = _c(knn_idx, np.int64) if kf > 0 else np.zeros((max(n, 1), 1), np.int64)
    cap = int(rp[-1] - rp[0]) + 2 * n * kf + 1
    row = np.zeros(cap, np.int64)
    col = np.zeros(cap, np.int64)
    E = lib().gdl_oracle_hybrid_graph(_p(rp), _p(src) if src.size else None, _p(knn), n, kf, _p(row), _p(col))
    return row[:E], col[:E]


def knn_idw_weights(idx, dist) -> np.ndarray:
    idx = _c(idx, np.int64)
    dist = _c(dist, np.float32)
    n, k = idx.shape
    w = np.zeros((n, k), np.float32)
    lib().gdl_oracle_knn_idw_weights(_p(idx), _p(dist), n, k, _p(w))
    return w


def knn_weighted_sum(src, idx, w) -> np.ndarray:
    src = _c(src, np.float32)
    shape = src.shape
    s2 = src.reshape(shape[0], -1)
    idx = _c(idx, np.int64)
    w = _c(w, np.float32)
    n, k = idx.shape
    out = np.zeros((n, s2.shape[1]), np.float32)
    lib().gdl_oracle_knn_weighted_sum(_p(s2), s2.shape[0], s2.shape[1], _p(idx), _p(w), n, k, _p(out))
    return out.reshape((n,) + shape[1:])


def knn_weighted_sum_backward(grad_out, idx, w, n_src: int) -> np.ndarray:
    g = _c(grad_out, np.float32)
    shape = g.shape
    g2 = g.reshape(shape[0], -1)
    idx = _c(idx, np.int64)
    w = _c(w, np.float32)
    n, k = idx.shape
    out = np.zeros((n_src, g2.shape[1]), np.float32)
    lib().gdl_oracle_knn_weighted_sum_backward(_p(g2), g2.shape[1], _p(idx), _p(w), n, k, n_src, _p(out))
    return out.reshape((n_src,) + shape[1:])


def knn_weighted_sum_weight_grad(grad_outs, srcs, idx) -> np.ndarray:
    idx = _c(idx, np.int64)
    n, k = idx.shape
    gw = np.zeros((n, k), np.float32)
    for t, (g, s) in enumerate(zip(grad_outs, srcs)):
        g2 = _c(g, np.float32).reshape(n, -1)
        s2 = _c(s, np.float32)
        s2 = s2.reshape(s2.shape[0], -1)
        lib().gdl_oracle_knn_weighted_sum_weight_grad(_p(g2), _p(s2), s2.shape[0], s2.shape[1], _p(idx), n, k,
                                                      int(t > 0), _p(gw))
    return gw


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (round to nearest even), as uint16."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)
