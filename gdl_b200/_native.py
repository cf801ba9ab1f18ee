"""ctypes binding of libgdl_b200.so (declared in include/gdl_b200.h).

Torch is used only as plumbing: device buffers from its caching allocator, the current
stream, and tensors in the signatures of the Python API. Every operator raises if the
library is missing or the tensors are not on a CUDA device; there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libgdl_b200.so"

# names and prototypes of every entry point in include/gdl_b200.h
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t


class EdgeGeometry(ctypes.Structure):
    """gdl_edge_geometry: nullable device pointers of the per-edge outputs."""
    _fields_ = [("diff", _P), ("dist", _P), ("direction", _P), ("sph", _P), ("sph_max_l", _I32)]


_PG = ctypes.POINTER(EdgeGeometry)


class Se3Paths(ctypes.Structure):
    """gdl_se3_paths: per-path node projections (nullable), their R columns, output channels."""
    _fields_ = [("p", _P * 9), ("r_col", _I32 * 9), ("ld", _I64 * 9), ("cs", _I64), ("cv", _I64), ("ct2", _I64)]


_PS = ctypes.POINTER(Se3Paths)
PROTOTYPES = {
    "gdl_version": (ctypes.c_int, []),
    "gdl_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "gdl_check_device": (ctypes.c_int, [ctypes.c_int]),
    "gdl_fp32_peak_flops": (_I64, [_I64, _I32, _I32]),
    "gdl_fp32_peak": (ctypes.c_int, [_P, _I64, _I32, _I32, _P]),
    "gdl_fps_workspace_size": (_SZ, [_I64, _I32, _I64]),
    "gdl_fps": (ctypes.c_int, [_P, _P, _P, _I32, _I64, _I64, _I32, _P, _P, _P, _SZ, _P]),
    "gdl_fps_ex": (ctypes.c_int, [_P, _P, _P, _I32, _I64, _I64, _I32, _P, _P, _P, _SZ, _P, _I32, _I32, _I64, _P]),
    "gdl_fps_round_count": (ctypes.c_int, [_P, _I64, _I32, _I64, _P]),
    "gdl_knn_workspace_size": (_SZ, [_I64, _I32, _I32, _I64]),
    "gdl_knn_distance_count": (ctypes.c_int, [_P, _I64, _I32, _I32, _I64, ctypes.POINTER(ctypes.c_ulonglong)]),
    "gdl_knn": (ctypes.c_int, [_P, _P, _P, _P, _I32, _I64, _I32, _I64, _P, _P, _P, _SZ, _P]),
    "gdl_radius_graph_workspace_size": (_SZ, [_I64, _I32, _I32]),
    "gdl_radius_graph": (ctypes.c_int,
                         [_P, _P, _I32, _I64, _I64, ctypes.c_double, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _SZ,
                          _P]),
    "gdl_radius_graph_geometry": (ctypes.c_int,
                                  [_P, _P, _I32, _I64, _I64, ctypes.c_double, _I32, _I32, _P, _P, _P, _P, _P, _P,
                                   _PG, _P, _SZ, _P]),
    "gdl_edge_geometry_coo": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _PG, _P]),
    "gdl_cloud_avg_degree_workspace_size": (_SZ, [_I32]),
    "gdl_cloud_avg_degree": (ctypes.c_int, [_P, _P, _I64, _P, _P, _I32, _P, _P, _SZ, _P]),
    "gdl_radius_csr_finish": (ctypes.c_int, [_P, _P, _I64, _I64, _P, _I32, _P, _P, _P, _P, _P, _P]),
    "gdl_hybrid_graph_capacity": (_I64, [_I64, _I32, _I32]),
    "gdl_hybrid_graph_workspace_size": (_SZ, [_I64, _I32, _I32]),
    "gdl_hybrid_graph": (ctypes.c_int,
                         [_P, _P, _P, _P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _PG, _P, _SZ, _P]),
    "gdl_se3_aggregate": (ctypes.c_int, [_PS, _P, _I64, _P, _P, _I32, _P, _P, _P, _P, _P, _P, _I64, _I64, _P, _P, _P,
                                         _P]),
    "gdl_se3_aggregate_backward": (ctypes.c_int, [_PS, _P, _P, _P, _P, _P, _P, _I64, _P, _P, _I32, _P, _P, _P, _P, _P,
                                                  _P, _P, _I64, _I64, _P]),
    "gdl_knn_idw_weights": (ctypes.c_int, [_P, _P, _I64, _I32, _P, _P]),
    "gdl_knn_weighted_sum": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _I64, _I32, _P, _P]),
    "gdl_knn_weighted_sum_backward_workspace_size": (_SZ, [_I64, _I32, _I64]),
    "gdl_knn_weighted_sum_backward": (ctypes.c_int, [_P, _P, _P, _I32, _P, _P, _I64, _I32, _I64, _P, _SZ, _P]),
    "gdl_knn_weighted_sum_weight_grad": (ctypes.c_int, [_P, _P, _I64, _I64, _P, _I64, _I32, _I32, _P, _P]),
    "gdl_sort_and_build_csr_workspace_size": (_SZ, [_I64, _I64]),
    "gdl_sort_and_build_csr": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _P, _P, _P, _SZ, _P]),
    "gdl_segment_reduce_workspace_size": (_SZ, [_I64, _I64]),
    "gdl_segment_reduce": (ctypes.c_int, [_P, _I32, _I64, _I64, _P, _P, _P, _I64, _I32, _P, _P, _P, _SZ, _P]),
    "gdl_weight_grad_workspace_size": (ctypes.c_size_t, [_I64, _I32, _I32, _I32]),
    "gdl_weight_grad": (ctypes.c_int, [_P, _I64, _P, _I64, _I64, _I32, _I32, _I32, _P, _P, _P, ctypes.c_size_t, _P]),
    "gdl_segment_reduce_noalloc": (ctypes.c_int, [_P, _I32, _I64, _I64, _P, _P, _P, _I64, _I32, _P, _P, _P]),
    "gdl_segment_reduce_backward": (ctypes.c_int,
                                    [_P, _P, _I32, _P, _P, _I64, _I64, _P, _P, _P, _I64, _I32, _P, _P, _SZ, _P]),
    "gdl_gather_rows": (ctypes.c_int, [_P, _I64, _I64, _P, _I64, _P, _P]),
}

TIE = {"reference": 0, "lowest_index": 1}
REDUCE = {"sum": 0, "mean": 1, "max": 2}
DTYPE = {torch.float32: 0, torch.bfloat16: 1}

_lib = None
_lock = threading.Lock()
_checked_devices = set()


class GdlError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the operator library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise GdlError(f"{LIB_PATH} is missing: build it with `python -m gdl_b200.build`")
                lib = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in PROTOTYPES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def status_string(code: int) -> str:
    return load().gdl_status_string(int(code)).decode()


def check(code: int, what: str) -> None:
    if code != 0:
        raise GdlError(f"{what} failed: {status_string(code)} (status {code})")


def require_cuda(*tensors: torch.Tensor, what: str) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise GdlError(f"{what}: tensors must be on a CUDA device (this build has no CPU fallback)")
        dev = t.device if dev is None else dev
        if t.device != dev:
            raise GdlError(f"{what}: all tensors must be on the same device")
    if dev is None:
        raise GdlError(f"{what}: no CUDA tensor given")
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _checked_devices:
        check(load().gdl_check_device(idx), f"{what} (device {idx} is not an sm_100 GPU)")
        _checked_devices.add(idx)
    return dev


def to_device(t: torch.Tensor, device: torch.device, dtype: torch.dtype | None = None) -> torch.Tensor:
    """``t`` on ``device`` (converted to ``dtype``), contiguous. A CPU tensor is staged in pinned
    memory first: a copy from pageable memory makes the host wait for the work already queued on
    the stream, which would serialise the caller's Python with the GPU."""
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    if t.is_cuda:
        return t.to(device).contiguous()
    return t.contiguous().pin_memory().to(device, non_blocking=True)


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


_stream_ws = {}


def stream_workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A scratch buffer of at least `nbytes` kept per (device, current stream) and reused by the
    next call on that stream: work queued on one stream runs in order, so the next call's kernels
    start after this call's are done with it. Saves an allocation per call on small, launch-bound
    operators."""
    s = torch.cuda.current_stream(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(), s.cuda_stream)
    buf = _stream_ws.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _stream_ws[key] = buf
    return buf
