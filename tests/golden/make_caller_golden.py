"""Record the graph-operator calls that the reference's MultiScaleSE3Net makes.

Run in the build container, where the reference tree is importable:

    python tests/golden/make_caller_golden.py [/path/to/reference]

It imports ``geoembodied`` read-only, wraps the operator entry points that the unchanged
callers reach (``csrc._fps_iterative_fallback`` -- the pooling layer calls it directly, as
``nn/modules/equivariant_pool.py:261-265`` does --, ``functional.knn._knn_dispatch`` behind
``knn`` / ``knn_self``, ``functional.radius_graph.radius_graph``,
``functional.segment_reduce.sort_and_build_csr`` and ``segment_reduce``) in every loaded
``geoembodied`` module, runs one seeded forward and backward of a small
``nn.modules.multi_scale_se3_net.MultiScaleSE3Net`` (``multi_scale_se3_net.py:427``) on two
clouds of unequal size on the CPU, and stores each call -- its arguments and what the
reference's CPU path returned -- in ``golden_caller.npz``. The GPU replay test
(``tests/test_gpu_caller_replay.py``) feeds the same calls, in the same order, to this
library's drop-in functions and to the reference's own CUDA kernels.

``segment_reduce`` calls keep their CSR structure (``col_sorted``, ``perm``, node ranges) and
the message shape; the messages themselves are regenerated from a seed in the replay.
"""

from __future__ import annotations

import inspect
import json
import os
import sys
from pathlib import Path

import numpy as np

os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
sys.dont_write_bytecode = True

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

import torch  # noqa: E402

SIZES = (448, 320)   # two clouds of unequal size
SEED = 11


def _np(t):
    t = t.detach().cpu()
    if t.dtype == torch.int64:
        lo, hi = (int(t.min()), int(t.max())) if t.numel() else (0, 0)
        if -2**31 <= lo and hi < 2**31:
            return t.numpy().astype(np.int32)
    return t.numpy()


def record(root: str) -> dict:
    sys.path.insert(0, root)
    import importlib

    from tests.golden.make_golden import _stub_data_package

    _stub_data_package()
    csrc = importlib.import_module("geoembodied.csrc")
    fknn = importlib.import_module("geoembodied.functional.knn")
    frg = importlib.import_module("geoembodied.functional.radius_graph")
    fseg = importlib.import_module("geoembodied.functional.segment_reduce")
    msn = importlib.import_module("geoembodied.nn.modules.multi_scale_se3_net")

    calls = []
    arrays = {}

    def put(i, name, t):
        arrays[f"c{i}_{name}"] = _np(t)

    def wrap_fps(orig):
        def fps(pos, ptr, k_per_batch):
            out = orig(pos, ptr, k_per_batch)
            i = len(calls)
            calls.append({"op": "fps"})
            put(i, "pos", pos), put(i, "ptr", ptr), put(i, "k", k_per_batch), put(i, "out", out)
            return out
        return fps

    def wrap_knn(orig):
        def knn(query, source, ptr_q, ptr_s, k):
            idx, dist = orig(query, source, ptr_q, ptr_s, k)
            i = len(calls)
            calls.append({"op": "knn", "k": int(k), "self": query is source})
            put(i, "query", query), put(i, "ptr_q", ptr_q), put(i, "ptr_s", ptr_s)
            if query is not source:
                put(i, "source", source)
            put(i, "idx", idx), put(i, "dist", dist)
            return idx, dist
        return knn

    sig_rg = inspect.signature(frg.radius_graph)

    def wrap_rg(orig):
        def radius_graph(*args, **kwargs):
            row, col = orig(*args, **kwargs)
            b = sig_rg.bind(*args, **kwargs)
            b.apply_defaults()
            a = dict(b.arguments)
            i = len(calls)
            meta = {"op": "radius_graph", "r": float(a["r"]), "max_num_neighbors": int(a["max_num_neighbors"]),
                    "loop": bool(a["loop"])}
            if a.get("num_batch_elements") is not None:
                meta["num_batch_elements"] = int(a["num_batch_elements"])
            calls.append(meta)
            put(i, "x", a["x"])
            if a.get("batch") is not None:
                put(i, "batch", a["batch"])
            if a.get("mask") is not None:
                put(i, "mask", a["mask"])
            put(i, "row", row), put(i, "col", col)
            return row, col
        return radius_graph

    def wrap_csr(orig):
        def sort_and_build_csr(col, N):
            out = orig(col, N)
            i = len(calls)
            calls.append({"op": "sort_and_build_csr", "N": int(N)})
            put(i, "col", col)
            for name, t in zip(("col_sorted", "perm", "node_start", "node_end"), out):
                put(i, name, t)
            return out
        return sort_and_build_csr

    def wrap_seg(orig):
        def segment_reduce(msg, col_sorted, perm, node_start, node_end, N):
            out = orig(msg, col_sorted, perm, node_start, node_end, N)
            i = len(calls)
            calls.append({"op": "segment_reduce", "N": int(N), "shape": list(msg.shape),
                          "dtype": str(msg.dtype).replace("torch.", "")})
            put(i, "col_sorted", col_sorted), put(i, "perm", perm)
            put(i, "node_start", node_start), put(i, "node_end", node_end)
            return out
        return segment_reduce

    originals = {
        "_fps_iterative_fallback": (csrc._fps_iterative_fallback, wrap_fps),
        "_knn_dispatch": (fknn._knn_dispatch, wrap_knn),
        "radius_graph": (frg.radius_graph, wrap_rg),
        "sort_and_build_csr": (fseg.sort_and_build_csr, wrap_csr),
        "segment_reduce": (fseg.segment_reduce, wrap_seg),
    }
    wrapped = {id(f): w(f) for f, w in originals.values()}
    for name, mod in list(sys.modules.items()):
        if not name.startswith("geoembodied") or mod is None:
            continue
        for attr, val in list(vars(mod).items()):
            if callable(val) and id(val) in wrapped:
                setattr(mod, attr, wrapped[id(val)])

    torch.manual_seed(SEED)
    g = torch.Generator().manual_seed(SEED)
    pts = []
    for n in SIZES:  # clustered clouds: 6 blobs in a 2 m cube
        centres = torch.rand(6, 3, generator=g) * 2.0
        comp = torch.randint(0, 6, (n,), generator=g)
        pts.append(centres[comp] + 0.15 * torch.randn(n, 3, generator=g))
    pos = torch.cat(pts).float()
    ptr = torch.tensor([0, *np.cumsum(SIZES)], dtype=torch.int64)
    net = msn.MultiScaleSE3Net(in_channels=1, hidden_scalar=8, hidden_vector=2, num_stages=3, layers_per_stage=1,
                               pool_ratio=0.25, pool_k=8, interp_k=3, fusion_k=4)
    out = net(pos, ptr)
    loss = sum(o.float().square().sum() for o in out if torch.is_tensor(o) and o.is_floating_point())
    loss.backward()
    arrays["meta"] = np.array(json.dumps({"calls": calls, "sizes": list(SIZES), "seed": SEED}))
    return arrays


def main(argv):
    from oracle.build_ref import reference_root

    root = str(reference_root(argv[1] if len(argv) > 1 else None))
    arrays = record(root)
    np.savez_compressed(HERE / "golden_caller.npz", **arrays)
    meta = json.loads(str(arrays["meta"]))
    print(f"{len(meta['calls'])} calls:", [c["op"] for c in meta["calls"]])


if __name__ == "__main__":
    main(sys.argv)
