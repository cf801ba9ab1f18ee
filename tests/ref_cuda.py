"""Loader of the reference's own CUDA extensions built by oracle/build_ref.py.

TEST INFRASTRUCTURE: the GPU parity tests use these modules, when present, as the
strongest checker -- the unmodified reference kernels run on the same B200 as ours.
"""

import importlib.machinery
import importlib.util
from pathlib import Path

REF_DIR = Path(__file__).resolve().parent.parent / "oracle" / "_ref"
_mods = {}


def load(name: str):
    """name in {'fps', 'knn', 'radius_graph', 'segment_reduce'}; None if not built."""
    if name in _mods:
        return _mods[name]
    full = f"geoembodied_{name}_cuda"
    so = REF_DIR / full / f"{full}.so"
    mod = None
    if so.exists():
        import torch  # noqa: F401  (the extension links against torch)

        loader = importlib.machinery.ExtensionFileLoader(full, str(so))
        spec = importlib.util.spec_from_file_location(full, str(so), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
    _mods[name] = mod
    return mod


def available() -> bool:
    return all(load(n) is not None for n in ("fps", "knn", "radius_graph", "segment_reduce"))
