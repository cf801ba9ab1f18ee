"""Build the reference's own CUDA operator extensions as a GPU-side parity checker.

TEST INFRASTRUCTURE ONLY. The product never imports anything under ``oracle/``.

This compiles the four unmodified reference sources
(``geoembodied/csrc/{fps,knn,radius_graph,segment_reduce}_kernel.cu``) exactly the way
the reference's loader does (``geoembodied/csrc/__init__.py:94-103``: flags
``-O3 --use_fast_math -lineinfo``), but for sm_100a, with all build output under
``oracle/_ref/``. The resulting Python extension modules are loaded by the GPU parity
tests (``tests/ref_cuda.py``) to pin the CPU restatement and the product kernels
against the reference kernels themselves. It runs only where the reference tree
exists (the build container); the built ``.so`` files travel with the repository
snapshot to the GPU box.

Usage: ``python oracle/build_ref.py [REFERENCE_ROOT]``. Without the argument the root comes from
the environment variable GDL_REFERENCE_ROOT, else from ``reference_path`` in the repository's
BASELINE.json (the record of where the reference was mounted for this build).
"""

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def reference_root(argv_root=None):
    """The reference tree: the given path, GDL_REFERENCE_ROOT, or BASELINE.json's reference_path
    (None if none is set)."""
    if argv_root:
        return Path(argv_root)
    env = os.environ.get("GDL_REFERENCE_ROOT")
    if env:
        return Path(env)
    baseline = HERE.parent / "BASELINE.json"
    if baseline.exists():
        import json

        p = json.loads(baseline.read_text()).get("reference_path")
        if p:
            return Path(p)
    return None

# (module name used by the reference loader, source file)
# geoembodied/csrc/__init__.py:95, :230, :346, :536
MODULES = [
    ("geoembodied_fps_cuda", "fps_kernel.cu"),
    ("geoembodied_knn_cuda", "knn_kernel.cu"),
    ("geoembodied_radius_graph_cuda", "radius_graph_kernel.cu"),
    ("geoembodied_segment_reduce_cuda", "segment_reduce_kernel.cu"),
]


def build(ref_root: Path, only=None) -> None:
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load

    csrc = ref_root / "geoembodied" / "csrc"
    for name, src in MODULES:
        if only and name not in only:
            continue
        bdir = OUT / name
        bdir.mkdir(parents=True, exist_ok=True)
        so = bdir / f"{name}.so"
        if so.exists() and so.stat().st_mtime > (csrc / src).stat().st_mtime:
            print(f"[build_ref] {name}: up to date")
            continue
        print(f"[build_ref] building {name} from {csrc / src}", flush=True)
        load(
            name=name,
            sources=[str(csrc / src)],
            extra_cuda_cflags=["-O3", "--use_fast_math", "-lineinfo"],
            build_directory=str(bdir),
            verbose=False,
        )


if __name__ == "__main__":
    root = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    only = sys.argv[2:] or None
    if root is None or not (root / "geoembodied" / "csrc").is_dir():
        print(f"[build_ref] reference tree not found at {root}; nothing to build")
        sys.exit(0)
    build(root, only)
