"""The segment-reduce custom ops under the reference's own op name.

The reference registers ``geoembodied::segment_reduce_sum`` (geoembodied/functional/
segment_reduce.py:223) and calls it as ``torch.ops.geoembodied.segment_reduce_sum`` (:311). This
library registers the same name with the same schema (plus ``_mean`` / ``_max``) when the namespace
is free, so code and saved graphs that name the reference op resolve to these kernels. The schema
is compared with the one the reference itself registers (the reference package imported in a
separate process, where the reference tree is present).
"""

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _schema_in_subprocess(code: str, extra_path: str) -> str:
    env_path = [extra_path, str(ROOT)]
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                         env={"PYTHONPATH": ":".join(env_path), "PYTHONDONTWRITEBYTECODE": "1",
                              "PATH": "/usr/bin:/bin"})
    assert out.returncode == 0, out.stderr[-2000:]
    return out.stdout.strip().splitlines()[-1]


def test_ops_are_registered_with_the_reference_schema():
    import gdl_b200.functional  # noqa: F401

    s = str(torch.ops.geoembodied.segment_reduce_sum.default._schema)
    assert s == ("geoembodied::segment_reduce_sum(Tensor msg, Tensor col_sorted, Tensor perm, Tensor node_start, "
                 "Tensor node_end, SymInt N) -> Tensor")
    assert hasattr(torch.ops.geoembodied, "segment_reduce_mean")
    assert hasattr(torch.ops.geoembodied, "segment_reduce_max")
    assert "Tensor? perm" in str(torch.ops.gdl_b200.segment_reduce_sum.default._schema)


def test_schema_equals_the_reference_registration():
    import importlib.util

    spec = importlib.util.spec_from_file_location("gdl_build_ref", ROOT / "oracle" / "build_ref.py")
    build_ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build_ref)
    ref = build_ref.reference_root()
    if ref is None or not (ref / "geoembodied" / "functional" / "segment_reduce.py").is_file():
        pytest.skip("reference tree not present")
    code = ("import torch, geoembodied.functional.segment_reduce as m; "
            "print(torch.ops.geoembodied.segment_reduce_sum.default._schema)")
    theirs = _schema_in_subprocess(code, str(ref))
    code = ("import torch, gdl_b200.functional; "
            "print(torch.ops.geoembodied.segment_reduce_sum.default._schema)")
    ours = _schema_in_subprocess(code, str(ROOT))
    assert ours == theirs, json.dumps([ours, theirs])
