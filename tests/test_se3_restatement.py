"""Pin the float64 restatement of SE3Conv (oracle/se3_ref.py), which the GPU tests use as the
reference of the fused message kernel, against the reference's own CPU outputs
(tests/golden/golden_se3.npz, made by tests/golden/make_golden.py). The reference computes in
fp32, so the bar is its rounding bound: |ref32 - f64| <= 1e-5 * (the same expression on
absolute values) + 1e-7, per element."""

import numpy as np
import pytest
import torch

from oracle import se3_ref as se3_f64


@pytest.fixture(scope="module")
def gs():
    from tests.conftest import ROOT

    return np.load(ROOT / "tests" / "golden" / "golden_se3.npz")


DIMS = {"full": (16, 8, 24, 6, 4, 3), "sv": (16, 8, 24, 6, 0, 0)}


def _sd(gs, tag):
    pre = f"se3_{tag}_sd_"
    return {k[len(pre):]: torch.from_numpy(gs[k]) for k in gs.files if k.startswith(pre)}


def _inputs(gs, tag):
    t = lambda k: torch.from_numpy(gs[k])  # noqa: E731
    t2 = t(f"se3_{tag}_in_t2") if f"se3_{tag}_in_t2" in gs.files else None
    return (t("se3_pos"), t("se3_row"), t("se3_col"), t(f"se3_{tag}_in_s"), t(f"se3_{tag}_in_v"), t2)


@pytest.mark.parametrize("tag", ["full", "sv"])
def test_restatement_matches_reference(gs, tag):
    sd, dims = _sd(gs, tag), DIMS[tag]
    pos, row, col, s, v, t2 = _inputs(gs, tag)
    clouds = [(0, 150), (150, 300)]
    ref = se3_f64.se3_forward(sd, dims, pos, row, col, s, v, t2, clouds, cutoff=0.3)
    bound = se3_f64.se3_forward(sd, dims, pos, row, col, s, v, t2, clouds, cutoff=0.3, absolute=True)
    names = ["s", "v", "t2"] if dims[5] else ["s", "v"]
    for i, nm in enumerate(names):
        got = torch.from_numpy(gs[f"se3_{tag}_out_{nm}"]).double()
        assert torch.all((got - ref[i]).abs() <= 1e-5 * bound[i] + 1e-7), nm
    assert torch.equal(sd.get("cg_11_2", torch.zeros(0)).float() if dims[5] else torch.zeros(0),
                       se3_f64.cg_cart().float() if dims[5] else torch.zeros(0))
