"""The small-bucket FPS kernel's warp-box pre-filter, restated in float32 on the CPU (no GPU).

``fps_bucket_kernel`` (gdl_b200/csrc/fps.cu) with buckets of 4 points tests each round's picks
first against its warp's box -- the union of its lanes' boxes, reduced with ``redux.sync`` over an
order-preserving integer image of each coordinate -- and its lanes' largest minimum, and lets a
lane test only the picks that pass. The pre-filter changes no result only if (1) the integer image
orders floats as the floats order (so the reduced box contains every lane's box) and (2) the
kernel's box bound ``box_dist2_lb`` never decreases from a box to a box inside it, so a pick that
fails against the warp's box fails every lane's own test. Both are checked here.
"""

import numpy as np

F = np.float32


def _key(x):
    b = np.asarray(x, F).view(np.int32)
    return np.where(b >= 0, b, b ^ np.int32(0x7FFFFFFF))


def _unkey(k):
    k = np.asarray(k, np.int32)
    return np.where(k >= 0, k, k ^ np.int32(0x7FFFFFFF)).view(F)


def _box_dist2_lb(s, bx):
    # box_dist2_lb: per axis fmaxf(fmaxf(lo - s, s - hi), 0), then fma(gz, gz, fma(gx, gx, gy * gy))
    # (np.fmax, like fmaxf, returns the other operand when one is NaN)
    g = np.fmax(np.fmax((bx[..., :3] - s).astype(F), (s - bx[..., 3:]).astype(F)), F(0.0)).astype(F)
    gy2 = (g[..., 1] * g[..., 1]).astype(F)
    t = (g[..., 0].astype(np.float64) ** 2 + gy2).astype(F)
    return (g[..., 2].astype(np.float64) ** 2 + t).astype(F)


def test_integer_image_orders_like_the_floats():
    rng = np.random.default_rng(0)
    special = np.array([0.0, -0.0, np.inf, -np.inf, 1e-45, -1e-45, 1.17549435e-38, -1.17549435e-38,
                        3.4028235e38, -3.4028235e38, 1.0, -1.0], F)
    x = np.concatenate([special, (rng.standard_normal(20000) * 10.0 ** rng.integers(-30, 30, 20000)).astype(F)])
    assert np.array_equal(_unkey(_key(x)).view(np.int32), x.view(np.int32))  # a bijection
    o = np.argsort(_key(x), kind="stable")
    xs = x[o]
    assert np.all(xs[:-1] <= xs[1:])  # integer order is float order (-0 before +0 among equals)
    for _ in range(200):  # warp reductions: 32 lanes' values, as redux.sync min / max would
        lanes = rng.choice(x, 32)
        assert _unkey(_key(lanes).min()) == lanes.min() and _unkey(_key(lanes).max()) == lanes.max()


def test_box_bound_never_decreases_into_a_contained_box():
    rng = np.random.default_rng(1)
    n = 200000
    c = (rng.standard_normal((n, 3)) * 50.0).astype(F)
    half = np.abs(rng.standard_normal((n, 3)) * 0.5).astype(F)
    inner = np.concatenate([(c - half).astype(F), (c + half).astype(F)], axis=1)
    grow = np.abs(rng.standard_normal((n, 6)) * rng.choice([0.0, 1e-6, 0.3], (n, 6))).astype(F)
    outer = np.concatenate([(inner[:, :3] - grow[:, :3]).astype(F), (inner[:, 3:] + grow[:, 3:]).astype(F)], axis=1)
    s = (c + (rng.standard_normal((n, 3)) * rng.choice([0.01, 1.0, 30.0], (n, 1))).astype(F)).astype(F)
    s[:100] = np.nan  # a non-finite pick: its axes bound 0 against both boxes
    s[100:200, 0] = np.inf
    lb_in, lb_out = _box_dist2_lb(s, inner), _box_dist2_lb(s, outer)
    assert np.all(lb_out <= lb_in)
