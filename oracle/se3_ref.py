"""Torch restatement of the reference SE3Conv forward.

TEST INFRASTRUCTURE ONLY (the checker of the fused SE3Conv message kernel and the CPU baseline
of its benchmark configuration); the product never imports it.

Restates geoembodied/nn/modules/se3_conv.py: RadialBasis (:271-284), _compute_messages paths 0-8
(:61-235) with the reference's per-edge association (gather the source rows, mix channels per
edge), the per-target sum, the division by the cloud's average degree and the scalar bias
(:487-545), in ``dtype`` (float64 for the checks) on whatever device the inputs are on.
``absolute=True`` evaluates every product and sum on absolute values, which bounds the rounding
error of any fp32 evaluation order of the same expression. Pinned against the reference's own CPU
outputs in tests/test_se3_restatement.py.
"""

from __future__ import annotations

import math

import torch

C0 = math.sqrt(1.0 / (4.0 * math.pi))
C1 = math.sqrt(3.0 / (4.0 * math.pi))
C20 = math.sqrt(5.0 / (16.0 * math.pi))
C21 = math.sqrt(15.0 / (4.0 * math.pi))
C22 = math.sqrt(15.0 / (16.0 * math.pi))


def cg_cart():
    h = 1.0 / math.sqrt(2.0)
    c = torch.zeros(3, 3, 5, dtype=torch.float64)
    c[0, 1, 0] = c[1, 0, 0] = h
    c[1, 2, 1] = c[2, 1, 1] = h
    c[2, 2, 2] = 2.0 / math.sqrt(6.0)
    c[0, 0, 2] = c[1, 1, 2] = -1.0 / math.sqrt(6.0)
    c[0, 2, 3] = c[2, 0, 3] = h
    c[0, 0, 4] = h
    c[1, 1, 4] = -h
    return c


def geometry(pos, row, col):
    diff = pos[col] - pos[row]
    dist = diff.norm(dim=-1).clamp(min=1e-8)
    u = diff / dist[:, None]
    x, y, z = u[:, 0], u[:, 1], u[:, 2]
    Y = torch.stack([torch.full_like(x, C0), C1 * y, C1 * z, C1 * x, C21 * x * y, C21 * y * z,
                     C20 * (3 * z * z - 1), C21 * x * z, C22 * (x * x - y * y)], dim=-1)
    return dist, u, Y


def avg_degree(col, N, clouds):
    deg = torch.zeros(N, dtype=torch.float64, device=col.device).index_add_(0, col, torch.ones_like(col,
                                                                                                  dtype=torch.float64))
    out = torch.empty(N, dtype=torch.float64, device=col.device)
    for a, b in clouds:
        out[a:b] = deg[a:b].sum() / max(b - a, 1)
    return out.clamp(min=1.0)


def radial(sd, dist, cutoff, num_basis):
    t = dist.dtype
    f = sd["radial_basis.freqs"].to(t)
    d = dist[:, None]
    basis = torch.sin(f * d) / d.clamp(min=1e-8)
    env = (0.5 * (1.0 + torch.cos(math.pi * dist / cutoff))).clamp(min=0.0)[:, None]
    h = torch.nn.functional.silu((basis * env) @ sd["radial_basis.mlp.0.weight"].to(t).t()
                                 + sd["radial_basis.mlp.0.bias"].to(t))
    return h @ sd["radial_basis.mlp.2.weight"].to(t).t() + sd["radial_basis.mlp.2.bias"].to(t)


def se3_forward(sd, dims, pos, row, col, s, v, t2, clouds, cutoff, num_basis=16, absolute=False, R=None,
                dtype=torch.float64):
    """(s_out, v_out, t2_out) in ``dtype``; sd = state dict (tensors), dims = (Cs_in, Cv_in, Cs_out,
    Cv_out, Ct2_in, Ct2_out). ``R`` (optional) replaces the radial weights."""
    cs_i, cv_i, cs_o, cv_o, ct_i, ct_o = dims
    N = pos.shape[0]
    dist, u, Y = geometry(pos.to(dtype), row, col)
    if R is None:
        R = radial(sd, dist, cutoff, num_basis)
    R = R.to(dtype)
    W = {k: sd[k].to(dtype) for k in sd if k.startswith("w_")}
    s, v = s.to(dtype)[row], v.to(dtype)[row]
    t2 = t2.to(dtype)[row] if t2 is not None else None
    Y0, Y2 = Y[:, 0:1], Y[:, 4:9]
    if absolute:
        ab = torch.abs
        R, u, Y0, Y2, s, v = ab(R), ab(u), ab(Y0), ab(Y2), ab(s), ab(v)
        t2 = ab(t2) if t2 is not None else None
        W = {k: ab(w) for k, w in W.items()}
    E = row.shape[0]
    ms = torch.zeros(E, cs_o, dtype=dtype, device=pos.device)
    mv = torch.zeros(E, cv_o, 3, dtype=dtype, device=pos.device)
    mt = torch.zeros(E, ct_o, 5, dtype=dtype, device=pos.device)
    p = 0

    def r():
        return R[:, p:p + 1]

    def cross(a, b):  # a [E,1,3] x b [E,C,3]; absolute: |a||b| products of the same pairs
        if absolute:
            return torch.stack([a[..., 1] * b[..., 2] + a[..., 2] * b[..., 1],
                                a[..., 2] * b[..., 0] + a[..., 0] * b[..., 2],
                                a[..., 0] * b[..., 1] + a[..., 1] * b[..., 0]], dim=-1)
        return torch.linalg.cross(a.expand_as(b), b, dim=-1)

    if "w_ss.weight" in W:
        ms = ms + r() * Y0 * (s @ W["w_ss.weight"].t())
        p += 1
    if "w_sv.weight" in W:
        mv = mv + (r() * (s @ W["w_sv.weight"].t())).unsqueeze(-1) * u.unsqueeze(-2)
        p += 1
    if "w_vv_scalar.weight" in W:
        mv = mv + r().unsqueeze(-1) * Y0.unsqueeze(-1) * (v.transpose(-1, -2) @ W["w_vv_scalar.weight"].t()
                                                         ).transpose(-1, -2)
        p += 1
    if "w_vs.weight" in W:
        ms = ms + r() * ((u.unsqueeze(-2) * v).sum(-1) @ W["w_vs.weight"].t())
        p += 1
    if "w_vv_cross.weight" in W:
        c = cross(u.unsqueeze(-2), v)
        mv = mv + r().unsqueeze(-1) * (c.transpose(-1, -2) @ W["w_vv_cross.weight"].t()).transpose(-1, -2)
        p += 1
    if ct_o > 0:
        if "w_st2.weight" in W:
            mt = mt + (r() * (s @ W["w_st2.weight"].t())).unsqueeze(-1) * Y2.unsqueeze(-2)
            p += 1
        if "w_t2t2.weight" in W and t2 is not None:
            mt = mt + r().unsqueeze(-1) * Y0.unsqueeze(-1) * (t2.transpose(-1, -2) @ W["w_t2t2.weight"].t()
                                                             ).transpose(-1, -2)
            p += 1
        if "w_vt2.weight" in W:
            cg = cg_cart().to(device=pos.device, dtype=dtype)
            cg = torch.abs(cg) if absolute else cg
            outer = (u[:, None, :, None] * v[:, :, None, :]).reshape(E, v.shape[1], 9)
            tp = outer @ cg.reshape(9, 5)
            mt = mt + r().unsqueeze(-1) * (tp.transpose(-1, -2) @ W["w_vt2.weight"].t()).transpose(-1, -2)
            p += 1
    if "w_t2s.weight" in W and t2 is not None:
        ms = ms + r() * ((t2 * t2).sum(-1) @ W["w_t2s.weight"].t())
        p += 1
    avg = avg_degree(col, N, clouds).to(dtype)
    so = torch.zeros(N, cs_o, dtype=dtype, device=pos.device).index_add_(0, col, ms) / avg[:, None]
    vo = torch.zeros(N, cv_o, 3, dtype=dtype, device=pos.device).index_add_(0, col, mv) / avg[:, None, None]
    to = torch.zeros(N, ct_o, 5, dtype=dtype, device=pos.device).index_add_(0, col, mt) / avg[:, None, None]
    if "scalar_bias" in sd and cs_o > 0:
        b = sd["scalar_bias"].to(dtype)
        so = so + (torch.abs(b) if absolute else b)
    return so, vo, to
