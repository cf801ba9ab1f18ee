"""Deterministic segment reduce -- drop-in for ``geoembodied.functional.segment_reduce``
(reference: geoembodied/functional/segment_reduce.py:41-313).

``segment_reduce`` keeps the reference signature and adds ``reduce`` ("sum" default, "mean",
"max"). Each variant is a ``torch.library.custom_op`` (namespace ``gdl_b200``, and also the
reference's ``geoembodied`` namespace when that is free) with a fake implementation and a
registered autograd formula, so ``torch.compile`` traces through it without graph breaks, as in
the reference (:206-279). Forward and backward are the
sm_100a kernels; nothing uses atomics on values, so results are bit-reproducible.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import Tensor

from .. import csrc


def sort_and_build_csr(col: Tensor, N: int) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """(col_sorted, perm, node_start, node_end), all int32: a stable sort of the edges by
    target plus CSR offsets; empty targets get start = end = 0 (reference :41-74)."""
    return csrc.sort_and_build_csr_cuda(col, N)


def _fake_out(msg: Tensor, N: int) -> Tensor:
    C = msg.shape[1] if msg.dim() > 1 else 1
    return msg.new_empty(N, C, dtype=torch.float32)


def _define_ops(ns: str, perm_optional: bool):
    """The three reductions as torch.library custom ops in namespace `ns`, each with a fake
    implementation and a registered autograd formula (reference: segment_reduce.py:206-279)."""
    perm_t = "Tensor?" if perm_optional else "Tensor"
    args = f"(Tensor msg, Tensor col_sorted, {perm_t} perm, Tensor node_start, Tensor node_end, SymInt N)"

    @torch.library.custom_op(f"{ns}::segment_reduce_sum", mutates_args=(), schema=f"{args} -> Tensor")
    def seg_sum(msg, col_sorted, perm, node_start, node_end, N):
        return csrc.segment_reduce_cuda(msg, perm, node_start, node_end, N, "sum")

    @seg_sum.register_fake
    def _(msg, col_sorted, perm, node_start, node_end, N):
        return _fake_out(msg, N)

    @torch.library.custom_op(f"{ns}::segment_reduce_mean", mutates_args=(), schema=f"{args} -> Tensor")
    def seg_mean(msg, col_sorted, perm, node_start, node_end, N):
        return csrc.segment_reduce_cuda(msg, perm, node_start, node_end, N, "mean")

    @seg_mean.register_fake
    def _(msg, col_sorted, perm, node_start, node_end, N):
        return _fake_out(msg, N)

    @torch.library.custom_op(f"{ns}::segment_reduce_max", mutates_args=(), schema=f"{args} -> (Tensor, Tensor)")
    def seg_max(msg, col_sorted, perm, node_start, node_end, N):
        return csrc.segment_reduce_cuda(msg, perm, node_start, node_end, N, "max", with_arg=True)

    @seg_max.register_fake
    def _(msg, col_sorted, perm, node_start, node_end, N):
        out = _fake_out(msg, N)
        return out, out.new_empty(out.shape, dtype=torch.int32)

    seg_sum.register_autograd(_backward_for("sum"), setup_context=_setup)
    seg_mean.register_autograd(_backward_for("mean"), setup_context=_setup)
    seg_max.register_autograd(_backward_for("max"), setup_context=_setup)
    return seg_sum, seg_mean, seg_max


# ----------------------------------------------------------------------------- autograd
def _setup(ctx, inputs, output):
    msg, col_sorted, perm, node_start, node_end, N = inputs
    ctx.N = N
    ctx.has_perm = perm is not None
    out, arg = (output if isinstance(output, tuple) else (None, None))
    ctx.save_for_backward(msg, col_sorted, perm if perm is not None else col_sorted, node_start, node_end, out, arg)


def _backward_for(reduce: str):
    def backward(ctx, grad_out, *unused):
        msg, col_sorted, perm, node_start, node_end, out, arg = ctx.saved_tensors
        g = csrc.segment_reduce_backward_cuda(grad_out.contiguous(), msg, out, arg, perm if ctx.has_perm else None,
                                              node_start, node_end, ctx.N, reduce)
        return g, None, None, None, None, None

    return backward


_seg_sum, _seg_mean, _seg_max = _define_ops("gdl_b200", perm_optional=True)


def _op_exists(ns: str, name: str) -> bool:
    try:
        return hasattr(getattr(torch.ops, ns), name)
    except Exception:
        return False


# The reference's own op name, torch.ops.geoembodied.segment_reduce_sum (segment_reduce.py:223,
# called at :311), with its schema (perm a Tensor), so that code and saved graphs that name it
# resolve to these kernels; plus geoembodied::segment_reduce_{mean,max}. Skipped when the
# namespace already holds the ops (the reference package was imported first: its own
# registration then stands, and callers reach these kernels through the geoembodied.csrc
# redirect instead).
GEOEMBODIED_OPS = None
if not _op_exists("geoembodied", "segment_reduce_sum"):
    GEOEMBODIED_OPS = _define_ops("geoembodied", perm_optional=False)


def segment_reduce(msg: Tensor, col_sorted: Tensor, perm: Optional[Tensor], node_start: Tensor, node_end: Tensor,
                   N: int, reduce: str = "sum") -> Tensor:
    """out [N, C] float32: reduce of msg[perm[j]] over slots j in [node_start[n], node_end[n]).

    sum  -- sequential fp32 fold in slot order, bit-identical to the reference kernel
            (segment_reduce_kernel.cu:66-93) for segments up to 4096 slots;
    mean -- sum / degree; max -- elementwise maximum (grad shared evenly among ties);
    empty segments give 0. msg may be float32 or bfloat16 (accumulated in float32; the
    gradient comes back in msg's dtype). perm=None means slot j reads row j.
    """
    if reduce == "sum":
        return _seg_sum(msg, col_sorted, perm, node_start, node_end, N)
    if reduce == "mean":
        return _seg_mean(msg, col_sorted, perm, node_start, node_end, N)
    if reduce == "max":
        return _seg_max(msg, col_sorted, perm, node_start, node_end, N)[0]
    raise ValueError(f"reduce must be 'sum', 'mean' or 'max', got {reduce!r}")


class SegmentReduceFunction(torch.autograd.Function):
    """autograd.Function form of the sum (reference: segment_reduce.py:112-158)."""

    @staticmethod
    def forward(ctx, msg, col_sorted, perm, node_start, node_end, N):
        ctx.save_for_backward(msg, col_sorted, perm, node_start, node_end)
        ctx.N = N
        return csrc.segment_reduce_cuda(msg, perm, node_start, node_end, N, "sum")

    @staticmethod
    def backward(ctx, grad_out):
        msg, col_sorted, perm, node_start, node_end = ctx.saved_tensors
        g = csrc.segment_reduce_backward_cuda(grad_out.contiguous(), msg, None, None, perm, node_start, node_end,
                                              ctx.N, "sum")
        return g, None, None, None, None, None
