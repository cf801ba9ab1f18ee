"""gdl_weight_grad (the weight / bias gradients of SE3Conv's projection and radial-MLP layers)
against a float64 torch contraction of the same fp32 inputs, within the fp32 rounding bound of a
sum of |terms|, over the shapes SE3Conv uses, ragged tiles, strided rows, sub = 1 / 3 / 5 and empty
inputs; repeated calls are bit-identical (fixed slice order)."""

import math

import pytest
import torch

from gdl_b200 import csrc

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]
DEV = "cuda"


def _ref(A, B, sub):
    rows = A.shape[0]
    a = A.double().reshape(rows, -1, sub)
    b = B.double().reshape(rows, -1, sub)
    return torch.einsum("rmj,rnj->mn", a, b), torch.einsum("rmj,rnj->mn", a.abs(), b.abs())


def _check(C, ref, bound, rows, sub):
    # fp32 accumulation: |error| <= (terms per chain) * 2^-24 * sum|terms|, with sqrt growth typical;
    # the bound below is the worst case over a chain of rows * sub terms
    tol = rows * sub * 2.0 ** -24 * bound + 1e-30
    assert torch.all((C.double() - ref).abs() <= tol)


@pytest.mark.parametrize("rows,M,N,sub", [
    (1, 1, 1, 1), (5, 3, 2, 1), (37, 9, 64, 1), (43_900, 9, 64, 1), (43_900, 64, 16, 1), (8192, 176, 128, 1),
    (8192, 208, 32, 3), (8192, 16, 16, 5), (1000, 130, 65, 3), (70_001, 65, 129, 1), (3, 70, 70, 5)])
def test_weight_grad_matches_float64(rows, M, N, sub):
    g = torch.Generator().manual_seed(rows * 7 + M * 3 + N + sub)
    A = torch.randn(rows, M, sub, generator=g).to(DEV)
    B = torch.randn(rows, N, sub, generator=g).to(DEV)
    if sub == 1:
        A, B = A[..., 0], B[..., 0]
    C, cs = csrc.weight_grad_cuda(A, B, sub, col_sum=sub == 1)
    ref, bound = _ref(A.reshape(rows, -1).cpu(), B.reshape(rows, -1).cpu(), sub)
    _check(C.cpu(), ref, bound, rows, sub)
    if sub == 1:
        a64 = A.double().cpu()
        tol = rows * 2.0 ** -24 * a64.abs().sum(0) + 1e-30
        assert torch.all((cs.double().cpu() - a64.sum(0)).abs() <= tol)
    C2, cs2 = csrc.weight_grad_cuda(A, B, sub, col_sum=sub == 1)
    assert torch.equal(C, C2)
    if sub == 1:
        assert torch.equal(cs, cs2)


def test_weight_grad_strided_column_slices():
    """A and B as column slices of wider row-major matrices (row stride > width), as the grouped
    projection gradients hand them over."""
    g = torch.Generator().manual_seed(5)
    wideA = torch.randn(4096, 3 * 100, generator=g).to(DEV)
    wideB = torch.randn(4096, 3 * 50, generator=g).to(DEV)
    A = wideA.view(4096, 100, 3)[:, 20:60, :]
    B = wideB.view(4096, 50, 3)[:, 10:33, :]
    C, _ = csrc.weight_grad_cuda(A, B, 3)
    ref, bound = _ref(A.contiguous().reshape(4096, -1).cpu(), B.contiguous().reshape(4096, -1).cpu(), 3)
    _check(C.cpu(), ref, bound, 4096, 3)
    A1, B1 = wideA[:, 7:90], wideB[:, :31]
    C1, _ = csrc.weight_grad_cuda(A1, B1, 1, col_sum=True)
    ref1, bound1 = _ref(A1.cpu(), B1.cpu(), 1)
    _check(C1.cpu(), ref1, bound1, 4096, 1)


def test_weight_grad_empty_rows_give_zeros():
    A = torch.empty(0, 7, device=DEV)
    B = torch.empty(0, 5, device=DEV)
    C, cs = csrc.weight_grad_cuda(A, B, 1, col_sum=True)
    assert C.shape == (7, 5) and torch.all(C == 0) and torch.all(cs == 0)


def test_weight_grad_no_input_columns_still_sums_the_output_gradient():
    """A layer with zero input features (N == 0) has no weight entries but a bias gradient."""
    g = torch.Generator().manual_seed(9)
    A = torch.randn(3000, 7, generator=g).to(DEV)
    B = torch.empty(3000, 0, device=DEV)
    C, cs = csrc.weight_grad_cuda(A, B, 1, col_sum=True)
    assert C.shape == (7, 0)
    want = A.double().sum(0).float()
    assert torch.allclose(cs, want, rtol=1e-6, atol=1e-5)


def test_radial_mlp_gradients_match_nn_linear():
    """The radial MLP through the row-linear function gives nn.Linear's gradients (float64 run of
    the same weights as the reference)."""
    from gdl_b200.se3_conv import RadialBasis

    torch.manual_seed(0)
    rb = RadialBasis(num_basis=16, cutoff=2.0, num_hidden=64, num_output=9).to(DEV)
    dist = torch.rand(20_000, device=DEV) * 2.0 + 0.01
    out = rb(dist)
    gy = torch.randn_like(out)
    out.backward(gy)
    grads = [p.grad.clone() for p in rb.mlp.parameters()]
    rb64 = RadialBasis(num_basis=16, cutoff=2.0, num_hidden=64, num_output=9).double().to(DEV)
    rb64.load_state_dict({k: v.double() for k, v in rb.state_dict().items()})
    d = dist.double().unsqueeze(-1)
    basis = torch.sin(rb64.freqs * d) / d.clamp(min=1e-8)
    envelope = (0.5 * (1.0 + torch.cos(math.pi * dist.double() / rb64.cutoff))).clamp(min=0.0).unsqueeze(-1)
    y = rb64.mlp(basis * envelope)
    y.backward(gy.double())
    assert (out.double() - y).abs().max().item() <= 1e-4 * y.abs().max().item()
    for g32, p in zip(grads, rb64.mlp.parameters()):
        assert (g32.double() - p.grad).abs().max().item() <= 1e-4 * p.grad.abs().max().item() + 1e-12
