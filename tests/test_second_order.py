"""Second derivatives through the kernels.

The backward of exp is L(A^T, G) = _frechet(A.mT, G).  When a graph of that backward is built
(create_graph=True), _frechet's own autograd formula gives the second derivative: for
Y = L(X, E) and upstream gradient H, dX = D^2 exp(X^T)[E^T, H] and dE = L(X^T, H).  The
second-order term is the upper-right block of the Frechet derivative of the doubled matrix
[[X^T, E^T], [0, X^T]] in direction diag(H, H): through the Frechet kernel while the doubled
size fits (n <= 16), through native operators beyond.  Checked against float64 autograd of the
float64 exponential.
"""

import pytest
import torch

import flash_hypercons as fh

from .reference import check_error, reference
from .test_routing import op_names

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [3, 8, 13, 16, 24, 32])
def test_second_derivative(n, dtype):
    gen = torch.Generator(device="cuda").manual_seed(9041 + n)
    a = (torch.randn(3, n, n, device="cuda", generator=gen) * (0.8 / n**0.5)).to(dtype).requires_grad_()
    g = (torch.randn(3, n, n, device="cuda", generator=gen) * 0.3).to(dtype)
    h = (torch.randn(3, n, n, device="cuda", generator=gen) * 0.3).to(dtype)
    y = fh.matrix_exp(a)
    (first,) = torch.autograd.grad(y, a, g, create_graph=True)
    second, names = op_names(lambda: torch.autograd.grad(first, a, h)[0])
    if 2 * n <= 32:
        assert "flash_hypercons::_frechet" in names
    # float64 autograd of the native float64 exponential on the CPU (the reference tests' ground truth)
    ref_a = a.detach().double().cpu().requires_grad_()
    (ref_first,) = torch.autograd.grad(torch.linalg.matrix_exp(ref_a), ref_a, g.double().cpu(), create_graph=True)
    (ref_second,) = torch.autograd.grad(ref_first, ref_a, h.double().cpu())
    check_error(first, ref_first.to(a.device), backward=True)
    check_error(second, ref_second.to(a.device), backward=True)


def test_second_derivative_of_direction():
    # d/dG <H, L(A^T, G)> = L(A, H)
    n = 8
    a = torch.randn(2, n, n, device="cuda") * 0.3
    g = (torch.randn(2, n, n, device="cuda") * 0.3).requires_grad_()
    h = torch.randn(2, n, n, device="cuda") * 0.3
    first = torch.ops.flash_hypercons._frechet(a.mT, g)
    (dg,) = torch.autograd.grad(first, g, h)
    check_error(dg, reference(a.double(), h.double()), backward=True)
