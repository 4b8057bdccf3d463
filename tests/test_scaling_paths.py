"""Large scaling exponents, far beyond the benchmark distributions.

A = c e_0 e_{n-1}^T is nilpotent (A^2 = 0), so exp(A) = I + A and L(A, E) = E + (AE + EA)/2 +
AEA/6 stay representable for norms far beyond theta_18: c = 1e3 (s = 9), 1e11 (s = 35) and
1e13 (s = 42).  Every matrix is checked against the float64 oracle with the reference's
per-matrix criterion, in a batch that mixes them with ordinary matrices.
"""

import pytest
import torch

import flash_hypercons as fh
from oracle import expm_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [4, 8, 16, 17, 32])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_nilpotent_large_norms(n, dtype):
    gen = torch.Generator().manual_seed(9041 + n)
    scales = [1e3, 1e11, 1e13]
    a = torch.randn((2 * len(scales), n, n), generator=gen) / n**0.5
    for i, c in enumerate(scales):
        a[2 * i] = 0
        a[2 * i, 0, n - 1] = c
    g = torch.randn(a.shape, generator=gen)
    a, g = a.to(dtype), g.to(dtype)
    x = a.cuda().requires_grad_()
    y = fh.matrix_exp(x)
    (grad,) = torch.autograd.grad(y, x, g.cuda())
    exact_y, exact_g = O.exp_fp64(a), O.frechet_fp64(a.mT, g)
    kind = "float32" if dtype == torch.float32 else "half"
    err_y = O.per_matrix_error(y, exact_y)
    err_g = O.per_matrix_error(grad, exact_g)
    assert err_y.max() <= O.tolerance(kind, False), err_y
    assert err_g.max() <= O.tolerance(kind, True), err_g
