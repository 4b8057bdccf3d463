"""Tensor subclasses in the backward of fh.matrix_exp.

The original package's backward checks ``has_torch_function((input, grad_output))`` and, for a
subclass that overrides ``__torch_function__``, computes the gradient with the native block
formula in Python, so that the subclass sees those operators and the gradient comes back as the
subclass (flash_hypercons/ops/matrix_exp/__init__.py:66-72).  Subclasses whose
``__torch_function__`` is disabled (``__torch_dispatch__`` subclasses) keep the package's
``_frechet`` operator there, and so they do here.
"""

import pytest
import torch
from torch.utils._pytree import tree_map

import flash_hypercons as fh
from oracle import expm_oracle as O

from .test_routing import op_names

pytestmark = pytest.mark.gpu


class Tagged(torch.Tensor):
    """A __torch_function__ subclass: every operator result is a Tagged."""


class RecordingTensor(torch.Tensor):
    """Wrapper subclass (__torch_dispatch__) that records every operator it sees."""

    seen: list = []

    @staticmethod
    def __new__(cls, elem):
        return torch.Tensor._make_wrapper_subclass(cls, elem.shape, dtype=elem.dtype, device=elem.device,
                                                   strides=elem.stride())

    def __init__(self, elem):
        self.elem = elem

    @classmethod
    def __torch_dispatch__(cls, func, types, args=(), kwargs=None):
        cls.seen.append(str(func))
        unwrap = lambda t: t.elem if isinstance(t, RecordingTensor) else t  # noqa: E731
        wrap = lambda t: RecordingTensor(t) if isinstance(t, torch.Tensor) else t  # noqa: E731
        return tree_map(wrap, func(*tree_map(unwrap, args), **tree_map(unwrap, kwargs or {})))


def test_torch_function_subclass_gradient_takes_native_formula():
    a = (torch.randn(6, 5, 5, device="cuda") * 0.5).requires_grad_()
    g = torch.randn(6, 5, 5, device="cuda")
    y = fh.matrix_exp(a)
    (grad,), names = op_names(lambda: torch.autograd.grad(y, a, g.as_subclass(Tagged)))
    assert type(grad) is Tagged
    assert "flash_hypercons::_frechet" not in names
    err = O.per_matrix_error(grad.as_subclass(torch.Tensor), O.frechet_fp64(a.detach().mT, g)).max()
    assert err <= O.tolerance("float32", True), err
    # plain gradients keep the kernel
    y = fh.matrix_exp(a)
    _, names = op_names(lambda: torch.autograd.grad(y, a, g))
    assert "flash_hypercons::_frechet" in names


def test_dispatch_subclass_gradient_keeps_frechet_operator():
    a = (torch.randn(6, 5, 5, device="cuda") * 0.5).requires_grad_()
    g = torch.randn(6, 5, 5, device="cuda")
    y = fh.matrix_exp(a)
    RecordingTensor.seen = []
    (grad,) = torch.autograd.grad(y, a, RecordingTensor(g))
    assert isinstance(grad, RecordingTensor)
    assert any("flash_hypercons._frechet" in name for name in RecordingTensor.seen), RecordingTensor.seen
    err = O.per_matrix_error(grad.elem, O.frechet_fp64(a.detach().mT, g)).max()
    assert err <= O.tolerance("float32", True), err
