"""Tensor subclasses with Python dispatch in the backward of fh.matrix_exp.

The original package's backward checks ``has_torch_function((input, grad_output))`` and then
computes the gradient with native operators (flash_hypercons/ops/matrix_exp/__init__.py:66-72),
so a ``__torch_dispatch__`` subclass passed as the incoming gradient sees only native aten
operators and the gradient comes back as that subclass.  Same here.
"""

import pytest
import torch
from torch.utils._pytree import tree_map

import flash_hypercons as fh
from oracle import expm_oracle as O

pytestmark = pytest.mark.gpu


class RecordingTensor(torch.Tensor):
    """Wrapper subclass that records every aten operator it sees."""

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


def test_subclass_gradient_takes_native_formula():
    a = (torch.randn(6, 5, 5, device="cuda") * 0.5).requires_grad_()
    g = torch.randn(6, 5, 5, device="cuda")
    y = fh.matrix_exp(a)
    RecordingTensor.seen = []
    (grad,) = torch.autograd.grad(y, a, RecordingTensor(g))
    assert isinstance(grad, RecordingTensor)
    assert not any("flash_hypercons" in name for name in RecordingTensor.seen), RecordingTensor.seen
    assert any("matrix_exp" in name for name in RecordingTensor.seen)
    err = O.per_matrix_error(grad.elem, O.frechet_fp64(a.detach().mT, g)).max()
    assert err <= O.tolerance("float32", True), err
