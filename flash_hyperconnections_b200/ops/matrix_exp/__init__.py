# Interface (function names, predicates, fakes, public docstrings) follows
# nickjeliopoulos/flash-hyperconnections, flash_hypercons/ops/matrix_exp/__init__.py.
# Copyright (c) 2023-2026 Nicholas John Eliopoulos, Purvish Jatin Jajal.  MIT License; the full
# permission notice is in tests/LICENSE.flash-hyperconnections.
"""Python operator layer: eligibility, native routing, fake kernels, scoped routing.

Behaviour mirrors flash_hypercons/ops/matrix_exp/__init__.py of the reference package
(file:lines cited per function) so that code written against ``flash_hypercons`` runs
unchanged.  The operators and the autograd formula of ``_matrix_exp`` (the reference's
``_setup_context`` / ``_backward`` / ``_frechet_reference``, __init__.py:32-37,61-77) are
registered in C++ (``csrc/torch_ops.cpp``) and launch the sm_100a kernels of ``libfhx.so``.
"""

from __future__ import annotations

import torch
from torch.overrides import TorchFunctionMode

from ... import _C  # noqa: F401  (registers flash_hypercons::_matrix_exp / _frechet)

_NATIVE = torch.ops.aten.linalg_matrix_exp.default
# The registered overloads, resolved once: a call through the overload packet
# (torch.ops.flash_hypercons._matrix_exp) costs about 0.7 us more per call.
_MATRIX_EXP_OP = torch.ops.flash_hypercons._matrix_exp.default
_MATRIX_EXP_FRECHET_OP = torch.ops.flash_hypercons._matrix_exp_frechet.default
_MATRIX_EXP_AND_GRAD_OP = torch.ops.flash_hypercons._matrix_exp_and_grad.default
_MIX_STREAMS_OP = torch.ops.flash_hypercons._mix_streams.default
_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
_ROUTED = (torch.linalg.matrix_exp, torch.matrix_exp, torch.Tensor.matrix_exp)
_MAX_N = 32
_MIX_MAX_N = 4


def _eligible(input: torch.Tensor) -> bool:
    """Kernel eligibility (reference __init__.py:13-23): a strided NVIDIA CUDA [B, N, N]
    tensor with 2 <= N <= 32 in float32 / float16 / bfloat16."""
    if not isinstance(input, torch.Tensor):
        return False
    if input.device.type != "cuda" or torch.version.hip is not None:
        return False
    if input.layout != torch.strided or input.ndim != 3:
        return False
    n = input.shape[-1]
    return input.shape[-2] == n and 1 < n <= _MAX_N and input.dtype in _DTYPES


def _native(input: torch.Tensor, *, promote: bool = False) -> torch.Tensor:
    """Native PyTorch exponential; CUDA half types are computed in float32 when ``promote``
    (reference __init__.py:26-29)."""
    if promote and input.is_cuda and input.dtype in (torch.float16, torch.bfloat16):
        return _NATIVE(input.float()).to(input.dtype)
    return _NATIVE(input)


def _frechet_reference(input: torch.Tensor, direction: torch.Tensor) -> torch.Tensor:
    """Differentiable L(input, direction): the upper-right block of the native float32
    exponential of [[A, E], [0, A]], cast back (reference __init__.py:32-37).  The C++ backward
    calls it for tensor subclasses that override __torch_function__, so that they see these
    operators."""
    n = input.shape[-1]
    a = input.float()
    e = direction.float()
    block = torch.cat((torch.cat((a, e), -1), torch.cat((torch.zeros_like(a), a), -1)), -2)
    return torch.linalg.matrix_exp(block)[..., :n, n:].to(input.dtype)


@torch.library.register_fake("flash_hypercons::_matrix_exp")
def _matrix_exp_fake(input):
    # Same metadata checks as the reference fake (__init__.py:40-49).
    torch._check(input.device.type == "cuda")
    torch._check(input.layout == torch.strided)
    torch._check(input.ndim == 3)
    torch._check(input.dtype in _DTYPES)
    torch._check(input.shape[-1] == input.shape[-2])
    torch._check(input.shape[-1] > 1)
    torch._check(input.shape[-1] <= _MAX_N)
    return input.new_empty(input.shape)


@torch.library.register_fake("flash_hypercons::_frechet")
def _frechet_fake(input, direction):
    # Reference __init__.py:52-58.
    torch._check(direction.shape == input.shape)
    torch._check(direction.device == input.device)
    torch._check(direction.dtype == input.dtype)
    torch._check(direction.layout == torch.strided)
    return _matrix_exp_fake(input)


@torch.library.register_fake("flash_hypercons::_matrix_exp_frechet")
def _matrix_exp_frechet_fake(input, direction):
    _frechet_fake(input, direction)
    return input.new_empty(input.shape), input.new_empty(input.shape)


@torch.library.register_fake("flash_hypercons::_matrix_exp_and_grad")
def _matrix_exp_and_grad_fake(input, grad):
    _frechet_fake(input, grad)
    return input.new_empty(input.shape), input.new_empty(input.shape)


def _has_tangent(t) -> bool:
    # Outside every forward-AD level no tensor can carry a tangent; unpack_dual would
    # return None, so the (comparatively slow) call is skipped.
    if torch.autograd.forward_ad._current_level < 0:
        return False
    return torch.autograd.forward_ad.unpack_dual(t).tangent is not None


def _jvp_through_kernel(input: torch.Tensor):
    """Forward-mode AD of exp on the kernel: primal exp(A) and tangent L(A, E) from one launch
    of the Frechet kernel (``_matrix_exp_frechet``).  Taken for a plain dual tensor in pure
    forward mode -- neither primal nor tangent needs a reverse-mode graph and no torch.func
    transform is active -- on an eligible input; returns None otherwise (the caller then uses
    native operators, as the reference does for every forward-AD input,
    flash_hypercons/ops/matrix_exp/__init__.py:89-94)."""
    if type(input) is not torch.Tensor or torch._C._are_functorch_transforms_active():
        return None
    primal, tangent = torch.autograd.forward_ad.unpack_dual(input)
    if tangent is None or primal.requires_grad or tangent.requires_grad or not _eligible(primal):
        return None
    if (type(tangent) is not torch.Tensor or tangent._is_zerotensor() or tangent.layout != torch.strided
            or tangent.shape != primal.shape or tangent.dtype != primal.dtype or tangent.device != primal.device):
        return None
    y, ty = _MATRIX_EXP_FRECHET_OP(primal, tangent)
    return torch.autograd.forward_ad.make_dual(y, ty)


def matrix_exp(input: torch.Tensor) -> torch.Tensor:
    """Compute exp(input), accelerating CUDA [B, N, N] tensors with 2 <= N <= 32.

    The CUDA implementation accepts float32, float16, and bfloat16. Other
    inputs use native PyTorch. Forward AD, function transforms, and tensor
    subclasses also use native operations; their CUDA low-precision inputs
    are promoted to float32 for the calculation and cast back on return.
    """
    # Transforms are checked before shape eligibility: vmap can hide batch dimensions
    # (reference __init__.py:88-97).
    if isinstance(input, torch.Tensor) and (
        type(input) not in (torch.Tensor, torch.nn.Parameter)
        or torch._C._are_functorch_transforms_active()
        or _has_tangent(input)
    ):
        # Extension: pure forward-mode AD of a plain tensor runs on the Frechet kernel.
        if _has_tangent(input):
            fused = _jvp_through_kernel(input)
            if fused is not None:
                return fused
        return _native(input, promote=True)
    if not _eligible(input):
        return _native(input)
    return _MATRIX_EXP_OP(input)


def matrix_exp_and_grad(input: torch.Tensor, grad_output: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Forward and backward of ``Y = exp(input)`` in one kernel launch, for a known upstream
    gradient: returns ``(Y, dL/dinput)`` with ``dL/dinput = L(input^T, grad_output)``, the
    gradient ``torch.autograd.grad(matrix_exp(input), input, grad_output)`` computes.

    Eligible inputs (as for ``matrix_exp``) run one launch of the Frechet kernel, which
    carries exp(input^T) through its program anyway and stores it transposed.  The results are
    not attached to an autograd graph.  Other inputs use native PyTorch operators.
    (Extension of this package: the reference has no single call for this.)
    """
    if (isinstance(input, torch.Tensor) and type(input) in (torch.Tensor, torch.nn.Parameter)
            and type(grad_output) is torch.Tensor and _eligible(input)
            and not torch._C._are_functorch_transforms_active()
            and grad_output.shape == input.shape and grad_output.dtype == input.dtype
            and grad_output.device == input.device and grad_output.layout == torch.strided):
        return _MATRIX_EXP_AND_GRAD_OP(input.detach(), grad_output.detach())
    with torch.enable_grad():
        x = input.detach().requires_grad_()
        y = _native(x, promote=True)
        (grad,) = torch.autograd.grad(y, x, grad_output)
    return y.detach(), grad


@torch.library.register_fake("flash_hypercons::_mix_streams")
def _mix_streams_fake(h, streams):
    torch._check(h.device.type == "cuda" and streams.device == h.device)
    torch._check(h.ndim == 3 and streams.ndim == 3)
    torch._check(h.shape[-1] == h.shape[-2])
    torch._check(1 < h.shape[-1] <= _MIX_MAX_N)
    torch._check(streams.shape[0] == h.shape[0] and streams.shape[1] == h.shape[1])
    torch._check(h.dtype in _DTYPES and streams.dtype in _DTYPES)
    return streams.new_empty(streams.shape)


@torch.library.register_fake("flash_hypercons::_mix_streams_backward")
def _mix_streams_backward_fake(h, streams, grad):
    _mix_streams_fake(h, streams)
    torch._check(grad.shape == streams.shape and grad.dtype == streams.dtype)
    return streams.new_empty(streams.shape), h.new_empty(h.shape)


def _mix_eligible(h, streams) -> bool:
    if not (isinstance(h, torch.Tensor) and isinstance(streams, torch.Tensor)):
        return False
    if any(type(t) not in (torch.Tensor, torch.nn.Parameter) for t in (h, streams)):
        return False
    if torch._C._are_functorch_transforms_active() or _has_tangent(h) or _has_tangent(streams):
        return False
    if h.device.type != "cuda" or torch.version.hip is not None or streams.device != h.device:
        return False
    if h.layout != torch.strided or streams.layout != torch.strided or h.ndim != 3 or streams.ndim != 3:
        return False
    n = h.shape[-1]
    return (h.shape[-2] == n and 1 < n <= _MIX_MAX_N and tuple(streams.shape[:2]) == tuple(h.shape[:2])
            and h.dtype in _DTYPES and streams.dtype in _DTYPES)


def mix_streams(h: torch.Tensor, streams: torch.Tensor) -> torch.Tensor:
    """Hyper-connection stream mixing with an exponential mixing matrix: ``exp(h) @ streams``.

    ``h`` is ``[T, n, n]`` (one mixing generator per token, 2 <= n <= 4) and ``streams`` is
    ``[T, n, D]`` (the token's n residual streams).  On CUDA, float32 / float16 / bfloat16, one
    kernel computes exp(h[t]) in registers and applies it to the streams -- the exponential is
    never written to memory -- and the backward is one kernel as well (d streams =
    exp(h)^T dY, d h = the Frechet backward of exp at h for dY streams^T).  The result has the
    streams' dtype; math is float32.  Other inputs, forward AD, function transforms and tensor
    subclasses use native PyTorch (half types computed in float32).
    (Extension of this package: the reference computes exp only.)
    """
    if _mix_eligible(h, streams):
        return _MIX_STREAMS_OP(h, streams)
    dt = torch.promote_types(h.dtype, streams.dtype)
    if dt in (torch.float16, torch.bfloat16):
        dt = torch.float32
    return (torch.linalg.matrix_exp(h.to(dt)) @ streams.to(dt)).to(streams.dtype)


class _MatrixExpMode(TorchFunctionMode):
    """Routes the three Python matrix-exp entry points to ``matrix_exp`` when called with a
    single tensor (positionally or as ``input=``); everything else passes through unchanged
    (reference __init__.py:100-108)."""

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func in _ROUTED:
            if len(args) == 1 and not kwargs:
                return matrix_exp(args[0])
            if not args and set(kwargs) == {"input"}:
                return matrix_exp(kwargs["input"])
        return func(*args, **kwargs)


def use_backend() -> TorchFunctionMode:
    """Route Python matrix-exp calls through flash-hypercons within a with block.

    Scopes nest and restore normal routing on exit, including exceptional exit.
    Enter the scope around calls to compiled functions as well as eager calls.
    Direct ATen/C++ calls are unaffected.
    """
    return _MatrixExpMode()


__all__ = ["matrix_exp", "matrix_exp_and_grad", "mix_streams", "use_backend"]
