"""The reference package's CPU path, timed as the CPU baseline.

TEST / BENCHMARK INFRASTRUCTURE ONLY (bench.py's CPU-baseline leg and ``--impl reference``).

On a CPU tensor ``flash_hypercons.matrix_exp`` routes to native PyTorch
(flash_hypercons/ops/matrix_exp/__init__.py:95-96 -> ``_native`` :26-29), and its backward is
native autograd of ``torch.linalg.matrix_exp``.  Low-precision inputs are computed in float32
and cast back, as the reference benchmark does for the stock path
(benchmarks/matrix_exp.py:30-33).
"""

from __future__ import annotations

import time

import torch


def fwd_bwd(a: torch.Tensor, g: torch.Tensor):
    low = a.dtype in (torch.float16, torch.bfloat16)
    x = (a.float() if low else a).detach().requires_grad_()
    y = torch.linalg.matrix_exp(x)
    (grad,) = torch.autograd.grad(y, x, g.float() if low else g)
    if low:
        return y.detach().to(a.dtype), grad.to(a.dtype)
    return y.detach(), grad


def time_fwd_bwd(a: torch.Tensor, g: torch.Tensor, repeat: int = 1) -> float:
    """Seconds per fwd+bwd call over ``repeat`` calls (wall clock, host cores)."""
    t0 = time.perf_counter()
    for _ in range(repeat):
        fwd_bwd(a, g)
    return (time.perf_counter() - t0) / repeat
