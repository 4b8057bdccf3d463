"""Algorithmic work of the exponential as the kernels' selection rule mandates it, for roofline
reporting.  Mirrors csrc/expm_common.cuh (choose_degree) with vectorised torch ops so that it
can run on the device over a full benchmark batch.

Per matrix of kernel size P (n padded to 4 / 8 / 16 / 32 for n > 4, n itself for n <= 4):
  forward            2 P^3 (pi(m) + s)  flops
  Frechet backward   6 P^3 (pi(m) + s)  flops   (three products per structured product)
pi(m) = 0, 1, 2, 3, 4, 5 products for m = 1, 2, 4, 8, 12, 18.  O(P^2) combination terms are
not counted.  Algorithmic bytes per matrix: read A and write Y (forward); read A and G and
write the gradient (backward): 5 n^2 elements.
"""

from __future__ import annotations

import torch

THETA = {
    1: 1.1920928007687876534e-07,
    2: 0.00059788588938052333158,
    4: 0.051166193634450861736,
    8: 0.58005246276887680854,
    12: 1.4616615072090336099,
    18: 3.0100663628176353719,
}
PRODUCTS = {1: 0, 2: 1, 4: 2, 8: 3, 12: 4, 18: 5}


def kernel_size(n: int) -> int:
    if n <= 4:
        return n
    return 8 if n <= 8 else 16 if n <= 16 else 32


def mandated_steps(a: torch.Tensor, chunk: int = 65536) -> torch.Tensor:
    """pi(m) + s per matrix for a [B, n, n] tensor (any device), computed in float64."""
    out = []
    for lo in range(0, a.shape[0], chunk):
        x = a[lo : lo + chunk].abs().double()
        nu = torch.minimum(x.sum(-2).amax(-1), x.sum(-1).amax(-1))
        steps = torch.full_like(nu, PRODUCTS[18], dtype=torch.int64)
        for m in (12, 8, 4, 2, 1):
            steps = torch.where(nu <= THETA[m], torch.full_like(steps, PRODUCTS[m]), steps)
        ratio = nu / THETA[18]
        mant, expo = torch.frexp(ratio)
        s = torch.where(mant == 0.5, expo - 1, expo).to(torch.int64)
        s = torch.where(nu > THETA[18], s, torch.zeros_like(s))
        out.append(steps + s)
    return torch.cat(out)


def algorithmic_flops(a: torch.Tensor, forward: bool = True, backward: bool = True) -> float:
    p = kernel_size(a.shape[-1])
    per = (2.0 if forward else 0.0) + (6.0 if backward else 0.0)
    return float(per * p**3 * mandated_steps(a).sum().item())


def algorithmic_bytes(batch: int, n: int, elem_bytes: int, forward: bool = True, backward: bool = True) -> float:
    elems = (2 if forward else 0) + (3 if backward else 0)
    return float(elems * batch * n * n * elem_bytes)
