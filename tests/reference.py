# Test cases adapted from nickjeliopoulos/flash-hyperconnections (tests/reference.py).
# Copyright (c) 2023-2026 Nicholas John Eliopoulos, Purvish Jatin Jajal.  MIT License; the full
# permission notice is in tests/LICENSE.flash-hyperconnections.
"""Test helpers mirroring the reference's tests/reference.py (float64 ground truth and the
per-matrix error criterion), backed by the CPU oracle in oracle/expm_oracle.py."""

import torch

from oracle import expm_oracle as O


def reference(a, direction=None):
    """float64 exp(a), or L(a, direction) as the upper-right block of exp([[a, d], [0, a]])."""
    if direction is None:
        return O.exp_fp64(a).to(a.device)
    return O.frechet_fp64(a, direction).to(a.device)


def check_error(actual, expected, *, backward=False):
    """max|actual - expected| / (1 + max|expected|) per matrix within the reference tolerances:
    1e-3 / 5e-3 (float32 forward / backward), 5e-2 / 1e-1 (float16, bfloat16)."""
    assert actual.shape == expected.shape
    if not actual.numel():
        return
    assert actual.isfinite().all()
    dtype_name = "float32" if actual.dtype == torch.float32 else "half"
    tol = O.tolerance(dtype_name, backward)
    err = O.per_matrix_error(actual, expected)
    torch.testing.assert_close(err, torch.zeros_like(err), atol=tol, rtol=0)
