"""The CPU oracle pinned against the reference's own kernels (golden vectors).

tests/golden/reference_kernels.npz holds inputs and the outputs of the reference's CUDA operators
(built from its sources and run on a GPU by tests/golden/make_golden.py): Y = exp(A) and
L = L(A, E) for n = 2..32 in float32, bfloat16 and float16.  On the CPU:

* the oracle's restatement of the reference algorithm (fixed degree 18, s from the column sums
  of |A| (+ |E|), float32 arithmetic) reproduces them to float32 rounding;
* the float64 ground truth agrees with them within the reference's own per-matrix tolerance.
"""

import pathlib

import numpy as np
import pytest
import torch

from oracle import expm_oracle as O

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "reference_kernels.npz"
SIZES = (2, 3, 4, 5, 8, 11, 16, 23, 32)
DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _cast(x, name):
    return torch.from_numpy(np.asarray(x, dtype=np.float64)).to(DTYPES[name]).double().numpy()


@pytest.mark.parametrize("name", list(DTYPES))
@pytest.mark.parametrize("n", SIZES)
def test_reference_restatement_matches_reference_kernels(golden, n, name):
    key = f"n{n}_{name}"
    a, e, y, l = (golden[f"{key}_{t}"] for t in "AEYL")
    ours_y = _cast(O.reference_algorithm(a), name)
    ours_l = _cast(O.reference_algorithm(a, e), name)
    # float32 rounding of a few products; for half outputs, one rounding step of the output type
    tol = 2e-5 if name == "float32" else (1e-2 if name == "bfloat16" else 2e-3)
    assert O.per_matrix_error(ours_y, y).max() <= tol
    assert O.per_matrix_error(ours_l, l).max() <= tol


@pytest.mark.parametrize("name", list(DTYPES))
@pytest.mark.parametrize("n", SIZES)
def test_float64_truth_against_reference_kernels(golden, n, name):
    key = f"n{n}_{name}"
    a, e, y, l = (golden[f"{key}_{t}"] for t in "AEYL")
    kind = "float32" if name == "float32" else "half"
    assert O.per_matrix_error(y, O.exp_fp64(a)).max() <= O.tolerance(kind, False)
    assert O.per_matrix_error(l, O.frechet_fp64(a, e)).max() <= O.tolerance(kind, True)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(DTYPES))
@pytest.mark.parametrize("n", SIZES)
def test_kernels_against_reference_kernels(golden, n, name):
    """This package's operators on the golden inputs agree with the reference kernels' outputs
    within the reference's per-matrix tolerance."""
    import flash_hypercons  # noqa: F401  (registers the operators)

    key = f"n{n}_{name}"
    a, e, y, l = (golden[f"{key}_{t}"] for t in "AEYL")
    at = torch.from_numpy(a).to(DTYPES[name]).cuda()
    et = torch.from_numpy(e).to(DTYPES[name]).cuda()
    ours_y = torch.ops.flash_hypercons._matrix_exp(at).float().cpu().numpy()
    ours_l = torch.ops.flash_hypercons._frechet(at, et).float().cpu().numpy()
    kind = "float32" if name == "float32" else "half"
    assert O.per_matrix_error(ours_y, y).max() <= O.tolerance(kind, False)
    assert O.per_matrix_error(ours_l, l).max() <= O.tolerance(kind, True)
