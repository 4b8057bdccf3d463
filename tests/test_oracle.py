"""CPU checks of the oracle (oracle/expm_oracle.py) and of the derived constants.

Pins the oracle on the known answers the reference's tests use (exp(0) = I with gradient G,
closed-form rotations, diagonal matrices, identity tangents, finite differences), checks the
generated coefficient header against a fresh derivation, and checks every polynomial scheme
against the truncated Taylor series it must equal."""

import math
import pathlib
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import derive_coefficients as D
from oracle import expm_oracle as O

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_generated_header_is_current():
    res = subprocess.run([sys.executable, str(ROOT / "oracle" / "derive_coefficients.py"), "--check"],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr


def test_thetas_match_published_single_precision_values():
    # Bader-Blanes-Casas 2019 single-precision thresholds (also PyTorch's); theta_18 is the
    # reference's constant (csrc/MatrixExpSmall.cuh:14).
    published = {1: 1.192092800768788e-07, 2: 5.978858893805233e-04, 4: 5.116619363445086e-02,
                 8: 5.800524627688768e-01, 12: 1.461661507209034, 18: 3.010066362817634}
    for m, v in published.items():
        assert O.THETA[m] == pytest.approx(v, rel=1e-12)


def _taylor_poly(a, m):
    out = np.zeros_like(a)
    p = np.broadcast_to(np.eye(a.shape[-1]), a.shape).copy()
    for k in range(m + 1):
        out += p / math.factorial(k)
        p = p @ a
    return out


@pytest.mark.parametrize("m", [1, 2, 4, 8, 12, 18])
def test_schemes_equal_truncated_taylor(m):
    rng = np.random.default_rng(m)
    a = rng.standard_normal((16, 6, 6))
    a *= (O.THETA[m] / np.abs(a).sum(-2).max(-1))[:, None, None]
    eye = np.eye(6)
    got = np.stack([O._taylor(m, (x, None), eye)[0] for x in a])
    ref = _taylor_poly(a, m)
    assert np.abs(got - ref).max() <= 1e-13 * np.abs(ref).max()


@pytest.mark.parametrize("m", [2, 4, 8, 12, 18])
def test_pair_schemes_equal_block_taylor(m):
    # The pair (derivative) evaluation equals the upper-right block of T_m([[A, E], [0, A]]).
    rng = np.random.default_rng(100 + m)
    n = 5
    a = rng.standard_normal((8, n, n)) * 0.2
    e = rng.standard_normal((8, n, n))
    eye = np.eye(n)
    got = np.stack([O._taylor(m, (x, y), eye)[1] for x, y in zip(a, e)])
    block = np.zeros((8, 2 * n, 2 * n))
    block[:, :n, :n] = a
    block[:, n:, n:] = a
    block[:, :n, n:] = e
    ref = _taylor_poly(block, m)[:, :n, n:]
    assert np.abs(got - ref).max() <= 1e-12 * max(1.0, np.abs(ref).max())


def test_t8_t12_t18_polynomials_exact():
    thetas, t8, t12, t18 = D.derive()
    for poly, m in ((D.t8_polynomial(t8), 8), (D.t12_polynomial(t12), 12), (D.t18_polynomial(t18), 18)):
        rel, tail = D.scheme_residual(poly, m)
        assert rel < 1e-30 and tail == 0
    # T1, T2, T4, T8 in the T12 structure (one evaluation path for every m <= 12)
    for m in (1, 2, 4, 8):
        rel, tail = D.scheme_residual(D.t12_polynomial(D.t12_structure_rows(m)), m)
        assert rel < 1e-30 and tail == 0
    # The refined T18 solution stays within 1e-10 of the published BBC-2019 digits.
    for r in range(5):
        for c in range(5):
            pub = D.T18_PUBLISHED[r][c]
            assert abs(float(t18[r][c]) - pub) <= 1e-10 * max(abs(pub), 1e-30)


@pytest.mark.parametrize("m", [1, 2, 4, 8, 12])
def test_unified_structure_equals_truncated_taylor(m):
    # the float header rows (t12u) evaluate T_m to round-off in float64, value and pair parts
    rng = np.random.default_rng(300 + m)
    n = 4
    a = rng.standard_normal((8, n, n)) * 0.2
    e = rng.standard_normal((8, n, n))
    eye = np.eye(n)
    got = np.stack([O._taylor_unified(m, (x, y), eye)[1] for x, y in zip(a, e)])
    got_d = np.stack([O._taylor_unified(m, (x, None), eye)[0] for x in a])
    block = np.zeros((8, 2 * n, 2 * n))
    block[:, :n, :n] = a
    block[:, n:, n:] = a
    block[:, :n, n:] = e
    ref = _taylor_poly(block, m)
    assert np.abs(got - ref[:, :n, n:]).max() <= 1e-6 * max(1.0, np.abs(ref).max())
    assert np.abs(got_d - ref[:, :n, :n]).max() <= 1e-6 * max(1.0, np.abs(ref).max())


def test_choose_degree_boundaries():
    for m in (1, 2, 4, 8, 12, 18):
        assert O.choose_degree(O.THETA[m]) == (m, 0)
    t = O.THETA[18]
    assert O.choose_degree(t * (1 + 1e-12)) == (18, 1)
    assert O.choose_degree(2 * t) == (18, 1)
    assert O.choose_degree(2 * t * (1 + 1e-12)) == (18, 2)
    assert O.choose_degree(0.0) == (1, 0)


@pytest.mark.parametrize("n", [2, 3, 4, 8, 13, 32])
def test_adaptive_float64_matches_exp(n):
    rng = np.random.default_rng(n)
    a = rng.standard_normal((48, n, n)) / np.sqrt(n) * 10 ** rng.uniform(-4, 1.2, (48, 1, 1))
    e = rng.standard_normal((48, n, n))
    _, per = O.rel_frobenius(O.adaptive_algorithm(a), O.exp_fp64(a))
    assert per.max() < 5e-7
    _, per = O.rel_frobenius(O.adaptive_algorithm(a, e), O.frechet_fp64(a, e))
    assert per.max() < 5e-6


@pytest.mark.parametrize("n", [4, 16, 32])
def test_reference_algorithm_float32_error_level(n):
    rng = np.random.default_rng(7 + n)
    a = rng.standard_normal((32, n, n)) * 0.3
    e = rng.standard_normal((32, n, n))
    glob, _ = O.rel_frobenius(O.reference_algorithm(a), O.exp_fp64(a))
    assert glob < 1e-5
    glob, _ = O.rel_frobenius(O.reference_algorithm(a, e), O.frechet_fp64(a, e))
    assert glob < 1e-5


@pytest.mark.parametrize("algo", ["reference", "adaptive"])
def test_known_answers(algo):
    run = O.reference_algorithm if algo == "reference" else (lambda a, e=None: O.adaptive_algorithm(a, e, np.float32))
    n = 6
    zero = np.zeros((2, n, n))
    g = np.random.default_rng(0).standard_normal((2, n, n))
    np.testing.assert_allclose(run(zero), np.broadcast_to(np.eye(n), zero.shape), atol=0)
    np.testing.assert_allclose(run(zero, g), g.astype(np.float32), atol=1e-7)
    # Rotations exp([[0, -t], [t, 0]]) (reference tests/test_matrix_exp.py:107-129).
    for angle in (0.5, 25.0, 100.0):
        r = np.zeros((1, n, n))
        r[0, 0, 1], r[0, 1, 0] = -angle, angle
        y = run(r)[0]
        assert abs(y[0, 0] - math.cos(angle)) < 2e-3 and abs(y[1, 0] - math.sin(angle)) < 2e-3
        assert abs(y[2, 2] - 1) < 1e-6
    # Diagonal matrices (reference tests/test_integration.py:75-83).
    d = np.linspace(-0.2, 0.2, n)
    y = run(np.diag(d)[None])[0]
    np.testing.assert_allclose(np.diag(y), np.exp(d), rtol=1e-6)
    # Identity tangent at zero: L(0, I) = I (reference tests/test_integration.py:59-69).
    np.testing.assert_allclose(run(zero[:1], np.eye(n)[None])[0], np.eye(n), atol=1e-7)


def test_nonfinite_rows_make_whole_matrix_nan():
    a = np.zeros((3, 4, 4))
    a[0, 1, 2] = np.nan
    a[1, 0, 0] = np.inf
    for run in (O.reference_algorithm, lambda x, e=None: O.adaptive_algorithm(x, e, np.float32)):
        y = run(a)
        assert np.isnan(y[0]).all() and np.isnan(y[1]).all() and np.isfinite(y[2]).all()


def test_finite_difference_of_frechet():
    rng = np.random.default_rng(3)
    a = rng.standard_normal((4, 7, 7)) * 0.4
    e = rng.standard_normal((4, 7, 7))
    h = 1e-6
    fd = (O.exp_fp64(a + h * e) - O.exp_fp64(a - h * e)).numpy() / (2 * h)
    np.testing.assert_allclose(O.frechet_fp64(a, e).numpy(), fd, atol=1e-7)
    np.testing.assert_allclose(O.adaptive_algorithm(a, e), fd, atol=5e-6)


def test_algorithmic_flops_counts():
    a = np.zeros((3, 4, 4))  # m = 1, s = 0 -> no products
    assert O.algorithmic_flops(a) == 0.0
    big = np.eye(4)[None] * 10.0  # nu = 10 -> m = 18, s = 2
    m, s = O.degree_choices(big)
    assert (int(m[0]), int(s[0])) == (18, 2)
    assert O.algorithmic_flops(big) == 8 * 64 * 7


def test_workload_generation_is_shard_invariant():
    from flash_hyperconnections_b200 import workloads as W

    cfg = W.CONFIGS[3]
    full, gfull = W.generate(cfg, 0, 2 * W.CHUNK)
    part, gpart = W.generate(cfg, W.CHUNK, W.CHUNK)
    assert torch.equal(full[W.CHUNK:], part) and torch.equal(gfull[W.CHUNK:], gpart)
    assert not full.is_contiguous() and full.mT.is_contiguous()
    assert W.shard(W.CONFIGS[5], 3, 8) == (3 * 131072, 131072)
