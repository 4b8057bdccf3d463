"""CPU oracle for the batched small-matrix exponential and its Frechet derivative.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may use this module, and only as the checker -- never as the measured or shipped
path.

Three restatements live here:

1. ``exp_fp64`` / ``frechet_fp64`` -- the ground truth used by the reference's own tests
   (tests/reference.py:4-11 of flash_hypercons): native float64 ``torch.linalg.matrix_exp``,
   and for the derivative the upper-right block of exp([[A, E], [0, A]]) in float64.
   ``check_error`` restates the reference's per-matrix metric and tolerances
   (tests/reference.py:14-22); ``rel_frobenius`` is the relative Frobenius error the
   north-star tolerance is stated in.
2. ``reference_algorithm`` -- a numpy restatement of the reference kernels' arithmetic
   (csrc/MatrixExpSmall.cuh): fixed degree-18 BBC polynomial (:83-106), scaling exponent
   s = ceil(log2(||.||_1 / theta_18)) from the float64 column sums of |A| (+|E| for the
   derivative) (:141-157, :332-361), s squarings (:164-169), structured pair products
   (:22-52), whole-matrix NaN on a non-finite entry (:127-140).
3. ``adaptive_algorithm`` / ``choose_degree`` -- a numpy restatement of THIS project's kernel
   algorithm (flash_hyperconnections_b200/csrc): (m, s) from nu = min(||A||_1, ||A||_inf) and the
   theta table, the BBC schemes for m in {1, 2, 4, 8, 12, 18}, s squarings.  Run in float64
   it must agree with (1) to ~1e-13, which pins the scheme coefficients and the selection
   logic; ``algorithmic_flops`` counts the work the selection mandates.

Pinning: tests/test_oracle.py checks (1)-(3) against the known answers the reference's tests
use (exp(0) = I with gradient G, closed-form rotations, diagonal matrices, identity tangents,
finite differences) and against golden vectors under tests/golden/.
"""

from __future__ import annotations

import math
import pathlib
import re

import numpy as np

_COEFF_HEADER = pathlib.Path(__file__).resolve().parents[1] / "flash_hyperconnections_b200" / "csrc" / "expm_coeffs.h"
DEGREES = (1, 2, 4, 8, 12, 18)
PRODUCTS = {1: 0, 2: 1, 4: 2, 8: 3, 12: 4, 18: 5}


def _load_coefficients():
    text = _COEFF_HEADER.read_text()
    theta = {int(m): float(v) for m, v in re.findall(r"kTheta(\d+) = ([0-9.eE+-]+);", text)}
    t8 = {k.lower(): float(v) for k, v in re.findall(r"kT8(\w+) = ([0-9.eE+-]+)f;", text)}

    def table(name, rows):
        block = text.split(f"constexpr float {name}(int r, int c)")[1].split("return")[0]
        vals = [float(v) for v in re.findall(r"(-?[0-9.]+(?:[eE][+-]?[0-9]+)?)f", block)]
        return np.array(vals).reshape(rows, -1)

    block = text.split("constexpr float t12u(int d, int r, int c)")[1].split("return")[0]
    t12u = np.array([float(v) for v in re.findall(r"(-?[0-9.]+(?:[eE][+-]?[0-9]+)?)f", block)]).reshape(5, 4, 4)
    return theta, t8, table("t12c", 4), table("t18c", 5), t12u


THETA, T8, T12, T18, T12U = _load_coefficients()


# --------------------------------------------------------------------------------------
# (1) Ground truth and metrics
# --------------------------------------------------------------------------------------
def exp_fp64(a):
    """float64 torch.linalg.matrix_exp on CPU (reference tests/reference.py:4-7)."""
    import torch

    return torch.linalg.matrix_exp(torch.as_tensor(a).detach().cpu().double())


def frechet_fp64(a, e):
    """L(A, E) as the upper-right block of exp([[A, E], [0, A]]) in float64
    (reference tests/reference.py:8-11)."""
    import torch

    a = torch.as_tensor(a).detach().cpu().double()
    e = torch.as_tensor(e).detach().cpu().double()
    n = a.shape[-1]
    block = torch.cat((torch.cat((a, e), -1), torch.cat((torch.zeros_like(a), a), -1)), -2)
    return torch.linalg.matrix_exp(block)[..., :n, n:]


def tolerance(dtype_name: str, backward: bool) -> float:
    """Per-matrix max-error tolerance of the reference tests (tests/reference.py:19)."""
    if dtype_name == "float32":
        return 0.005 if backward else 0.001
    return 0.1 if backward else 0.05


def per_matrix_error(actual, expected):
    """max|actual - expected| / (1 + max|expected|) per matrix (tests/reference.py:20-21)."""
    import torch

    actual = torch.as_tensor(actual).detach().cpu().double()
    expected = torch.as_tensor(expected).detach().cpu().double()
    delta = (actual - expected).abs().flatten(-2).amax(-1)
    scale = 1 + expected.abs().flatten(-2).amax(-1)
    return delta / scale


def rel_frobenius(actual, expected):
    """(batch-global, per-matrix) relative Frobenius error against a float64 reference."""
    import torch

    actual = torch.as_tensor(actual).detach().cpu().double()
    expected = torch.as_tensor(expected).detach().cpu().double()
    diff = (actual - expected).flatten(-2)
    ref = expected.flatten(-2)
    per = diff.norm(dim=-1) / ref.norm(dim=-1).clamp_min(1e-300)
    glob = diff.norm() / ref.norm().clamp_min(1e-300)
    return float(glob), per


# --------------------------------------------------------------------------------------
# (2) The reference kernels' algorithm (csrc/MatrixExpSmall.cuh)
# --------------------------------------------------------------------------------------
_THETA18_REF = 3.010066362817634  # MatrixExpSmall.cuh:14


def _pair_mul(x, y):
    """(Xd, Xu)(Yd, Yu) = (Xd Yd, Xd Yu + Xu Yd) (MatrixExpSmall.cuh:22-52)."""
    xd, xu = x
    yd, yu = y
    return (xd @ yd, None if xu is None else xd @ yu + xu @ yd)


def _pair_lin(coeffs, mats, eye):
    """c0 I + sum c_k M_k on pairs; the identity term has no derivative part (:66-81)."""
    d = coeffs[0] * eye
    u = None if mats[0][1] is None else np.zeros_like(mats[0][1])
    for c, (md, mu) in zip(coeffs[1:], mats):
        d = d + c * md
        if u is not None:
            u = u + c * mu
    return (d, u)


def _pair_add(x, y):
    return (x[0] + y[0], None if x[1] is None else x[1] + y[1])


def _t18(a, eye):
    """Degree-18 BBC polynomial in five products (MatrixExpSmall.cuh:83-106)."""
    a2 = _pair_mul(a, a)
    a3 = _pair_mul(a2, a)
    a6 = _pair_mul(a3, a3)
    basis = [a, a2, a3, a6]
    b = [_pair_lin(T18[r], basis, eye) for r in range(5)]
    a9 = _pair_add(_pair_mul(b[0], b[4]), b[3])
    return _pair_add(b[1], _pair_mul(_pair_add(b[2], a9), a9))


def reference_algorithm(a, e=None, dtype=np.float32):
    """Restatement of the reference kernels: exp(A) (e is None) or L(A, E), in ``dtype``."""
    a = np.asarray(a, dtype=np.float64)
    batch, n, _ = a.shape
    out = np.empty((batch, n, n), dtype=np.float64)
    eye = np.eye(n, dtype=dtype)
    for b in range(batch):
        x = a[b].astype(dtype)
        y = None if e is None else np.asarray(e[b]).astype(dtype)
        if not np.isfinite(x).all() or (y is not None and not np.isfinite(y).all()):
            out[b] = np.nan
            continue
        col = np.abs(x.astype(np.float64)).sum(0)
        if y is not None:
            col = col + np.abs(y.astype(np.float64)).sum(0)
        norm = col.max()
        s = int(math.ceil(math.log2(norm / _THETA18_REF))) if norm > _THETA18_REF else 0
        scale = dtype(2.0**-s)
        pair = (x * scale, None if y is None else y * scale)
        r = _t18(pair, eye)
        for _ in range(s):
            r = _pair_mul(r, r)
        out[b] = r[0] if y is None else r[1]
    return out


# --------------------------------------------------------------------------------------
# (3) This project's adaptive algorithm (flash_hyperconnections_b200/csrc/expm_*.cuh)
# --------------------------------------------------------------------------------------
def choose_degree(nu: float):
    """(m, s): smallest m with nu <= theta_m, else m = 18 and s = ceil(log2(nu/theta_18)),
    computed exactly through frexp (csrc/expm_common.cuh: choose_degree)."""
    for m in DEGREES:
        if nu <= THETA[m]:
            return m, 0
    f, e = math.frexp(nu / THETA[18])
    return 18, (e - 1 if f == 0.5 else e)


def selection_norm(a) -> np.ndarray:
    """nu = min(||A||_1, ||A||_inf) per matrix, float64 sums of the float32 values."""
    x = np.abs(np.asarray(a, dtype=np.float32).astype(np.float64))
    return np.minimum(x.sum(-2).max(-1), x.sum(-1).max(-1))


def _taylor_unified(m, a, eye):
    """The n <= 4 kernel's evaluation (csrc/expm_reg.cuh: taylor): every m <= 12 in the
    four-product structure of T12 with its own B1..B4 rows (expm_coeffs.h: t12u), T18 as usual."""
    if m == 18:
        return _t18(a, eye)
    a2 = _pair_mul(a, a)
    a3 = _pair_mul(a2, a)
    rows = T12U[(1, 2, 4, 8, 12).index(m)]
    b1, b2, b3, b4 = (_pair_lin(rows[r], [a, a2, a3], eye) for r in range(4))
    a6 = _pair_add(_pair_mul(b4, b4), b3)
    return _pair_add(_pair_mul(_pair_add(b2, a6), a6), b1)


def _taylor(m, a, eye):
    if m == 1:
        return _pair_lin([1.0, 1.0], [a], eye)
    a2 = _pair_mul(a, a)
    if m == 2:
        return _pair_lin([1.0, 1.0, 0.5], [a, a2], eye)
    if m == 4:
        c = _pair_lin([0.5, 1 / 6, 1 / 24], [a, a2], eye)
        return _pair_add(_pair_mul(a2, c), _pair_lin([1.0, 1.0], [a], eye))
    if m == 8:
        c1 = _pair_lin([0.0, T8["x1"], T8["x2"]], [a, a2], eye)
        a4 = _pair_mul(a2, c1)
        left = _pair_lin([0.0, T8["x3"], 1.0], [a2, a4], eye)
        right = _pair_lin([T8["x4"], T8["x5"], T8["x6"], T8["x7"]], [a, a2, a4], eye)
        return _pair_add(_pair_mul(left, right), _pair_lin([1.0, 1.0, T8["y2"]], [a, a2], eye))
    a3 = _pair_mul(a2, a)
    if m == 12:
        basis = [a, a2, a3]
        b1, b2, b3, b4 = (_pair_lin(T12[r], basis, eye) for r in range(4))
        a6 = _pair_add(_pair_mul(b4, b4), b3)
        return _pair_add(_pair_mul(_pair_add(b2, a6), a6), b1)
    return _t18(a, eye)


def adaptive_algorithm(a, e=None, dtype=np.float64, unified=None):
    """Restatement of the kernels' algorithm: exp(A) or L(A, E) in ``dtype`` arithmetic.
    ``unified`` (default: n <= 4, as the kernels) evaluates degrees m <= 12 in the T12 structure."""
    a = np.asarray(a, dtype=np.float64)
    batch, n, _ = a.shape
    out = np.empty((batch, n, n), dtype=np.float64)
    eye = np.eye(n, dtype=dtype)
    nus = selection_norm(a)
    taylor = _taylor_unified if (n <= 4 if unified is None else unified) else _taylor
    for b in range(batch):
        x = a[b].astype(dtype)
        y = None if e is None else np.asarray(e[b], dtype=np.float64).astype(dtype)
        if not np.isfinite(x).all() or (y is not None and not np.isfinite(y).all()):
            out[b] = np.nan
            continue
        m, s = choose_degree(float(nus[b]))
        pair = (np.ldexp(x, -s).astype(dtype), None if y is None else np.ldexp(y, -s).astype(dtype))
        r = taylor(m, pair, eye)
        for _ in range(s):
            r = _pair_mul(r, r)
        out[b] = r[0] if y is None else r[1]
    return out


def degree_choices(a):
    """Per-matrix (m, s) arrays of the adaptive selection."""
    nus = selection_norm(a)
    ms = np.array([choose_degree(float(v)) for v in nus], dtype=np.int64).reshape(-1, 2)
    return ms[:, 0], ms[:, 1]


def algorithmic_flops(a, pad_to=None, forward=True, backward=True):
    """Matrix-product flops the selection mandates: 2 P^3 (pi(m) + s) for the forward and
    6 P^3 (pi(m) + s) for the structured Frechet backward, P the (padded) kernel size.
    O(P^2) combination terms are not counted."""
    m, s = degree_choices(a)
    steps = np.array([PRODUCTS[int(v)] for v in m]) + s
    p = pad_to or np.asarray(a).shape[-1]
    per = (2.0 if forward else 0.0) + (6.0 if backward else 0.0)
    return float(per * p**3 * steps.sum())
