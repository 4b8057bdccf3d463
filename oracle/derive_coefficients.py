"""Derive the Taylor-degree thresholds and polynomial-scheme coefficients used by the kernels.

TEST INFRASTRUCTURE / BUILD STEP — not part of the product path.  It regenerates
``flash_hyperconnections_b200/csrc/expm_coeffs.h`` and is re-run by the CPU test-suite to
check that the committed header still matches the mathematics.

What is derived (Bader, Blanes, Casas 2019, "Computing the matrix exponential with an
optimized Taylor polynomial approximation", Mathematics 7(12):1174):

* theta_m for m in {1, 2, 4, 8, 12, 18}: the largest ||A|| for which the truncated Taylor
  polynomial T_m satisfies T_m(A) = exp(A + dA) with ||dA|| / ||A|| <= u = 2^-24.  With
  h_m(x) = log(exp(-x) T_m(x)) = sum_{k>m} c_k x^k, the bound is sum_k |c_k| theta^(k-1) <= u,
  solved by bisection in 50-digit arithmetic.  The reference selects only between theta_18
  and squarings (csrc/MatrixExpSmall.cuh:14,154); the full table drives the adaptive degree.
* T8 in three products (closed form of the coefficient-matching system with x3 = 2/3).
* T12 in four products: A6 = B3 + B4*B4, T12 = B1 + (B2 + A6)*A6 with B1..B4 cubic in A.
  The 13 matching equations in 16 unknowns leave a 3-parameter family; we fix B4(0) = 0,
  B3(0) = 0, B2(0) = 6 and refine the real root found by a float search (see
  ``T12_START``) to 40 digits.  Any member of the family is exactly T12 in exact arithmetic;
  this member was picked for the smallest float32 evaluation error at ||A||_1 = theta_12.
* T1, T2, T4 and T8 in the four-product structure of T12 (same B1..B4 layout), so that one
  evaluation path serves every degree m <= 12 (the n <= 4 kernel keeps its lanes on one
  program whatever degree each matrix picked): T_m = B1 + (B2 + A6) A6 with A6 = a A^(m/2)
  (B4 = sqrt(a) A^(m/4), B3 = 0), a = 1/sqrt(m!), B2 = sum_{k=m/2}^{m-1} A^(k-m/2) / (k! a) and
  B1 = sum_{k<m/2} A^k / k! for m = 4, 8; B1 = T_m itself for m = 1, 2.  Exact in exact
  arithmetic (A6^2 = A^m / m!).
* T18 in five products: A9 = B1 B5 + B4, T18 = B2 + (B3 + A9) A9 with B1..B5 combinations
  of (I, A, A2, A3, A6).  The 19 matching equations in 20 unknowns are solved by Newton's
  method in 50-digit arithmetic, seeded with the BBC-2019 published solution (their eq.
  (16)-(17); the same 17-digit numbers appear in the reference at
  csrc/MatrixExpSmall.cuh:89-103) and with the B1 coefficient of A held fixed.  The refined
  solution differs from the published digits by < 1e-11 relative and reproduces T18 to
  1e-45.
"""

from __future__ import annotations

import argparse
import pathlib

import mpmath as mp

mp.mp.dps = 50
U = mp.mpf(2) ** -24
DEGREES = (1, 2, 4, 8, 12, 18)
# Float search result for (p1, p2, p3, c1, c2, c3) of the T12 family with c0 = 6, p0 = 0.
T12_C0 = 6
T12_START = (0.11598307, 0.10541606, 0.01026131, 1.07735774, 0.02274073, 0.01347155)
# BBC 2019 degree-18 scheme: rows B1..B5, columns the coefficients of (I, A, A^2, A^3, A^6).
T18_PUBLISHED = (
    (0.0, -0.10036558103014462, -0.008029246482411570, -0.000892138498045730, 0.0),
    (0.0, 0.39784974949645076, 1.36783778460411719, 0.49828962252538268, -0.00063789819459247233),
    (-10.96763960529620626, 1.68015813878906197, 0.05717798464788655, -0.00698210122488052, 3.349750170860705e-05),
    (-0.09043168323908106, -0.06764045190713819, 0.06759613017740597, 0.02955525704293155, -1.391802575160607e-05),
    (0.0, 0.0, -0.09233646193671186, -0.01693649390020817, -1.400867981820361e-05),
)

HEADER = pathlib.Path(__file__).resolve().parents[1] / "flash_hyperconnections_b200" / "csrc" / "expm_coeffs.h"


def _fact(k):
    return 1 / mp.factorial(k)


def _pmul(a, b):
    r = [mp.mpf(0)] * (len(a) + len(b) - 1)
    for i, x in enumerate(a):
        for j, y in enumerate(b):
            r[i + j] += x * y
    return r


def _padd(*ps):
    n = max(len(p) for p in ps)
    return [mp.fsum((p[i] if i < len(p) else 0) for p in ps) for i in range(n)]


def backward_error_series(m: int, terms: int = 60):
    """Coefficients c_k of h_m(x) = log(exp(-x) T_m(x)) up to x^(m+terms)."""
    k_max = m + terms
    en = [(-1) ** k * _fact(k) for k in range(k_max + 1)]
    t = [_fact(k) for k in range(m + 1)] + [mp.mpf(0)] * (k_max - m)
    f = [mp.fsum(en[i] * t[k - i] for i in range(k + 1)) for k in range(k_max + 1)]
    g = f[:]
    g[0] = mp.mpf(0)
    out = [mp.mpf(0)] * (k_max + 1)
    power = [mp.mpf(1)] + [mp.mpf(0)] * k_max
    for j in range(1, k_max + 1):
        power = _pmul(power, g)[: k_max + 1]
        if all(abs(x) < mp.mpf(10) ** -(mp.mp.dps - 5) for x in power):
            break
        for k in range(k_max + 1):
            out[k] += (-1) ** (j + 1) * power[k] / j
    return out


def theta(m: int):
    c = backward_error_series(m)

    def bound(x):
        return mp.fsum(abs(c[k]) * x ** (k - 1) for k in range(m + 1, len(c)))

    lo, hi = mp.mpf(0), mp.mpf(10)
    for _ in range(180):
        mid = (lo + hi) / 2
        if bound(mid) <= U:
            lo = mid
        else:
            hi = mid
    return lo


def t8_coefficients():
    """x1..x7, y0..y2 of A4 = A2 (x1 A + x2 A2); A8 = (x3 A2 + A4)(x4 I + x5 A + x6 A2 + x7 A4);
    T8 = y0 I + y1 A + y2 A2 + A8."""
    r = mp.sqrt(177)
    x3 = mp.mpf(2) / 3
    return {
        "x1": x3 * (1 + r) / 88,
        "x2": x3 * (1 + r) / 352,
        "x3": x3,
        "x4": (-271 + 29 * r) / (315 * x3),
        "x5": 11 * (-1 + r) / (1260 * x3),
        "x6": 11 * (-9 + r) / (5040 * x3),
        "x7": (89 - r) / (5040 * x3**2),
        "y0": mp.mpf(1),
        "y1": mp.mpf(1),
        "y2": (857 - 58 * r) / 630,
    }


def t8_polynomial(c):
    a4 = [0, 0, 0, c["x1"], c["x2"]]
    left = _padd([0, 0, c["x3"]], a4)
    right = _padd([c["x4"], c["x5"], c["x6"]], [c["x7"] * v for v in a4])
    return _padd([c["y0"], c["y1"], c["y2"]], _pmul(left, right))


def t12_coefficients():
    """Rows B1..B4 of the T12 scheme, each the coefficients of (I, A, A2, A3)."""
    p6 = mp.sqrt(_fact(12))
    p5 = _fact(11) / (2 * p6)
    p4 = (_fact(10) - p5 * p5) / (2 * p6)
    c0 = mp.mpf(T12_C0)

    def equations(p1, p2, p3, c1, c2, c3):
        p = [mp.mpf(0), p1, p2, p3, p4, p5, p6]
        c = [c0, c1, c2, c3]
        t = _padd(_pmul(c, p), _pmul(p, p))
        return [t[k] - _fact(k) for k in range(4, 10)]

    p1, p2, p3, c1, c2, c3 = mp.findroot(equations, [mp.mpf(x) for x in T12_START], tol=mp.mpf(10) ** -45)
    q3 = mp.sqrt(p6)
    q2 = p5 / (2 * q3)
    q1 = (p4 - q2 * q2) / (2 * q3)
    p = [mp.mpf(0), p1, p2, p3, p4, p5, p6]
    c = [c0, c1, c2, c3]
    cp, pp = _pmul(c, p), _pmul(p, p)
    b1 = [_fact(k) - cp[k] - pp[k] for k in range(4)]
    b2 = c
    b3 = [mp.mpf(0), p1, p2 - q1 * q1, p3 - 2 * q1 * q2]
    b4 = [mp.mpf(0), q1, q2, q3]
    return (b1, b2, b3, b4)


def t12_polynomial(rows):
    b1, b2, b3, b4 = rows
    a6 = _padd(b3, _pmul(b4, b4))
    return _padd(b1, _pmul(_padd(b2, a6), a6))


# Free coefficients of the T18 scheme (row, column); B1's coefficient of A stays at the
# published value, structural zeros stay zero.
_T18_FREE = ((0, 2), (0, 3), (1, 1), (1, 2), (1, 3), (1, 4), (2, 0), (2, 1), (2, 2), (2, 3), (2, 4),
             (3, 0), (3, 1), (3, 2), (3, 3), (3, 4), (4, 2), (4, 3), (4, 4))


def t18_polynomial(rows):
    basis = ([1], [0, 1], [0, 0, 1], [0, 0, 0, 1], [0, 0, 0, 0, 0, 0, 1])

    def comb(row):
        return _padd(*[[mp.mpf(cf) * v for v in b] for cf, b in zip(row, basis)])

    b1, b2, b3, b4, b5 = (comb(r) for r in rows)
    a9 = _padd(_pmul(b1, b5), b4)
    return _padd(b2, _pmul(_padd(b3, a9), a9))


def t18_coefficients():
    """Rows B1..B5 of the T18 scheme on (I, A, A2, A3, A6), Newton-refined."""

    def rows_from(values):
        rows = [[mp.mpf(0)] * 5 for _ in range(5)]
        rows[0][1] = mp.mpf(T18_PUBLISHED[0][1])
        for (r, c), v in zip(_T18_FREE, values):
            rows[r][c] = v
        return rows

    def equations(*values):
        poly = t18_polynomial(rows_from(values))
        return [poly[k] - _fact(k) for k in range(19)]

    start = [mp.mpf(T18_PUBLISHED[r][c]) for r, c in _T18_FREE]
    return rows_from(mp.findroot(equations, start, tol=mp.mpf(10) ** -45, maxsteps=50))


def t12_structure_rows(m: int):
    """B1..B4 on (I, A, A2, A3) evaluating T_m (m in 1, 2, 4, 8) in the T12 structure."""
    z = [mp.mpf(0)] * 4
    if m in (1, 2):
        b1 = [_fact(k) if k <= m else mp.mpf(0) for k in range(4)]
        return (b1, list(z), list(z), list(z))
    h = m // 2                    # A6 = a A^h
    a = 1 / mp.sqrt(mp.factorial(m))
    b4 = list(z)
    b4[h // 2] = mp.sqrt(a)       # B4 = sqrt(a) A^(h/2): A (m = 4) or A2 (m = 8)
    b2 = list(z)
    for k in range(h, m):
        b2[k - h] = _fact(k) / a
    b1 = [_fact(k) if k < h else mp.mpf(0) for k in range(4)]
    return (b1, b2, list(z), b4)


def scheme_residual(poly, m):
    """Largest |coefficient - 1/k!| relative to 1/k! over k <= m, and the largest term above m."""
    rel = max(abs(poly[k] - _fact(k)) / _fact(k) for k in range(m + 1))
    tail = max([abs(x) for x in poly[m + 1 :]] or [mp.mpf(0)])
    return rel, tail


def derive():
    thetas = {m: theta(m) for m in DEGREES}
    return thetas, t8_coefficients(), t12_coefficients(), t18_coefficients()


def _f(x):
    return mp.nstr(x, 20, min_fixed=-30, max_fixed=30)


def render_header(thetas, t8, t12, t18) -> str:
    lines = [
        "// Generated by oracle/derive_coefficients.py -- do not edit by hand.",
        "// Degree thresholds and polynomial-scheme coefficients for the adaptive Taylor",
        "// scaling-and-squaring exponential (Bader, Blanes, Casas 2019).",
        "#pragma once",
        "",
        "namespace fhx {",
        "// theta_m: largest ||A|| with float32 backward error <= 2^-24 for Taylor degree m.",
    ]
    for m in DEGREES:
        lines.append(f"constexpr double kTheta{m} = {_f(thetas[m])};")
    lines.append("")
    lines.append("// T8 = y0 I + y1 A + y2 A2 + (x3 A2 + A4)(x4 I + x5 A + x6 A2 + x7 A4), A4 = A2 (x1 A + x2 A2).")
    for k in ("x1", "x2", "x3", "x4", "x5", "x6", "x7", "y2"):
        lines.append(f"constexpr float kT8{k.upper()} = {_f(t8[k])}f;")
    lines.append("")
    lines.append("// T12 = B1 + (B2 + A6) A6, A6 = B3 + B4 B4; t12c(r, c) is the coefficient of")
    lines.append("// (I, A, A2, A3)[c] in B(r+1).")
    lines.append("__host__ __device__ constexpr float t12c(int r, int c) {")
    lines.append("  constexpr float tab[4][4] = {")
    for row in t12:
        lines.append("      {" + ", ".join(_f(v) + "f" for v in row) + "},")
    lines.append("  };")
    lines.append("  return tab[r][c];")
    lines.append("}")
    lines.append("")
    lines.append("// T1, T2, T4, T8 and T12 in the T12 structure: t12u(d, r, c) is the coefficient of")
    lines.append("// (I, A, A2, A3)[c] in B(r+1) for degree index d (m = 1, 2, 4, 8, 12).")
    lines.append("__host__ __device__ constexpr float t12u(int d, int r, int c) {")
    lines.append("  constexpr float tab[5][4][4] = {")
    for m in (1, 2, 4, 8):
        lines.append("      {")
        for row in t12_structure_rows(m):
            lines.append("          {" + ", ".join(_f(v) + "f" for v in row) + "},")
        lines.append("      },")
    lines.append("      {")
    for row in t12:
        lines.append("          {" + ", ".join(_f(v) + "f" for v in row) + "},")
    lines.append("      },")
    lines.append("  };")
    lines.append("  return tab[d][r][c];")
    lines.append("}")
    lines.append("")
    lines.append("// T18 = B2 + (B3 + A9) A9, A9 = B1 B5 + B4; t18c(r, c) is the coefficient of")
    lines.append("// (I, A, A2, A3, A6)[c] in B(r+1).")
    lines.append("__host__ __device__ constexpr float t18c(int r, int c) {")
    lines.append("  constexpr float tab[5][5] = {")
    for row in t18:
        lines.append("      {" + ", ".join(_f(v) + "f" for v in row) + "},")
    lines.append("  };")
    lines.append("  return tab[r][c];")
    lines.append("}")
    lines.append("}  // namespace fhx")
    return "\n".join(lines) + "\n"


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--check", action="store_true", help="compare with the committed header instead of writing it")
    args = parser.parse_args()
    thetas, t8, t12, t18 = derive()
    for name, poly, m in (("T8", t8_polynomial(t8), 8), ("T12", t12_polynomial(t12), 12), ("T18", t18_polynomial(t18), 18),
                          *((f"T{k} (T12 structure)", t12_polynomial(t12_structure_rows(k)), k) for k in (1, 2, 4, 8))):
        rel, tail = scheme_residual(poly, m)
        print(f"{name}: max rel coefficient error {mp.nstr(rel, 3)}, largest term above degree {m}: {mp.nstr(tail, 3)}")
    text = render_header(thetas, t8, t12, t18)
    if args.check:
        same = HEADER.read_text() == text
        print("header matches" if same else "header differs")
        raise SystemExit(0 if same else 1)
    HEADER.write_text(text)
    print(f"wrote {HEADER}")


if __name__ == "__main__":
    main()
