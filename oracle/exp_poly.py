"""The degree-5 polynomial of ky_exp (kyro_b200/csrc/kyro_math.h): its fit
and a check of the committed coefficients.

TEST INFRASTRUCTURE: run by tests/test_oracle.py and by hand
(`python oracle/exp_poly.py`); nothing in the product imports it.

ky_exp reduces x = n*ln2 + r with |r| <= ln2/2 and evaluates
p(r) = 1 + c1 r + c2 r^2 + c3 r^3 + c4 r^4 + c5 r^5 by Horner's rule in
fp32.  The coefficients were fitted for this project by iterated weighted
least squares (Lawson's algorithm: least squares in the relative error
(p - e^r) / e^r on a dense grid, each round reweighting by the previous
round's absolute error) with c0 fixed at 1, and rounded to fp32.  The
iteration was stopped early, so the committed set is not the minimax set:
its largest relative error before rounding is 9.3e-8, against 7.4e-8 for
the discrete minimax polynomial of the same degree (found here by linear
programming).  The bar that matters is the rounded ky_exp itself, which
tests/test_oracle.py holds to <= 6 ulp of double exp.
"""
from __future__ import annotations

import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
HEADER = os.path.join(HERE, "..", "kyro_b200", "csrc", "kyro_math.h")


def committed() -> list:
    """c0..c5 as written in kyro_math.h (KY_EXP_C0..C5)."""
    text = open(HEADER).read()
    return [float.fromhex(re.search(rf"#define KY_EXP_C{i} (\S+)f", text).group(1))
            for i in range(6)]


def grid(n: int = 20001) -> np.ndarray:
    h = np.log(2.0) / 2
    return np.linspace(-h, h, n)


def max_rel_error(c, r=None) -> float:
    """Largest |p(r) - e^r| / e^r over the grid, p evaluated in double."""
    r = grid() if r is None else r
    p = np.zeros_like(r)
    for ci in reversed(c):
        p = p * r + ci
    return float(np.max(np.abs(p - np.exp(r)) / np.exp(r)))


def lawson_fit(rounds: int = 60, n: int = 20001) -> list:
    """Lawson's iteration for the relative-error fit with c0 = 1."""
    r = grid(n)
    f = np.exp(r)
    A = np.stack([r ** i for i in range(1, 6)], axis=1) / f[:, None]
    b = (f - 1.0) / f
    w = np.full(r.size, 1.0 / r.size)
    for _ in range(rounds):
        sw = np.sqrt(w)
        c, *_ = np.linalg.lstsq(A * sw[:, None], b * sw, rcond=None)
        err = np.abs(A @ c - b)
        w = w * err
        w /= w.sum()
    return [1.0] + [float(np.float32(x)) for x in c]


def minimax_fit(n: int = 4001) -> tuple:
    """The discrete minimax relative-error polynomial (c0 = 1), by linear
    programming: minimise t subject to |(p(r_i) - e^r_i) / e^r_i| <= t."""
    from scipy.optimize import linprog
    r = grid(n)
    f = np.exp(r)
    A = np.stack([r ** i for i in range(1, 6)], axis=1) / f[:, None]
    b = (f - 1.0) / f
    ones = np.ones((r.size, 1))
    G = np.vstack([np.hstack([A, -ones]), np.hstack([-A, -ones])])
    res = linprog(np.r_[np.zeros(5), 1.0], A_ub=G, b_ub=np.r_[b, -b],
                  bounds=[(None, None)] * 6, method="highs")
    return [1.0] + [float(x) for x in res.x[:5]], float(res.x[5])


def main():
    c = committed()
    print("committed  c0..c5:", " ".join(float(x).hex() for x in c))
    print(f"committed  max relative error before rounding: {max_rel_error(c):.3e}")
    lf = lawson_fit()
    print("lawson     c1..c5:", " ".join(float(x).hex() for x in lf[1:]))
    print(f"lawson     max relative error: {max_rel_error(lf):.3e}")
    mm, t = minimax_fit()
    print(f"minimax    max relative error: {t:.3e}")


if __name__ == "__main__":
    main()
