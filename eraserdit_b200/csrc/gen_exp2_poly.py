"""Derive the exp2 polynomial used by the attention softmax (run once; prints C++).

2^x for x <= 0 is split Cody-Waite style into 2^floor(x) * 2^f, f in [0, 1).
2^floor(x) is built by adding floor(x) to the exponent field; 2^f is a cubic
whose coefficients minimise the maximum relative error over [0, 1), found here
as a linear program over a dense grid and then checked in fp32 Horner form.
The relative error (about 7.5e-5) is far below the 2^-9 rounding of the BF16
P operand it feeds.
"""

import numpy as np
from scipy.optimize import linprog


def minimax_exp2(degree: int, points: int = 20001):
    f = np.linspace(0.0, 1.0, points)
    basis = np.vstack([f ** k for k in range(degree + 1)]).T / (2.0 ** f)[:, None]
    n = degree + 1
    a_ub = np.vstack([np.hstack([basis, -np.ones((points, 1))]),
                      np.hstack([-basis, -np.ones((points, 1))])])
    b_ub = np.concatenate([np.ones(points), -np.ones(points)])
    cost = np.zeros(n + 1)
    cost[-1] = 1.0
    res = linprog(cost, A_ub=a_ub, b_ub=b_ub, bounds=[(None, None)] * n + [(0, None)],
                  method="highs")
    coef = res.x[:n].astype(np.float32)
    ff = f.astype(np.float32)
    p = np.full_like(ff, coef[-1])
    for k in range(degree - 1, -1, -1):
        p = (p * ff + coef[k]).astype(np.float32)
    err = float(np.abs(p.astype(np.float64) / 2.0 ** ff.astype(np.float64) - 1).max())
    return coef, err


if __name__ == "__main__":
    coef, err = minimax_exp2(3)
    print(f"// max relative error {err:.3e}")
    for k, c in enumerate(coef):
        print(f"constexpr float kExp2C{k} = {float(c).hex()}f;  // {float(c):.9g}")
