"""Provenance of the GELU coefficients of the residual tensor-core kernel
(tc_resid.cu, gelu_phi).

GELU(x) = x * Phi(x), Phi the standard normal distribution function.  For
t = |x|, 1 - Phi(t) = Phi(-t) = 0.5 * exp(-t^2 / 2) * erfcx(t / sqrt(2)),
erfcx the scaled complementary error function.  erfcx(t / sqrt(2)) is
smooth and bounded on [0, 12], so a rational function P4(t) / Q5(t) with
Q(0) = 1 fits it to 4.8e-9 relative error (double).  The fit is an
iteratively reweighted linearised least-squares rational fit on 4000
Chebyshev nodes of [0, 12] (minimising |f Q - P| / |f Q_prev|).

Evaluated in float32 with the exp as one hardware exp2, GELU's maximum
absolute error over [-14, 14] is 3.8e-7 (0.5 x (1 + erf(x / sqrt 2)) in
float32: 4.5e-7), its rms error 4.6e-8 (5.1e-8), and its relative error at
most 1.5e-6 where |GELU| > 1e-6 (the erf form loses all relative accuracy in
the left tail to cancellation).

    python ponni_b200/csrc/fit_gelu.py   # prints the coefficients
"""
import numpy as np
from scipy.special import erfcx


def fit(m=4, n=5, T=12.0, nodes=4000, iters=30):
    t = np.sort(np.cos(np.linspace(0, np.pi, nodes)) * T / 2 + T / 2)
    f = erfcx(t / np.sqrt(2))
    w = np.ones_like(t)
    for _ in range(iters):
        A = np.hstack([-np.vander(t, m + 1, increasing=True), f[:, None] * np.vander(t, n + 1, increasing=True)[:, 1:]])
        W = w / f
        coef, *_ = np.linalg.lstsq(A * W[:, None], -f * W, rcond=None)
        p, q = coef[:m + 1], np.concatenate([[1.0], coef[m + 1:]])
        w = 1.0 / np.abs(np.polyval(q[::-1], t))
    rel = np.max(np.abs(np.polyval(p[::-1], t) / np.polyval(q[::-1], t) - f) / f)
    return p, q, rel


if __name__ == "__main__":
    p, q, rel = fit()
    print("P", [float(np.float32(v)) for v in p])
    print("Q", [float(np.float32(v)) for v in q])
    print("max relative error (double)", rel)
