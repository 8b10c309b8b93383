"""Accuracy of the oracle's erf_inv (M. Giles, "Approximating the erfinv function", GPU
Computing Gems Jade, 2011, with w = -log1p(-x*x) as StableHLO's chlo.erf_inv forms it)
against mpmath at 50 digits.

The reference's formula rounds x*x before anything else, and near |x| = 1 the
cancellation in 1 - x*x turns that one rounding into a large error in the result (64 ulp
at x = 0.9998 in float32): that error is the reference's own, kept for parity.  Measured
net of it -- against x * erf_inv(sqrt(s)) / sqrt(s), s = fl(x*x) -- the polynomials and their evaluation are
within a few ulp over the whole domain, the tails included.  The kernels compute the same
operations as the oracle (bit-exact, test_gpu_parity), so this bounds them too."""

import numpy as np
import pytest

from oracle import oracle as orc

mpmath = pytest.importorskip("mpmath")


def _cases(npdt, rng, n):
    digits = 7 if npdt == np.float32 else 15
    parts = [rng.uniform(0, 0.5, n), rng.uniform(0.5, 0.9, n), rng.uniform(0.9, 0.999, n),
             1 - 10.0 ** -rng.uniform(3, digits, n), np.array([1e-30, 1e-10, 2.0 ** -30])]
    x = np.concatenate(parts).astype(npdt)
    x = x[x < 1]
    return np.concatenate([x, -x])


def _formula(x, s):
    """x * g(s), g(s) = erf_inv(sqrt s) / sqrt s (g(0) = sqrt(pi) / 2): what the algorithm
    (x times a polynomial in w(s)) approximates once x*x has been rounded to s."""
    s = mpmath.mpf(float(s))
    g = mpmath.sqrt(mpmath.pi) / 2 if s == 0 else mpmath.erfinv(mpmath.sqrt(s)) / mpmath.sqrt(s)
    return float(mpmath.mpf(float(x)) * g)


@pytest.mark.parametrize("dt,bound", [("float32", 4.0), ("float64", 5.0)])
def test_erf_inv_within_a_few_ulp_of_its_formula(dt, bound):
    npdt = np.float32 if dt == "float32" else np.float64
    x = _cases(npdt, np.random.default_rng(0), 300)
    y = orc.erfinv(x, dt).astype(np.float64)
    mpmath.mp.dps = 50
    xx = (x * x).astype(npdt)
    ref = np.array([_formula(v, s) for v, s in zip(x, xx)])
    ulp = np.abs(y - ref) / np.spacing(np.abs(ref).astype(npdt)).astype(np.float64)
    assert ulp.max() <= bound, (ulp.max(), x[np.argmax(ulp)])


def test_erf_inv_error_near_one_is_the_formulas():
    """Against the exact erf_inv(x) the error near 1 is large, and it is the x*x rounding:
    the formula evaluated from the rounded s = fl(x*x) accounts for it."""
    mpmath.mp.dps = 50
    x = np.float32(0.9998295)
    y = float(orc.erfinv(np.array([x]), "float32")[0])
    exact = float(mpmath.erfinv(mpmath.mpf(float(x))))
    formula = _formula(x, np.float32(x * x))
    sp = float(np.spacing(np.float32(exact)))
    assert abs(y - exact) / sp > 16
    assert abs(y - formula) / sp <= 4


@pytest.mark.parametrize("dt,bound", [("float32", 2.0), ("float64", 3.0)])
def test_accurate_erf_inv_within_a_few_ulp_of_exact(dt, bound):
    """The accurate erf_inv (jax_accurate_erf_inv, R/lax_special.R:1022-1082) forms
    w = -log(q (1 + |x|)) from q = 1 - |x|, which is exact near |x| = 1: against mpmath's
    erf_inv of x itself it is within 2 ulp over the whole domain, tails included."""
    npdt = np.float32 if dt == "float32" else np.float64
    x = _cases(npdt, np.random.default_rng(1), 300)
    y = orc.erfinv(x, dt, accurate=True).astype(np.float64)
    mpmath.mp.dps = 50
    ref = np.array([float(mpmath.erfinv(mpmath.mpf(float(v)))) for v in x])
    ulp = np.abs(y - ref) / np.spacing(np.abs(ref).astype(npdt)).astype(np.float64)
    assert ulp.max() <= bound, (ulp.max(), x[np.argmax(ulp)])
