"""The GEMM epilogue's GELU: x*Phi(x) with the normal tail Q(t) = erfc(t/sqrt2)/2
evaluated as 2^P(t) for a degree-7 polynomial P (csrc/common.cuh, gelu_tail).

The coefficients are read from the source and evaluated here the way the
kernel does (fp32 Horner steps on t = min(|x|, 5.5), then 2^P), so the error
bound quoted in the source is checked against scipy's erf on the CPU."""
import os
import re

import numpy as np

from conftest import PKG


def _coefficients():
    src = open(os.path.join(PKG, "csrc", "common.cuh")).read()
    body = src[src.index("void gelu_tail(") :]
    m = re.search(r"kC\[8\]\s*=\s*\{([^}]*)\}", body)
    assert m, "gelu_tail coefficients not found"
    return np.array([float(v.strip().rstrip("f")) for v in m.group(1).split(",")], np.float32)


def _gelu_tail(x, c):
    x = x.astype(np.float32)
    t = np.minimum(np.abs(x), np.float32(5.5))
    p = np.full_like(t, c[-1])
    for ci in c[-2::-1]:
        p = (p * t + ci).astype(np.float32)  # one rounding per step, as fma.rn.f32x2 gives
    q = np.exp2(p.astype(np.float64)).astype(np.float32)
    r = x * q
    return np.where(x >= 0, x - r, r)


def test_gelu_tail_matches_erf_gelu():
    from scipy.special import erf

    c = _coefficients()
    assert c.shape == (8,)
    x = np.concatenate([np.linspace(-12, 12, 400001), np.linspace(-1e-3, 1e-3, 2001)]).astype(np.float32)
    ref = 0.5 * x.astype(np.float64) * (1 + erf(x.astype(np.float64) / np.sqrt(2)))
    got = _gelu_tail(x, c).astype(np.float64)
    err = np.abs(got - ref)
    # the bound the source states (below 5e-7 absolute over the whole real line),
    # plus the fp32 rounding of results of magnitude up to 12
    assert err.max() <= 5e-7 + 12 * 2.0 ** -24 * 2, err.max()
    # and relatively tight where gelu is not tiny
    big = np.abs(ref) > 1e-2
    assert (err[big] / np.abs(ref[big])).max() <= 2e-5
