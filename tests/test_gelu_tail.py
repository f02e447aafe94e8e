"""The GEMM epilogue's GELU, the reference's 0.5 x (1 + erf(x)), with the tail
Q(u) = erfc(u)/2 evaluated as 2^P(u) for a degree-7 polynomial P
(csrc/common.cuh, gelu_tail).

The coefficients and the clamp are read from the source and evaluated here the
way the kernel does (fp32 Horner steps on u = min(|x|, clamp), then 2^P), so
the error bound quoted in the source is checked against scipy's erf on the
CPU."""
import os
import re

import numpy as np

from conftest import PKG
from metrics import gelu_ref


def _coefficients():
    src = open(os.path.join(PKG, "csrc", "common.cuh")).read()
    body = src[src.index("void gelu_tail(") :]
    m = re.search(r"kC\[8\]\s*=\s*\{([^}]*)\}", body)
    assert m, "gelu_tail coefficients not found"
    k = re.search(r"kClamp\s*=\s*([0-9.eE+-]+)f", body)
    assert k, "gelu_tail clamp not found"
    return (np.array([float(v.strip().rstrip("f")) for v in m.group(1).split(",")], np.float32),
            np.float32(float(k.group(1))))


def _gelu_tail(x, c, clamp):
    x = x.astype(np.float32)
    t = np.minimum(np.abs(x), clamp)
    p = np.full_like(t, c[-1])
    for ci in c[-2::-1]:
        p = (p * t + ci).astype(np.float32)  # one rounding per step, as fma.rn.f32x2 gives
    q = np.exp2(p.astype(np.float64)).astype(np.float32)
    r = x * q
    return np.where(x >= 0, x - r, r)


def test_gelu_tail_matches_erf_gelu():
    c, clamp = _coefficients()
    assert c.shape == (8,)
    x = np.concatenate([np.linspace(-12, 12, 400001), np.linspace(-1e-3, 1e-3, 2001)]).astype(np.float32)
    ref = gelu_ref(x)
    got = _gelu_tail(x, c, clamp).astype(np.float64)
    err = np.abs(got - ref)
    # the bound the source states (below 5e-7 absolute over the whole real line),
    # plus the fp32 rounding of results of magnitude up to 12
    assert err.max() <= 5e-7 + 12 * 2.0 ** -24 * 2, err.max()
    # and relatively tight where gelu is not tiny
    big = np.abs(ref) > 1e-2
    assert (err[big] / np.abs(ref[big])).max() <= 2e-5
