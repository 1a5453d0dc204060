"""CPU restatement of the bootstrapping circuit of helrm_b200/bootstrap.py.

TEST INFRASTRUCTURE ONLY: the checker for the GPU path's Bootstrap; the
product package never imports it.

The reference's bootstrapping is Cheddar's BootContext (reached through
orion/backend/cheddar/bindings.py:1326-1342, cheddar_pybind.cu:2049-2187),
third-party code absent from the checkout.  This file restates, on the
oracle's exact operators, the published circuit the B200 library runs
(ModRaise, SubSum, a dense CoeffsToSlots, the cosine / double-angle /
arcsine EvalMod, a dense SlotsToCoeffs; see the library module for the
derivation), in the same order with the same constants, so that given the
same keys and transform plaintexts the GPU output must match residue for
residue.  `bootstrap` takes the transform plaintexts and keys as inputs
(the library's, or ones the CPU test builds with the oracle's encoder).
"""
from __future__ import annotations

import math

import numpy as np

from . import poly


def _qs(o, nq):
    return np.array(o.primes[:nq], dtype=object)[None, :, None]


def add(o, a, b):
    nq = min(a.shape[1], b.shape[1])
    return ((a[:, :nq].astype(object) + b[:, :nq].astype(object)) % _qs(o, nq)).astype(np.uint64)


def add_scalar(o, ct, v, scale):
    """c0 + round(v * scale) with the library's rounding: the product in
    80-bit long double, then half away from zero"""
    x = np.longdouble(v) * np.longdouble(scale)
    r = np.floor(x + np.longdouble(0.5)) if x >= 0 else -np.floor(-x + np.longdouble(0.5))
    num, den = r.as_integer_ratio()
    k = num // den
    out = ct.astype(object).copy()
    for i in range(ct.shape[1]):
        out[0, i] = (out[0, i] + k) % o.primes[i]
    return out.astype(np.uint64)


def mod_raise(o, ct, nq_all):
    q0 = o.primes[0]
    out = np.zeros((2, nq_all, o.N), dtype=np.uint64)
    for pl in range(2):
        coef = o.intt(0, ct[pl, 0]).astype(object)
        cen = [int(v) - q0 if int(v) > q0 // 2 else int(v) for v in coef]
        for i in range(nq_all):
            out[pl, i] = o.ntt(i, np.array([v % o.primes[i] for v in cen], dtype=np.uint64))
    return out


def bootstrap(o, ct, scale_in, ctx, keys, rlk, cts_pts, stc_pts, replicate=False):
    """ctx: the scales and constants of helrm_b200.bootstrap.BootContext
    (dict with n, R, B, q0, s_u, s_cos, s_evalmod, subsum_steps, cts_bs,
    stc_bs, cos_coeffs, asin_coeffs (None: no arcsine), top); keys: {galois: switching key};
    cts_pts / stc_pts: the transforms' extended-basis plaintexts, diagonal k
    at index k (n of CtS, 2n of StC).  replicate: the input holds its values in slots [0, n) and
    zeros elsewhere and is first tiled over the subring by rotations at
    level 0.  Returns (ciphertext, output scale)."""
    n, S = ctx["n"], o.N // 2
    nq_all = ctx["top"] + 1
    def fold(c):  # c += rot(c, k) for k = slots/2, slots/4, ..., n (the hybrid fold's order)
        for k in reversed(ctx["subsum_steps"]):
            g = o.galois(k)
            c = add(o, c, o.rotate(c, keys[g], g))
        return c
    x = np.ascontiguousarray(ct[:, :1])
    if replicate:
        x = fold(x)
    t = fold(mod_raise(o, x, nq_all))
    # CtS onto 2n slots (n diagonals), plus its conjugate: the real coefficients
    w = o.rescale(o.bsgs_lt(t, list(range(n)), cts_pts, ctx["cts_bs"], keys))
    gc = 2 * o.N - 1
    cj = o.rotate(w, keys[gc], gc)
    u = add_scalar(o, add(o, w, cj), -1.0 / (4.0 * ctx["B"]), ctx["s_u"])
    y, _ = poly.evaluate(o, rlk, u, ctx["s_u"], ctx["cos_coeffs"], ctx["s_cos"], chebyshev=True)
    s = ctx["s_cos"]
    for _ in range(ctx["double_angles"]):
        sq = o.rescale(o.relinearize(o.tensor(y, y), rlk))
        s = s * s / float(o.primes[y.shape[1] - 1])
        y = add_scalar(o, add(o, sq, sq), -1.0, s)
    if ctx["asin_coeffs"] is not None:
        y, _ = poly.evaluate(o, rlk, y, s, ctx["asin_coeffs"], ctx["s_evalmod"], chebyshev=False)
    # StC from the 2n real slots (2n diagonals)
    out = o.rescale(o.bsgs_lt(y, list(range(2 * n)), stc_pts, ctx["stc_bs"], keys))
    q_stc = float(o.primes[y.shape[1] - 1])
    return out, ctx["s_evalmod"] * ctx["s_stc"] * scale_in / (q_stc * ctx["q0"])
