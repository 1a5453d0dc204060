"""The exact FP64 modular product used by the NTT, the ModUp conversion and
phase A of the fused MAC (hb_arith.cuh: mulmod_d), checked in exact rational
arithmetic on the CPU.

For q < 2^40, w in [0, q), |y| < 2^44 and a quotient estimate w' (either
fl(w / q) from a host table, or fl(w * fl(1/q)) formed in a kernel):
  Q  = round(y * w')                       (fma with the 1.5 * 2^52 constant)
  ph = fl(Q * q),  pl = Q * q - ph         (TwoProduct: pl is a double)
  t  = fl(y * w - ph) - pl                 (the fma is exact, so is the sub)
must give t = y * w - Q * q exactly with |t| <= 0.502 q, so that sums of up
to 2^53 / (0.502 q) such remainders stay exact.
"""
from fractions import Fraction

import numpy as np
import pytest


def _round_half_even(x: Fraction) -> int:
    f = x.numerator // x.denominator
    r = x - f
    if r > Fraction(1, 2) or (r == Fraction(1, 2) and f % 2 == 1):
        return f + 1
    return f


def _is_double(v: int) -> bool:
    return float(v) == v


def _check(y: int, w: int, q: int, wq: float):
    # Q: the exact product y * w' rounded once to the nearest integer
    Q = _round_half_even(Fraction(y) * Fraction(wq))
    ph = float(Q) * float(q)  # correctly rounded product of two exact doubles
    assert _is_double(Q) and _is_double(q)
    pl = Q * q - int(ph)
    assert _is_double(pl), "TwoProduct low part must be a double"
    d = y * w - int(ph)  # what fma(y, w, -ph) rounds
    assert abs(d) < 2**53, "fma(y, w, -ph) must be exact"
    t = d - pl
    assert _is_double(t)
    assert t == y * w - Q * q
    assert abs(t) <= 0.502 * q, (y, w, q, t / q)
    assert (t - y * w) % q == 0


@pytest.mark.parametrize("bits", [30, 36, 39])
def test_mulmod_d_bounds(bits):
    rng = np.random.default_rng(bits)
    for _ in range(3000):
        q = int(rng.integers(2 ** (bits - 1), 2**bits)) | 1
        w = int(rng.integers(0, q))
        # operand magnitudes seen in the kernels: canonical residues, the
        # NTT's grown values (below 21 q) and the 2^44 limit
        lim = [q, 21 * q, 2**44][int(rng.integers(0, 3))]
        y = int(rng.integers(-lim + 1, lim))
        _check(y, w, q, float(w) / float(q))  # table estimate fl(w / q)
        _check(y, w, q, float(w) * (1.0 / float(q)))  # kernel estimate fl(w fl(1/q))


def test_mulmod_d_extremes():
    for q in [(1 << 36) - 5, (1 << 39) + 7, (1 << 30) + 3]:
        for w in [0, 1, q - 1, q // 2, q // 2 + 1]:
            for y in [0, 1, -1, q - 1, 21 * q, -21 * q, 2**44 - 1, -(2**44) + 1]:
                _check(y, w, q, float(w) / float(q))
                _check(y, w, q, float(w) * (1.0 / float(q)))
