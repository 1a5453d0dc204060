"""CPU restatement of the polynomial evaluation behind EvaluatePolynomial.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path's
``helrm_EvaluatePolynomial``; the product package never imports it.

The reference reaches Cheddar's native ``EvalPoly`` through
``EvaluatePolynomialNative`` (orion/backend/cheddar/ext/cheddar_pybind.cu:
2207-2262, from bindings.py:1102-1116).  Cheddar is a third-party library
that is not part of the reference checkout, so this file restates the
published algorithm it implements -- baby-step giant-step evaluation in the
Chebyshev basis (Bossuat, Mouchet, Troncoso-Pastoriza, Hubaux, Eurocrypt
2021) -- with the properties the reference's call site checks: the output
sits ceil(log2(d+1)) levels below the input (cheddar_pybind.cu:2231-2238,
orion/nn/activation.py:22-28,101-110), at exactly the requested scale, and
degree < 2 stays on Horner's rule (bindings.py:1104-1116).

Planning (the CUDA library's host code builds the same plan):
  p = q T_{2^k} + r with 2^k <= deg p < 2^(k+1); q is evaluated one level up
  at scale S q_{L+1} / s(T_{2^k}); the product and the remainder's leaf sum
  sum_i round(r_i S q_{L+1} / s_i) T_i + round(r_0 S q_{L+1}) meet before one
  rescale.  A node is a leaf when its powers are all in the basis (T_1..T_bs
  and the powers of two) above its target level.  Basis: T_{2a} = 2 T_a^2 - 1
  and T_{a+b} = 2 T_a T_b - round(s_a s_b / s_{a-b}) T_{a-b} before their
  rescale (a the largest power of two below a+b); x^(a+b) = x^a x^b in the
  monomial basis.  bs in {2, 4, .., 32} with the fewest products, then the
  fewest rescales.  Constants round half away from zero.

Execution uses the oracle's exact tensor, relinearization, rescale and
multiply-accumulate, so the CUDA path must match it residue for residue.
"""
from __future__ import annotations

import math
from fractions import Fraction

import numpy as np

MUL, LIN, RESCALE, ADD = range(4)


def round_half_away(v: float) -> int:
    f = Fraction(v)
    return math.floor(f + Fraction(1, 2)) if f >= 0 else -math.floor(-f + Fraction(1, 2))


def _ceil_log2(v: int) -> int:
    k = 0
    while (1 << k) < v:
        k += 1
    return k


def _floor_pow2(v: int) -> int:
    p = 1
    while p * 2 <= v:
        p *= 2
    return p


def _degree(c) -> int:
    d = len(c) - 1
    while d > 0 and c[d] == 0.0:
        d -= 1
    return max(d, 0)


class Plan:
    def __init__(self, primes, cheb, nq0, s1, bs):
        self.primes = [int(p) for p in primes]
        self.cheb, self.nq0, self.bs = cheb, nq0, bs
        self.ops = []           # (kind, out, a, b, terms [(value, int coef)], k0 int or None)
        self.vnq, self.vscale = [], []
        self.products = self.rescales = 0
        self.powers = {1: self._value(nq0, s1)}

    # -- value bookkeeping
    def _value(self, nq, scale):
        self.vnq.append(nq)
        self.vscale.append(scale)
        return len(self.vnq) - 1

    def _q(self, nq):
        return float(self.primes[nq - 1])

    def _mul(self, a, b):
        v = self._value(min(self.vnq[a], self.vnq[b]), self.vscale[a] * self.vscale[b])
        self.ops.append((MUL, v, a, b, None, None))
        self.products += 1
        return v

    def _lin(self, nq, scale, terms, k0):
        for t, _ in terms:
            assert self.vnq[t] >= nq
        v = self._value(nq, scale)
        self.ops.append((LIN, v, -1, -1, [(t, round_half_away(c)) for t, c in terms],
                         None if k0 is None else round_half_away(k0)))
        return v

    def _rescale(self, a, scale):
        assert self.vnq[a] >= 2
        v = self._value(self.vnq[a] - 1, scale)
        self.ops.append((RESCALE, v, a, -1, None, None))
        self.rescales += 1
        return v

    def _add(self, a, b):
        assert self.vnq[a] == self.vnq[b]
        v = self._value(self.vnq[a], self.vscale[a])
        self.ops.append((ADD, v, a, b, None, None))
        return v

    # -- the power basis
    def power(self, i):
        if i in self.powers:
            return self.powers[i]
        pow2 = (i & (i - 1)) == 0
        if not self.cheb:
            a = i // 2 if pow2 else _floor_pow2(i)
            va, vb = self.power(a), self.power(i - a)
            P = self._mul(va, vb)
            v = self._rescale(P, self.vscale[P] / self._q(self.vnq[P]))
        elif pow2:
            va = self.power(i // 2)
            P = self._mul(va, va)
            sp = self.vscale[P]
            v = self._rescale(self._lin(self.vnq[P], sp, [(P, 2.0)], -sp), sp / self._q(self.vnq[P]))
        else:
            a = _floor_pow2(i)
            b, c = i - a, a - (i - a)
            va, vb, vc = self.power(a), self.power(b), self.power(c)
            P = self._mul(va, vb)
            sp = self.vscale[P]
            K = float(round_half_away(sp / self.vscale[vc]))
            v = self._rescale(self._lin(self.vnq[P], sp, [(P, 2.0), (vc, -K)], None), sp / self._q(self.vnq[P]))
        self.powers[i] = v
        return v

    def _leafable(self, c, L):
        for i in range(1, len(c)):
            if c[i] == 0.0:
                continue
            if not (i <= self.bs or (i & (i - 1)) == 0) or self.nq0 - _ceil_log2(i) < L + 2:
                return False
        return True

    def _leaf_terms(self, c, Sp, terms):
        for i in range(1, len(c)):
            if c[i] == 0.0:
                continue
            v = self.power(i)
            terms.append((v, (c[i] * Sp) / self.vscale[v]))
        return c[0] * Sp

    def eval(self, c0, L, S):
        d = _degree(c0)
        c = list(c0[:d + 1])
        Sp = S * self._q(L + 2)
        if self._leafable(c, L):
            terms = []
            k0 = self._leaf_terms(c, Sp, terms)
            if not terms:
                terms.append((self.power(1), 0.0))
            return self._rescale(self._lin(L + 2, Sp, terms, k0), S)
        n2 = _floor_pow2(d)
        qv = [0.0] * (d - n2 + 1)
        rv = list(c[:n2])
        if self.cheb:
            qv[0] = c[n2]
            for i in range(1, d - n2 + 1):
                qv[i] = 2.0 * c[n2 + i]
                rv[n2 - i] -= c[n2 + i]
        else:
            qv = list(c[n2:d + 1])
        G = self.power(n2)
        assert self.vnq[G] >= L + 2
        qconst = _degree(qv) == 0
        if qconst:
            terms = [(G, (qv[0] * Sp) / self.vscale[G])]
        else:
            terms = [(self._mul(self.eval(qv, L + 1, Sp / self.vscale[G]), G), 1.0)]
        if self._leafable(rv, L):
            k0 = self._leaf_terms(rv, Sp, terms)
            return self._rescale(self._lin(L + 2, Sp, terms, k0), S)
        R = self.eval(rv, L, S)
        v = self._lin(L + 2, Sp, terms, None) if qconst else terms[0][0]
        return self._add(self._rescale(v, S), R)


def plan(primes, cheb, nq0, s1, coeffs, scale):
    """The plan with the fewest products (then rescales) over bs = 2 .. 32."""
    coeffs = [float(c) for c in coeffs]
    if len(coeffs) < 3:
        raise ValueError("the log-depth evaluation needs degree >= 2")
    levels = _ceil_log2(len(coeffs))
    if nq0 - 1 - levels < 0:
        raise ValueError("not enough levels for the polynomial's degree")
    best = None
    bs = 2
    while bs <= 32 and bs <= (1 << levels):
        p = Plan(primes, cheb, nq0, s1, bs)
        p.out = p.eval(coeffs, nq0 - 1 - levels, float(scale))
        p.depth = levels
        if best is None or (p.products, p.rescales) < (best.products, best.rescales):
            best = p
        bs *= 2
    return best


def evaluate(o, rlk, ct, in_scale, coeffs, scale, chebyshev=True):
    """Run the plan on the oracle: ct (2, nq, N) at in_scale -> (ciphertext, plan)."""
    ct = np.ascontiguousarray(ct, dtype=np.uint64)
    p = plan(o.primes[:o.L], chebyshev, ct.shape[1], float(in_scale), coeffs, scale)
    vals = {0: ct}
    for kind, out, a, b, terms, k0 in p.ops:
        nq = p.vnq[out]
        if kind == MUL:
            vals[out] = o.relinearize(o.tensor(vals[a][:, :nq], vals[b][:, :nq]), rlk)
        elif kind == LIN:
            qs = o.primes[:nq]
            cts = [vals[t][:, :nq] for t, _ in terms]
            pts = [np.repeat(np.array([k % q for q in qs], dtype=np.uint64)[:, None], o.N, axis=1)
                   for _, k in terms]
            acc = o.mac(cts, pts)
            if k0 is not None:
                kr = np.array([k0 % q for q in qs], dtype=np.uint64)[:, None]
                acc[0] = o.fold_add(acc[None, 0], np.broadcast_to(kr, acc[0].shape)[None])[0]
            vals[out] = acc
        elif kind == RESCALE:
            vals[out] = o.rescale(vals[a])
        else:
            vals[out] = o.fold_add(vals[a], vals[b])
    return vals[p.out], p
