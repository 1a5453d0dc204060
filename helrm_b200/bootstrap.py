"""CKKS bootstrapping for sparse slot counts on the B200 backend.

The reference exposes ``NewBootstrapper(logPs, slots)`` / ``Bootstrap(ct,
slots)`` (orion/backend/cheddar/bindings.py:1326-1342, reaching Cheddar's
BootContext, cheddar_pybind.cu:2049-2187, which is not in the checkout).
Orion places the calls (orion/core/auto_bootstrap.py:227-331) and hands the
backend ciphertexts whose slot values it has already scaled into [-1, 1]
(orion/nn/operations.py:38-115).  This module is the circuit, built on the
library's native operators, after the published method (Cheon, Han, Kim,
Kim, Song, "Bootstrapping for approximate homomorphic encryption",
EUROCRYPT 2018; sparse packing and the cosine / double-angle EvalMod of
Chen, Chillotti, Song, EUROCRYPT 2019):

  Replicate  a ciphertext tagged wider than n slots carries its values in
             slots [0, n) and zeros elsewhere (Orion's Bootstrap layer zeroes
             the rest with its prescale multiply, orion/nn/operations.py:
             98-104): log2(N / 2n) rotations by n 2^i at level 0 (no level)
             tile it into the sparse subring; one tagged with n slots
             (SetCiphertextSlots, the reference's sparse ciphertexts) is
             periodic already;
  ModRaise   the level-0 ciphertext, lifted to every prime, decrypts to
             t = m + q0 I (I small: the overflow of c0 + c1 s over q0);
  SubSum     log2(N / 2n) rotations by n 2^i add the conjugates of the
             sparse subring: R t_sub with R = N / 2n, so read at scale
             R q0 the n slots hold E(t_sub) / q0;
  CtS        one dense 2n x n transform [M^-1; -i M^-1] / 2B, M the
             subring's encoding matrix (slot j = sum_k w_k zeta^(k g_j),
             w_k = t_k + i t_{k+n}, g_j = 5^j mod 4n), onto 2n slots; with
             its conjugate added (one conjugation) the 2n slots hold the
             real coefficients t_k / (B q0), k < 2n (sparse packing of the
             real and imaginary parts side by side: 2n <= N / 2);
  EvalMod    on that one ciphertext: u = (x - 1/4) / B in [-1, 1], a
             Chebyshev approximation of cos(2 pi B u / 2^r), r double angles
             c <- 2 c^2 - 1 giving sin(2 pi x), then, for message ratios
             q0 / scale below 2^10, arcsin(s) on the odd Taylor terms
             (s + s^3/6 + 3 s^5/40) so that the result is 2 pi (m / q0) up
             to (2 pi m / q0)^7 terms; at 2^10 and above sin(x) = x within a
             relative x^2 / 6 <= 6e-6 and the arcsine is left out;
  StC        one dense n x 2n transform [M, i M] / 2 pi from the 2n real
             slots back to the n-slot packing, landing at the top level of
             the usable chain at the default scale.

Levels: CtS 1, cosine 6 (degree 63), double angles 3, arcsine 3 (when
used), StC 1 -- boot_levels() primes of 60 bits are reserved above the
usable chain, as the
reference's Cheddar setup reserves its boot primes there
(bindings.py:279-294).  The input must satisfy q0 >= 2^4 scale (the
message ratio) and slots n <= 4096 (CtS holds n diagonals, StC 2n).
"""
from __future__ import annotations

import math

import numpy as np

COS_DEGREE = 63      # depth 6
DOUBLE_ANGLES = 3
ASIN_COEFFS = [0.0, 1.0, 0.0, 1.0 / 6.0, 0.0, 3.0 / 40.0]  # arcsin Taylor to s^5 (depth 3)
ASIN_DEPTH = 3
ASIN_MAX_RATIO_BITS = 10  # message ratios q0 / scale below 2^10 take the arcsine
MAX_SLOTS = 4096


def uses_arcsin(logq0: float, logscale: float) -> bool:
    return logq0 - logscale < ASIN_MAX_RATIO_BITS


def boot_levels(logq0: float, logscale: float) -> int:
    """Reserved primes: CtS, the cosine, the double angles, the arcsine when
    the message ratio needs it, StC."""
    return 1 + 6 + DOUBLE_ANGLES + (ASIN_DEPTH if uses_arcsin(logq0, logscale) else 0) + 1


def boot_prime_bits(logscale: int, logq0: int) -> list[int]:
    """Bit sizes of the reserved primes, lowest first (the top one is the
    CtS level).  All of 60 bits: EvalMod's scales sit at these primes, and
    its rescale noise (about sqrt(N h) per product) is amplified by the
    degree-63 Chebyshev basis (up to 63^2) and the double angles (4^3); at
    LogN 16 and h = 192, 51-bit primes (logscale + 15, the reference's
    Cheddar sizing) left 2e-4 in the slots, 60-bit primes 2^9 less."""
    return [60] * boot_levels(logq0, logscale)


def level_plan(q, top: int, asin: bool) -> dict:
    """Scales and levels of the circuit on the prime chain q (floats) whose
    top index is `top`: the CtS output scale s_u = q[top - 1], the cosine's
    output at q[l] for l = top - 7, each double angle squaring and dropping
    one prime, the arcsine (when used) landing at q[l - 3]; s_evalmod is the
    scale entering StC and lvl_stc its level."""
    lvl = top - 1 - 6
    out = {"s_u": q[top - 1], "s_cos": q[lvl]}
    s = out["s_cos"]
    for _ in range(DOUBLE_ANGLES):
        s = s * s / q[lvl]
        lvl -= 1
    out["s_dbl"] = s
    if asin:
        out["s_evalmod"], out["lvl_stc"] = q[lvl - ASIN_DEPTH], lvl - ASIN_DEPTH
    else:
        out["s_evalmod"], out["lvl_stc"] = s, lvl
    return out


def encoding_matrix(n: int) -> np.ndarray:
    """M[j, k] = zeta^(k g_j), zeta = exp(i pi / 2n), g_j = 5^j mod 4n: the
    slots of a subring polynomial from its packed coefficients
    w_k = t_k + i t_{k+n}."""
    g = np.ones(n, dtype=np.int64)
    for j in range(1, n):
        g[j] = g[j - 1] * 5 % (4 * n)
    k = np.arange(n)
    return np.exp(1j * np.pi * np.outer(g, k) / (2 * n))


def diagonals(A: np.ndarray, slots: int) -> np.ndarray:
    """Orion's diagonal convention out[i] = sum_l d_l[i] in[(i + l) mod S]
    for an r x c matrix (r, c powers of two) acting on c-periodic slots and
    giving r-periodic ones: d_l[i] = A[i mod r, (i + l) mod c] for
    l < c, period max(r, c), repeated over all slots: [c][slots] complex."""
    r, c = A.shape
    p = max(r, c)
    i = np.arange(p)
    d = np.stack([A[i % r, (i + l) % c] for l in range(c)])
    return np.tile(d, (1, slots // p))


def cos_coeffs(B: float, r: int, degree: int) -> list[float]:
    """Chebyshev coefficients of cos(2 pi B u / 2^r) on [-1, 1]."""
    from numpy.polynomial import chebyshev as C
    x = np.cos(np.pi * (np.arange(4 * degree) + 0.5) / (4 * degree))
    return C.chebfit(x, np.cos(2.0 * math.pi * B / 2 ** r * x), degree).tolist()


def overflow_bound(h: int) -> int:
    """|I| bound of ModRaise's overflow: a sum of h terms uniform in
    [-1/2, 1/2] (variance h/12), taken at 7 standard deviations."""
    return int(math.ceil(7.0 * math.sqrt(max(h, 1) / 12.0)))


class BootContext:
    """The transforms, the polynomials and the scales for one slot count."""

    def __init__(self, lib, slots: int):
        S = lib._slots
        n = int(slots)
        if n < 1 or n & (n - 1) or n > S:
            raise ValueError(f"Bootstrap: slots must be a power of two up to {S}")
        if n > MAX_SLOTS or 2 * n > S:
            raise ValueError(f"Bootstrap: at most {min(MAX_SLOTS, S // 2)} slots (dense transforms over 2n slots)")
        self.n, self.R = n, S // n
        q = lib.GetAllModuliChain()
        self.q = [float(x) for x in q]
        self.q0 = self.q[0]
        self.top = len(q) - 1
        self.usable_top = lib._max_level
        # the bit sizes the scheme was set up with (boot_prime_bits)
        logscale, logq0 = int(lib._default_scale).bit_length() - 1, int(q[0]).bit_length()
        self.asin = uses_arcsin(logq0, logscale)
        if self.top - boot_levels(logq0, logscale) != self.usable_top:
            raise RuntimeError("Bootstrap: the scheme was created without the reserved bootstrapping primes")
        self.B = overflow_bound(lib._h) + 1
        M = encoding_matrix(n)
        Minv = np.linalg.inv(M)
        # CtS at the top level: the SubSum output read at scale R q0, the
        # plaintext scale chosen so that the output scale is q[top - 1]
        self.s_u = self.q[self.top - 1]
        s_cts = self.s_u * self.q[self.top] / (self.R * self.q0)
        self.cts = self._transform(lib, np.vstack([Minv, -1j * Minv]) / (2 * self.B), self.top, s_cts)
        self.poly_cos = lib.GenerateChebyshev(cos_coeffs(self.B, DOUBLE_ANGLES, COS_DEGREE))
        # ascending, as the backend takes them
        self.poly_asin = lib.GenerateMonomial(list(ASIN_COEFFS)) if self.asin else None
        # scales through EvalMod (deterministic: targets at the primes)
        plan = level_plan(self.q, self.top, self.asin)
        self.s_cos, self.s_dbl = plan["s_cos"], plan["s_dbl"]
        self.s_evalmod, self.lvl_stc = plan["s_evalmod"], plan["lvl_stc"]
        assert self.lvl_stc == self.usable_top + 1 and plan["s_u"] == self.s_u
        # StC: slots 2 pi (m / q0) packed -> E(m) / q0, pt scale chosen so
        # that an input at the default scale comes out at the default scale
        d = float(lib._default_scale)
        self.s_stc = d * self.q0 * self.q[self.lvl_stc] / (d * self.s_evalmod)
        self.stc = self._transform(lib, np.hstack([M, 1j * M]) / (2 * math.pi), self.lvl_stc, self.s_stc)
        # keys: the SubSum rotations, both transforms', the conjugation
        self.subsum_steps = []
        step = n
        while step < S:
            self.subsum_steps.append(step)
            step *= 2
        for k in self.subsum_steps:
            lib.AddRotationKey(k)
        for lt in (self.cts, self.stc):
            for k in lib.GetLinearTransformRotationKeys(lt):
                lib.GenerateLinearTransformRotationKey(k)

    @staticmethod
    def transform_ratio(ndiag: int) -> float:
        """BSGS ratio giving 32 baby steps (64 above 512 diagonals): the
        fused MAC's full-chunk shapes, the fastest splits measured on the
        LogN-16 transforms (bs 23 or 46 ran up to 1.8x slower)."""
        bs = 64 if ndiag > 512 else 32
        return bs * bs / float(ndiag)

    @staticmethod
    def _transform(lib, A, level, scale):
        S = lib._slots
        d = diagonals(A, S)
        inter = np.stack([d.real, d.imag], axis=-1).reshape(A.shape[1], 2 * S)
        return lib.GenerateLinearTransformEx(list(range(A.shape[1])), inter, S, level,
                                             BootContext.transform_ratio(A.shape[1]), True, scale)


def bootstrap(lib, ctx: BootContext, ct: int) -> int:
    """The circuit on one ciphertext (bootstrap_batch of one)."""
    return bootstrap_batch(lib, ctx, [ct])[0]


def bootstrap_batch(lib, ctx: BootContext, cts) -> list[int]:
    """The circuit on a batch of ciphertexts of the same slot count: the
    rotations, transforms, rescales and polynomials run through the
    library's batched entry points.  Returns new ciphertexts at the top of
    the usable chain holding the same slot values."""
    cts = [int(c) for c in cts]
    if not cts:
        return []
    scales = [lib.GetCiphertextScale(c) for c in cts]
    for s_in in scales:
        if ctx.q0 < 16.0 * s_in:
            raise RuntimeError("Bootstrap: the message ratio q0 / scale must be at least 2^4 "
                               f"(q0 = 2^{math.log2(ctx.q0):.1f}, scale = 2^{math.log2(s_in):.1f})")
    reps = len(ctx.subsum_steps)
    # level 0; a full-width input is tiled into the subring by the same
    # rotations (slots/2, slots/4, ..., n: the hybrid fold's)
    xs = [lib.AlignToLevelNew(c, 0) for c in cts]
    wide = [x for x, c in zip(xs, cts) if lib.GetCiphertextSlots(c) > ctx.n]
    if wide and reps:
        lib.HybridFoldBatch(wide, reps)
    ts = [lib.ModRaiseNew(x) for x in xs]
    for x in xs:
        lib.DeleteCiphertext(x)
    if reps:
        lib.HybridFoldBatch(ts, reps)   # SubSum
    for t in ts:
        lib.SetCiphertextScale(t, ctx.R * ctx.q0)
    ws = lib.EvaluateLinearTransformBatch(ctx.cts, ts)
    for t in ts:
        lib.DeleteCiphertext(t)
    lib.RescaleBatch(ws)
    # u = w + conj(w) - 1/4B: the 2n real coefficients side by side
    us = []
    for w in ws:
        cj = lib.ConjugateNew(w)
        lib.AddCiphertext(w, cj)
        lib.DeleteCiphertext(cj)
        lib.SetCiphertextScale(w, ctx.s_u)
        lib.AddScalar(w, -1.0 / (4.0 * ctx.B))
        us.append(w)
    ys = lib.EvaluatePolynomialBatch(us, ctx.poly_cos, ctx.s_cos)
    for u in us:
        lib.DeleteCiphertext(u)
    for _ in range(DOUBLE_ANGLES):  # y <- 2 y^2 - 1
        sqs = lib.MulRelinCiphertextBatchNew(ys, ys)
        for y in ys:
            lib.DeleteCiphertext(y)
        lib.RescaleBatch(sqs)
        for sq in sqs:
            lib.AddCiphertext(sq, sq)
            lib.AddScalar(sq, -1.0)
        ys = sqs
    if ctx.asin:
        zs = lib.EvaluatePolynomialBatch(ys, ctx.poly_asin, ctx.s_evalmod)
        for y in ys:
            lib.DeleteCiphertext(y)
    else:
        zs = ys
    outs = lib.EvaluateLinearTransformBatch(ctx.stc, zs)
    for z in zs:
        lib.DeleteCiphertext(z)
    lib.RescaleBatch(outs)
    # the values: E(m) / q0 at scale s_evalmod s_stc / q_stc, i.e. the
    # input's slots at s_evalmod s_stc scale_in / (q_stc q0)
    for o, c, s_in in zip(outs, cts, scales):
        lib.SetCiphertextScale(o, ctx.s_evalmod * ctx.s_stc * s_in / (ctx.q[ctx.lvl_stc] * ctx.q0))
        lib.SetCiphertextSlots(o, lib.GetCiphertextSlots(c))
    return outs
