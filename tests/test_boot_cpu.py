"""The bootstrapping circuit on the CPU oracle (oracle/boot.py), pinned
before the GPU path is compared with it: a level-0 ciphertext of sparse
complex slots comes back at the top of the usable chain within 1e-5, with
the transforms, constants and scales of helrm_b200/bootstrap.py built here
from the oracle's own encoder and keys.  Also the pieces with closed forms:
the subring encoding matrix against the oracle's canonical embedding, and
the ModRaise overflow bound.
"""
import math

import numpy as np
import pytest

from helrm_b200 import bootstrap as BT
from helrm_b200 import workload as W


def _scheme(oracle_mod, logq0):
    logn, logscale = 10, 36
    logq = [logq0, 36, 36] + BT.boot_prime_bits(logscale, logq0)
    main, aux = oracle_mod.scheme_primes(logq, [60] * 4, logn)
    o = oracle_mod.Oracle(logn, main, aux, dnum=5)
    sk = o.secret_ntt(o.sample_secret(9, 64))
    return o, sk, logscale


@pytest.fixture(scope="module")
def scheme(oracle_mod):
    return _scheme(oracle_mod, 50)


@pytest.fixture(scope="module")
def scheme_asin(oracle_mod):
    return _scheme(oracle_mod, 44)  # message ratio 2^8: the arcsine is taken


def test_encoding_matrix_is_the_canonical_embedding(scheme):
    """Slots of a subring polynomial (coefficients at multiples of N/2n)
    equal M (t_k + i t_{k+n})."""
    o, _, _ = scheme
    n, N = 8, scheme[0].N
    rng = np.random.default_rng(0)
    t = rng.integers(-50, 50, 2 * n)
    coef = np.zeros(N, dtype=np.int64)
    coef[np.arange(2 * n) * (N // (2 * n))] = t
    pt = np.stack([o.ntt(i, (coef % o.primes[i]).astype(np.uint64)) for i in range(2)])
    slots = o.decode(pt, 1.0, complex_out=True)[:n]
    w = t[:n] + 1j * t[n:]
    assert np.abs(slots - BT.encoding_matrix(n) @ w).max() < 1e-9


def test_overflow_bound():
    assert BT.overflow_bound(64) == 17 and BT.overflow_bound(192) == 28  # 7 sigma, sigma^2 = h / 12


def _transform_pts(o, A, level, scale, bs):
    S = o.N // 2
    d = BT.diagonals(A, S)
    return [o.encode(W.preroll(d[k], k // bs, bs), level + 1, scale, ext=True) for k in range(A.shape[1])]


def test_arcsine_only_below_ratio_2_10():
    assert BT.boot_levels(50, 36) == 11 and BT.boot_levels(44, 36) == 14 and BT.boot_levels(46, 36) == 11
    assert BT.boot_prime_bits(36, 45) == [60] * 14


@pytest.mark.parametrize("logq0", [50, 44])
def test_level_plan_spends_exactly_the_reserved_primes(logq0):
    """CtS, the cosine, the double angles, the arcsine when taken and StC
    use every reserved prime once: StC's output sits at the top of the
    usable chain, and each double angle keeps the cosine's scale when it
    squares at a prime of that size."""
    usable_top, logscale = 23, 36
    nboot = BT.boot_levels(logq0, logscale)
    q = [2.0 ** 50] + [2.0 ** 36] * usable_top + [2.0 ** 60] * nboot
    top = len(q) - 1
    plan = BT.level_plan(q, top, BT.uses_arcsin(logq0, logscale))
    assert plan["lvl_stc"] - 1 == usable_top
    assert plan["s_u"] == q[top - 1] and plan["s_cos"] == q[top - 7]
    assert plan["s_dbl"] == plan["s_cos"] and plan["s_evalmod"] == q[plan["lvl_stc"]]


@pytest.mark.parametrize("padded,asin", [(False, False), (True, False), (False, True)])
def test_oracle_bootstrap_precision(request, padded, asin):
    from oracle import boot as OB
    o, sk, logscale = request.getfixturevalue("scheme_asin" if asin else "scheme")
    n, S = 8, o.N // 2
    R = S // n
    q = [float(p) for p in o.primes[:o.L]]
    assert BT.uses_arcsin(int(o.primes[0]).bit_length(), logscale) == asin
    top, usable_top = o.L - 1, o.L - 1 - BT.boot_levels(int(o.primes[0]).bit_length(), logscale)
    B = BT.overflow_bound(64) + 1
    s_u = q[top - 1]
    s_cts = s_u * q[top] / (R * q[0])
    r1, r2 = BT.BootContext.transform_ratio(n), BT.BootContext.transform_ratio(2 * n)
    bs = W.bsgs_plan(list(range(n)), r1, S)["stride"]
    bs2 = W.bsgs_plan(list(range(2 * n)), r2, S)["stride"]
    M = BT.encoding_matrix(n)
    Minv = np.linalg.inv(M)
    cts_pts = _transform_pts(o, np.vstack([Minv, -1j * Minv]) / (2 * B), top, s_cts, bs)
    # the circuit's scales, restated (helrm_b200.bootstrap.level_plan)
    lvl = top - 7
    s_cos = q[lvl]
    s = s_cos
    for _ in range(BT.DOUBLE_ANGLES):
        s = s * s / q[lvl]
        lvl -= 1
    s_evalmod, lvl_stc = (q[lvl - 3], lvl - 3) if asin else (s, lvl)
    assert lvl_stc == usable_top + 1
    assert BT.level_plan(q, top, asin) == {"s_u": s_u, "s_cos": s_cos, "s_dbl": s, "s_evalmod": s_evalmod,
                                           "lvl_stc": lvl_stc}
    s_stc = q[0] * q[lvl_stc] / s_evalmod
    stc_pts = _transform_pts(o, np.hstack([M, 1j * M]) / (2 * math.pi), lvl_stc, s_stc, bs2)
    plan = W.bsgs_plan(list(range(n)), r1, S)
    plan2 = W.bsgs_plan(list(range(2 * n)), r2, S)
    steps = []
    step = n
    while step < S:
        steps.append(step)
        step *= 2
    gal = ({o.galois(k) for k in steps} | {o.galois(d) for d in plan["rotation_keys"] + plan2["rotation_keys"]}
           | {2 * o.N - 1})
    keys = {g: o.rotation_key(sk, 5, g) for g in gal}
    rlk = o.relin_key(sk, 5)
    ctx = {"n": n, "R": R, "B": B, "q0": q[0], "s_u": s_u, "s_cos": s_cos, "s_evalmod": s_evalmod, "s_stc": s_stc,
           "subsum_steps": steps, "cts_bs": bs, "stc_bs": bs2, "top": top, "double_angles": BT.DOUBLE_ANGLES,
           "cos_coeffs": BT.cos_coeffs(B, BT.DOUBLE_ANGLES, BT.COS_DEGREE),
           "asin_coeffs": BT.ASIN_COEFFS if asin else None}
    rng = np.random.default_rng(4)
    z = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)) * 0.7
    scale = float(1 << logscale)
    if padded:  # values in slots [0, n), zeros after them (tiled first)
        v = np.zeros(S, complex)
        v[:n] = z
    else:       # the sparse (periodic) form
        v = np.tile(z, R)
    ct = o.encrypt(sk, o.encode(v, 1, scale), 11)
    out, s_out = OB.bootstrap(o, ct, scale, ctx, keys, rlk, cts_pts, stc_pts, replicate=padded)
    assert out.shape[1] == usable_top + 1
    assert s_out == pytest.approx(scale, rel=1e-9)
    got = o.decode(o.decrypt(sk, out), s_out, complex_out=True)
    assert np.abs(got - np.tile(z, R)).max() < 1e-5
