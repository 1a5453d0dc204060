"""Polynomial evaluation on the CPU: the oracle's plan and the host-side
coefficient generator, pinned before the CUDA path is compared with them.

Pins: the reference's own composite sign coefficients (golden fixture made
by tests/golden/make_minimax_sign.py from orion/backend/cheddar/bindings.py:
1164-1230); the depth contract of the reference's call site (output level =
input level - ceil(log2(d+1)), cheddar_pybind.cu:2231-2258, which
orion/nn/activation.py:22-28,101-110 places layers with); the reference's
polynomial tests (tests/oracle/test_poly_eval.py), replayed through the
oracle's CKKS at small N; and Orion's ReLU (activation.py:201-300: x times
the composite step polynomial) within the north star's 1e-3.
"""
import json
import math
import os

import numpy as np
import pytest

from conftest import assert_fhe_close

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def poly_mod():
    from oracle import poly
    return poly


@pytest.fixture(scope="module")
def deep(oracle_mod):
    """logN 10 with 16 levels: enough for the ReLU composite [15, 15, 27]."""
    logn = 10
    main, aux = oracle_mod.scheme_primes([40] + [36] * 16, [60] * 4, logn)
    o = oracle_mod.Oracle(logn, main, aux, dnum=5)
    sk = o.secret_ntt(o.sample_secret(5, 64))
    return o, sk, o.relin_key(sk, 99)


def _cheb(x, c):
    return np.polynomial.chebyshev.chebval(x, c)


def test_minimax_sign_matches_reference():
    from helrm_b200.library import _composite_sign_coeffs
    with open(os.path.join(GOLDEN, "minimax_sign.json")) as f:
        cases = json.load(f)["cases"]
    for c in cases:
        got = _composite_sign_coeffs(c["degrees"], 2.0 ** -c["logalpha"])
        assert len(got) == sum(d + 1 for d in c["degrees"])
        np.testing.assert_allclose(got, c["coeffs"], rtol=0, atol=1e-12)


@pytest.mark.parametrize("d", list(range(2, 64)) + [127, 255])
@pytest.mark.parametrize("cheb", [True, False])
def test_plan_depth_is_ceil_log2(poly_mod, oracle_mod, d, cheb):
    main, _ = oracle_mod.scheme_primes([40] + [36] * 10, [60], 12)
    rng = np.random.default_rng(d)
    c = rng.uniform(-1, 1, d + 1)
    p = poly_mod.plan(main, cheb, 11, 2.0 ** 36, c, 2.0 ** 36)
    levels = math.ceil(math.log2(d + 1))
    assert p.depth == levels
    assert p.vnq[p.out] == 11 - levels
    # no more products than a pure giant-step chain (one per coefficient)
    assert p.products <= d


def test_plan_zero_coefficients_keep_depth(poly_mod, oracle_mod):
    """Trailing and interior zeros (odd polynomials) still land on the
    declared depth: the layer placement counts len(coeffs) - 1."""
    main, _ = oracle_mod.scheme_primes([40] + [36] * 8, [60], 12)
    for c in ([0.0, 1.0, 0.0, -0.5, 0.0, 0.0, 0.0, 0.0, 0.0],
              [0.5, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
              [0.0] * 16 + [1.0]):
        p = poly_mod.plan(main, True, 9, 2.0 ** 36, c, 2.0 ** 36)
        assert p.vnq[p.out] == 9 - math.ceil(math.log2(len(c)))


def test_plan_refuses_too_few_levels(poly_mod, oracle_mod):
    main, _ = oracle_mod.scheme_primes([40] + [36] * 3, [60], 12)
    with pytest.raises(ValueError, match="not enough levels"):
        poly_mod.plan(main, True, 4, 2.0 ** 36, np.ones(16), 2.0 ** 36)


def _run(poly_mod, deep, vals, coeffs, cheb, nq=17, in_scale=2.0 ** 36, out_scale=2.0 ** 36):
    o, sk, rlk = deep
    ct = o.encrypt(sk, o.encode(vals, nq, in_scale), 3)
    out, p = poly_mod.evaluate(o, rlk, ct, in_scale, coeffs, out_scale, chebyshev=cheb)
    assert out.shape[1] == nq - math.ceil(math.log2(len(coeffs)))
    return o.decode(o.decrypt(sk, out), out_scale), p


def test_reference_monomial_cases(poly_mod, deep):
    """tests/oracle/test_poly_eval.py:30-63 (descending coefficients there,
    ascending here after the poly_evaluator's reversal)."""
    n = deep[0].N // 2
    v = np.resize([0.5, 1.0, -0.5, 0.0], n)
    got, _ = _run(poly_mod, deep, v, [1.0, 1.0, 1.0], False)
    assert_fhe_close(got, v ** 2 + v + 1.0, atol=1e-6, msg="monomial quadratic")
    v = np.resize([0.25, 0.5, -0.25, -0.5], n)
    got, _ = _run(poly_mod, deep, v, [0.0, -1.0, 0.0, 1.0], False)
    assert_fhe_close(got, v ** 3 - v, atol=1e-6, msg="monomial cubic")


def test_reference_chebyshev_degree2(poly_mod, deep):
    """tests/oracle/test_poly_eval.py:68-84: [1, 0, 1] is 2 x^2."""
    v = np.resize([0.25, 0.5, -0.25, -0.5], deep[0].N // 2)
    got, _ = _run(poly_mod, deep, v, [1.0, 0.0, 1.0], True)
    assert_fhe_close(got, 2.0 * v ** 2, atol=1e-6, msg="chebyshev deg-2")


@pytest.mark.parametrize("d", [5, 8, 15, 16, 27, 31, 63])
def test_chebyshev_random_degrees(poly_mod, deep, d):
    rng = np.random.default_rng(100 + d)
    c = rng.uniform(-1, 1, d + 1) / np.arange(1, d + 2)
    v = rng.uniform(-1, 1, deep[0].N // 2)
    got, _ = _run(poly_mod, deep, v, c, True)
    assert_fhe_close(got, _cheb(v, c), atol=1e-5, msg=f"chebyshev degree {d}")


def test_scales_off_the_chain(poly_mod, deep):
    """Input and output scales that are neither 2^36 nor a prime."""
    rng = np.random.default_rng(7)
    c = rng.uniform(-1, 1, 12)
    v = rng.uniform(-1, 1, deep[0].N // 2)
    got, _ = _run(poly_mod, deep, v, c, True, in_scale=2.0 ** 35 * 1.37, out_scale=float(deep[0].primes[9]))
    assert_fhe_close(got, _cheb(v, c), atol=1e-5, msg="off-chain scales")


def test_relu_composite(poly_mod, deep):
    """Orion's ReLU (activation.py:246-300): prescaled x times the composite
    step polynomial [15, 15, 27] (logalpha 6), the last stage's output at
    scale q[level] so the product's rescale is exact."""
    from helrm_b200.library import _composite_sign_coeffs
    o, sk, rlk = deep
    degs = [15, 15, 27]
    flat = _composite_sign_coeffs(degs, 2.0 ** -6)
    stages = np.split(np.array(flat), np.cumsum([d + 1 for d in degs])[:-1])
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, o.N // 2)
    x[np.abs(x) < 2.0 ** -5] = 0.5  # outside the sign's gap
    nq = 17
    ct = o.encrypt(sk, o.encode(x, nq, 2.0 ** 36), 9)
    cur, scale = ct, 2.0 ** 36
    for i, c in enumerate(stages):
        last = i == len(stages) - 1
        out_nq = cur.shape[1] - math.ceil(math.log2(len(c)))
        target = float(o.primes[out_nq - 1]) if last else 2.0 ** 36
        cur, _ = poly_mod.evaluate(o, rlk, cur, scale, c, target)
        scale = target
    step = o.decode(o.decrypt(sk, cur), scale)
    assert np.abs(step - (x > 0)).max() < 1e-3
    xs = ct[:, :cur.shape[1]]
    relu = o.rescale(o.relinearize(o.tensor(xs, cur), rlk))
    got = o.decode(o.decrypt(sk, relu), 2.0 ** 36)
    assert np.abs(got - np.maximum(x, 0)).max() < 1e-3


def test_pack_lanes_layout():
    """orion/core/lane_packing.py:60-81: chunk 2m in the real lane and chunk
    2m+1 in the imaginary lane of packed m, scaled by 0.5, zero padded."""
    from helrm_b200 import lanes
    slots = 8
    v = np.arange(1, 3 * slots - 2, dtype=np.float64)
    packed, n = lanes.pack_lanes(v, slots)
    assert n == 3 and lanes.plan_packing(v.size, slots) == (3, 2)
    flat = np.concatenate([v, np.zeros(4 * slots - v.size)])
    ch = flat.reshape(4, slots)
    assert np.array_equal(packed.reshape(2, slots), 0.5 * (ch[0::2] + 1j * ch[1::2]))
    assert lanes.is_profitable(2 * slots, slots) and not lanes.is_profitable(slots, slots)
