"""Polynomial evaluation on the GPU path (EvaluatePolynomial).

The reference's Orion evaluates activations through
``poly_evaluator.evaluate_polynomial`` (orion/backend/python/
poly_evaluator.py:25-35) -> ``EvaluatePolynomial`` (cheddar bindings.py:
1102-1116) -> Cheddar's native EvalPoly (cheddar_pybind.cu:2207-2262).
Here the native evaluation must equal oracle/poly.py residue for residue
(same plan, same constants, the oracle's exact tensor / relinearization /
rescale), land ceil(log2(d+1)) levels down at exactly the requested scale,
pass the reference's own polynomial tests (tests/oracle/test_poly_eval.py),
and run Orion's ReLU composite [15, 15, 27] within 1e-3.
"""
import math

import numpy as np
import pytest

from conftest import assert_fhe_close
from gpu_helpers import Pair
from helrm_b200 import CKKSConfig

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=12, logq=[40] + [36] * 16, logp=[60] * 4, logscale=36, h=64)
TOP = 16


@pytest.fixture(scope="module")
def pair(oracle_mod):
    p = Pair(CFG, dnum=5, seed=20261202, oracle_mod=oracle_mod)
    p.rlk = p.key(0)
    assert np.array_equal(p.rlk, p.o.relin_key(p.sk, p.seed))
    yield p
    p.close()


@pytest.fixture(scope="module")
def poly_mod():
    from oracle import poly
    return poly


def _native(pair, ct, coeffs, cheb, scale):
    pid = pair.lib.GenerateChebyshev(list(coeffs)) if cheb else pair.lib.GenerateMonomial(list(coeffs))
    return pair.lib.EvaluatePolynomial(ct, pid, scale), pid


@pytest.mark.parametrize("d,cheb", [(2, True), (3, False), (7, True), (15, True), (16, False), (27, True),
                                    (31, True), (63, True)])
def test_residues_match_oracle(pair, poly_mod, d, cheb):
    rng = np.random.default_rng(d)
    coeffs = rng.uniform(-1, 1, d + 1) / np.arange(1, d + 2)
    x = rng.uniform(-1, 1, pair.slots)
    ct = pair.encrypt(x, TOP)
    out, pid = _native(pair, ct, coeffs, cheb, pair.scale)
    ref, plan = poly_mod.evaluate(pair.o, pair.rlk, pair.ct_data(ct), pair.scale, coeffs, pair.scale, chebyshev=cheb)
    got = pair.ct_data(out)
    assert got.shape == ref.shape
    assert np.array_equal(got, ref)
    levels = math.ceil(math.log2(d + 1))
    assert pair.lib.GetCiphertextLevel(out) == TOP - levels
    assert pair.lib.GetCiphertextScale(out) == pair.scale
    info = pair.lib.PolynomialPlanInfo(pid, TOP, pair.scale)
    assert info == {"depth": plan.depth, "products": plan.products, "rescales": plan.rescales, "bs": plan.bs}
    assert pair.lib.GetPolyDepth(pid) == levels
    want = np.polynomial.chebyshev.chebval(x, coeffs) if cheb else np.polynomial.polynomial.polyval(x, coeffs)
    assert_fhe_close(pair.decrypt(out), want, atol=1e-5, msg=f"degree {d}")


def test_batch_equals_single(pair):
    rng = np.random.default_rng(11)
    coeffs = rng.uniform(-1, 1, 12)
    cts = [pair.encrypt(rng.uniform(-1, 1, pair.slots), TOP) for _ in range(3)]
    cts.append(pair.encrypt(rng.uniform(-1, 1, pair.slots), TOP - 2))  # a second (rows, scale) group
    pid = pair.lib.GenerateChebyshev(list(coeffs))
    outs = pair.lib.EvaluatePolynomialBatch(cts, pid, pair.scale)
    for c, o in zip(cts, outs):
        one = pair.lib.EvaluatePolynomial(c, pid, pair.scale)
        assert np.array_equal(pair.ct_data(o), pair.ct_data(one))


def test_off_chain_scales(pair, poly_mod):
    """Input scale off 2^36 and an output scale equal to a chain prime (the
    sign's last stage, activation.py:246-258)."""
    rng = np.random.default_rng(5)
    coeffs = rng.uniform(-1, 1, 10)
    x = rng.uniform(-1, 1, pair.slots)
    s_in = 2.0 ** 35 * 1.37
    ct = pair.encrypt(x, TOP, s_in)
    target = float(pair.o.primes[TOP - 4])
    out, _ = _native(pair, ct, coeffs, True, target)
    ref, _ = poly_mod.evaluate(pair.o, pair.rlk, pair.ct_data(ct), s_in, coeffs, target)
    assert np.array_equal(pair.ct_data(out), ref)
    assert pair.lib.GetCiphertextScale(out) == target


def test_reference_poly_eval_cases(pair):
    """tests/oracle/test_poly_eval.py:12-97 through the backend surface
    (degree < 2 on Horner's rule, as bindings.py:1104-1116)."""
    lib = pair.lib

    def run(values, coeffs, cheb):
        x = np.resize(values, pair.slots)
        ct = pair.encrypt(x, TOP)
        pid = lib.GenerateChebyshev(coeffs) if cheb else lib.GenerateMonomial(coeffs)
        return x, pair.decrypt(lib.EvaluatePolynomial(ct, pid, pair.scale))

    x, got = run([0.5, 1.0, -0.5, 0.0], [1.0, 2.0], False)  # 2x + 1 (ascending)
    assert_fhe_close(got, 2 * x + 1, atol=1e-6, msg="monomial linear")
    x, got = run([0.5, 1.0, -0.5, 0.0], [1.0, 1.0, 1.0], False)
    assert_fhe_close(got, x ** 2 + x + 1, atol=1e-6, msg="monomial quadratic")
    x, got = run([0.25, 0.5, -0.25, -0.5], [0.0, -1.0, 0.0, 1.0], False)
    assert_fhe_close(got, x ** 3 - x, atol=1e-6, msg="monomial cubic")
    x, got = run([0.25, 0.5, -0.25, -0.5], [1.0, 0.0, 1.0], True)
    assert_fhe_close(got, 2 * x ** 2, atol=1e-6, msg="chebyshev deg-2")
    x, got = run([0.1, 0.5, -0.3, 0.9], [0.0, 1.0], True)
    assert_fhe_close(got, x, atol=1e-6, msg="chebyshev identity")


def test_minimax_sign_interface(pair):
    """tests/oracle/test_poly_eval.py:100-116: one coefficient list per degree."""
    flat = pair.lib.GenerateMinimaxSignCoeffs([7], 64, 6, 6, 0)
    assert len(flat) == 8
    flat = pair.lib.GenerateMinimaxSignCoeffs([3, 5], 64, 6, 6, 0)
    assert len(flat) == 10


def test_relu_composite(pair, poly_mod):
    """Orion's ReLU (activation.py:246-300): x * step(x) with the composite
    [15, 15, 27] sign polynomial, the last stage at scale q[level]."""
    lib = pair.lib
    degs = [15, 15, 27]
    flat = lib.GenerateMinimaxSignCoeffs(degs, 128, 6, 12, 0)
    stages = np.split(np.array(flat), np.cumsum([d + 1 for d in degs])[:-1])
    rng = np.random.default_rng(8)
    x = rng.uniform(-1, 1, pair.slots)
    x[np.abs(x) < 2.0 ** -5] = -0.25  # outside the sign's gap
    ct = pair.encrypt(x, TOP)
    cur = ct
    for i, c in enumerate(stages):
        lvl = lib.GetCiphertextLevel(cur) - math.ceil(math.log2(len(c)))
        target = float(lib.GetModuliChain()[lvl]) if i == len(stages) - 1 else pair.scale
        pid = lib.GenerateChebyshev(list(c))
        nxt = lib.EvaluatePolynomial(cur, pid, target)
        assert lib.GetCiphertextLevel(nxt) == lvl
        cur = nxt
    assert lib.GetCiphertextLevel(cur) == TOP - 13
    step = pair.decrypt(cur)
    assert np.abs(step - (x > 0)).max() < 1e-3
    relu = lib.Rescale(lib.MulRelinCiphertextNew(ct, cur))
    assert lib.GetCiphertextScale(relu) == pytest.approx(pair.scale, rel=1e-12)
    assert np.abs(pair.decrypt(relu) - np.maximum(x, 0)).max() < 1e-3


def test_errors(pair):
    lib = pair.lib
    ct = pair.encrypt(np.zeros(pair.slots), 3)
    pid = lib.GenerateChebyshev([0.1] * 32)  # 5 levels > 3
    with pytest.raises(RuntimeError, match="not enough levels"):
        lib.EvaluatePolynomial(ct, pid, pair.scale)
    sq = lib.MulRelinCiphertextNew(ct, ct)
    assert lib.GetCiphertextDegree(sq) == 1  # relinearized: accepted
