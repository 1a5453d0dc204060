"""Edge cases of the batch entry points on the GPU path: empty batches,
batches mixing levels, repeated handles, empty value lists, and the
boundaries of the polynomial and lane-unpacking calls.  Residues are
compared with the single-ciphertext path or the oracle.
"""
import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig
from helrm_b200 import workload as W

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=12, logq=[40, 36, 36, 36, 36], logp=[60, 60], logscale=36, h=64)


@pytest.fixture(scope="module")
def pair(oracle_mod):
    p = Pair(CFG, dnum=2, seed=20261204, oracle_mod=oracle_mod)
    yield p
    p.close()


@pytest.fixture(scope="module")
def lt(pair):
    rng = np.random.default_rng(1)
    ks = [0, 1, 2, 5, 9, 17, 40]
    data = np.concatenate([rng.uniform(-0.5, 0.5, pair.slots) for _ in ks])
    t = pair.lib.GenerateLinearTransform(ks, data, 3, 2.0, "none")
    for k in pair.lib.GetLinearTransformRotationKeys(t):
        pair.lib.GenerateLinearTransformRotationKey(k)
    yield t, ks
    pair.lib.DeleteLinearTransform(t)


def test_empty_batches_are_no_ops(pair, lt):
    t, _ = lt
    assert pair.lib.EvaluateLinearTransformBatch(t, []) == []
    pair.lib.RescaleBatch([])
    pair.lib.HybridFoldBatch([], 3)
    assert pair.lib.UnpackLanes([pair.encrypt(np.zeros(pair.slots), 2)], 0) == []
    with pytest.raises(ValueError):
        pair.lib.EvaluatePolynomialBatch([], pair.lib.GenerateChebyshev([0.1, 0.2, 0.3]))


def test_mixed_levels_and_repeated_handles(pair, lt):
    """A batch mixing inputs above, at and below the transform's level, with
    one handle twice: every output equals its own single-ciphertext run."""
    t, ks = lt
    rng = np.random.default_rng(2)
    cts = [pair.encrypt(rng.uniform(-1, 1, pair.slots), lv) for lv in (4, 3, 2, 3)]
    batch = cts + [cts[1]]
    outs = pair.lib.EvaluateLinearTransformBatch(t, batch)
    assert len(outs) == len(batch) and len(set(outs)) == len(outs)
    for c, o in zip(batch, outs):
        one = pair.lib.EvaluateLinearTransform(t, c)
        assert np.array_equal(pair.ct_data(o), pair.ct_data(one))
        assert pair.lib.GetCiphertextLevel(o) == min(3, pair.lib.GetCiphertextLevel(c))
    # and the oracle on the one below the transform's level
    plan = W.bsgs_plan(ks, 2.0, pair.slots)
    keys = {pair.o.galois(d): pair.key(pair.o.galois(d)) for d in plan["rotation_keys"]}
    # the transform's extended plaintexts (4 q rows + 2 special rows) read at
    # the input's 3 q rows
    full = [pair.lib.GetLinearTransformPlaintext(t, k) for k in ks]
    pts = [np.concatenate([P[:3], P[4:]]) for P in full]
    want = pair.o.bsgs_lt(pair.ct_data(cts[2]), ks, pts, plan["stride"], keys)
    assert np.array_equal(pair.ct_data(outs[2]), want)


def test_encode_empty_and_ragged_values(pair):
    pt = pair.lib.Encode([], 2, pair.scale)
    assert np.abs(np.array(pair.lib.Decode(pt))).max() == 0.0
    vals = np.arange(1, 38) / 40.0  # 37 values, the rest of the slots zero
    pt = pair.lib.Encode(list(vals), 2, pair.scale)
    got = np.array(pair.lib.Decode(pt))
    assert np.abs(got[:37] - vals).max() < 1e-8 and np.abs(got[37:]).max() < 1e-8
    with pytest.raises(ValueError):
        pair.lib.Encode(list(np.zeros(pair.slots + 1)), 2, pair.scale)


def test_polynomial_at_the_level_floor(pair):
    """Degree 7 needs 3 levels: at level 3 it lands on level 0; at level 2
    it is refused."""
    p = pair.lib.GenerateChebyshev(list(np.linspace(0.1, 0.8, 8)))
    x = np.linspace(-0.9, 0.9, pair.slots)
    out = pair.lib.EvaluatePolynomial(pair.encrypt(x, 3), p, pair.scale)
    assert pair.lib.GetCiphertextLevel(out) == 0
    want = np.polynomial.chebyshev.chebval(x, np.linspace(0.1, 0.8, 8))
    assert np.abs(pair.decrypt(out) - want).max() < 1e-4
    with pytest.raises(RuntimeError, match="not enough levels"):
        pair.lib.EvaluatePolynomial(pair.encrypt(x, 2), p, pair.scale)
