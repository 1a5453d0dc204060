"""Bit-exact parity of the fixed-shape fused MAC over mixed prime sizes,
through the C ABI: full 32-baby chunks of 2 to 7 key-switching digits on a
chain holding a 50-bit q0, 36-bit primes and 60-bit primes (the
bootstrapping chain's shape), where the product form is chosen per row.
Its own module: the library holds one scheme per process.
"""
import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig
from helrm_b200 import workload as W
from test_gpu_fixed_shape import KS, RATIO

pytestmark = pytest.mark.gpu

# mixed rows: a 50-bit q0, 36-bit primes and 60-bit primes in the q chain
# (the bootstrapping chain's shape), alpha 3, so full chunks run the
# fixed-shape kernels of 2 to 7 digits with the product form per row
CFG_MIXED = CKKSConfig(logn=12, logq=[50] + [36] * 14 + [60] * 6, logp=[60] * 4, logscale=36, h=64)


@pytest.fixture(scope="module")
def pair_mixed(oracle_mod):
    p = Pair(CFG_MIXED, dnum=7, seed=20261207, oracle_mod=oracle_mod)
    assert p.info["alpha"] == 3
    yield p
    p.close()


@pytest.mark.parametrize("level,beta", [(20, 7), (17, 6), (14, 5), (11, 4), (8, 3), (5, 2)])
def test_fixed_shape_mixed_rows_bit_exact(pair_mixed, level, beta):
    lib, o = pair_mixed.lib, pair_mixed.o
    assert -(-(level + 1) // 3) == beta
    rng = np.random.default_rng(level)
    slots = pair_mixed.slots
    diags = {k: rng.uniform(-0.5, 0.5, slots) for k in KS}
    lt = lib.GenerateLinearTransform(KS, np.concatenate([diags[k] for k in KS]), level, RATIO, "none")
    plan = W.bsgs_plan(KS, RATIO, slots)
    assert lib.GetLinearTransformInfo(lt)["bs"] == 32
    for kk in lib.GetLinearTransformRotationKeys(lt):
        lib.GenerateLinearTransformRotationKey(kk)
    xs = [rng.uniform(-1, 1, slots) for _ in range(3)]
    cts = [pair_mixed.encrypt(x, level) for x in xs]
    outs = lib.EvaluateLinearTransformBatch(lt, cts)
    pts = [lib.GetLinearTransformPlaintext(lt, k) for k in KS]
    keys = {o.galois(d): pair_mixed.key(o.galois(d)) for d in plan["rotation_keys"]}
    for c, out in zip(cts, outs):
        assert np.array_equal(pair_mixed.ct_data(out), o.bsgs_lt(pair_mixed.ct_data(c), KS, pts, plan["stride"], keys))
    got = pair_mixed.decrypt(outs[0])  # before the rescale (the top primes are 60-bit)
    assert np.abs(got - W.cleartext_lt(xs[0], diags, slots)).max() < 1e-3
    lib.DeleteLinearTransform(lt)
