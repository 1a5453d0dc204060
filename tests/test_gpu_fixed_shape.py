"""Bit-exact parity of the fixed-shape kernels of the hot path, through the C ABI.

The headline PCMM runs specialised kernels: the fused baby-step MAC compiled
for full 32-baby chunks and four key-switching digits and launched once for
the q rows (36-bit primes: FP64 phase A, split-29 phase B) and once for the
special rows (60-bit primes: split-30 Karatsuba phase B), the batch-looping
key multiplication for four digits, and the hybrid fold with its add inside
the ModDown combine.  The small-parameter parity tests reach only the
generic kernels, so this file builds a scheme with the same shape at LogN 12:
8 q limbs and 2 special primes at dnum 4 (alpha 2, four digits), and a
transform whose baby-step stride is 32 with every baby present.
"""
import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig
from helrm_b200 import workload as W

pytestmark = pytest.mark.gpu

CFG4 = CKKSConfig(logn=12, logq=[40] + [36] * 7, logp=[60, 60], logscale=36, h=64)
LEVEL = 7
# babies 0..31 all present (full chunk), giants 0, 1, 3 and 4; bs = 32
KS = list(range(64)) + [96, 97, 130]
RATIO = 15.2


@pytest.fixture(scope="module")
def pair4(oracle_mod):
    p = Pair(CFG4, dnum=4, seed=20261202, oracle_mod=oracle_mod)
    assert p.info["alpha"] == 2 and p.info["dnum"] == 4
    yield p
    p.close()


def test_fixed_shape_bsgs_bit_exact(pair4):
    rng = np.random.default_rng(40)
    slots = pair4.slots
    diags = {k: rng.uniform(-0.5, 0.5, slots) for k in KS}
    data = np.concatenate([diags[k] for k in KS])
    lt = pair4.lib.GenerateLinearTransform(KS, data, LEVEL, RATIO, "none")
    plan = W.bsgs_plan(KS, RATIO, slots)
    assert plan["bs"] == 32 and pair4.lib.GetLinearTransformInfo(lt)["bs"] == 32
    for kk in pair4.lib.GetLinearTransformRotationKeys(lt):
        pair4.lib.GenerateLinearTransformRotationKey(kk)
    xs = [rng.uniform(-1, 1, slots) for _ in range(3)]
    cts = [pair4.encrypt(x) for x in xs]
    outs = pair4.lib.EvaluateLinearTransformBatch(lt, cts)
    pts = [pair4.lib.GetLinearTransformPlaintext(lt, k) for k in KS]
    keys = {pair4.o.galois(d): pair4.key(pair4.o.galois(d)) for d in plan["rotation_keys"]}
    for c, o in zip(cts, outs):
        want = pair4.o.bsgs_lt(pair4.ct_data(c), KS, pts, plan["stride"], keys)
        assert np.array_equal(pair4.ct_data(o), want)
    got = pair4.decrypt(pair4.lib.RescaleNew(outs[0]))
    ref = W.cleartext_lt(xs[0], diags, slots)
    assert np.abs(got - ref).max() < 1e-3
    pair4.lib.DeleteLinearTransform(lt)


def test_fixed_shape_fold_bit_exact(pair4):
    rng = np.random.default_rng(41)
    cts = [pair4.encrypt(rng.uniform(-1, 1, pair4.slots)) for _ in range(2)]
    before = [pair4.ct_data(c) for c in cts]
    pair4.lib.HybridFoldBatch(cts, 3)
    q = np.array(pair4.o.primes[:LEVEL + 1], dtype=np.uint64)[None, :, None].astype(object)
    for c, x in zip(cts, before):
        for i in range(1, 4):
            g = pair4.o.galois(pair4.slots >> i)
            r = pair4.o.rotate(x, pair4.key(g), g)
            x = ((x.astype(object) + r.astype(object)) % q).astype(np.uint64)
        assert np.array_equal(pair4.ct_data(c), x)


@pytest.mark.parametrize("nb", [2, 4, 5])
def test_paired_items_bit_exact(pair4, nb):
    """Chunks of at most 8 giant slots run two batch items per iteration:
    512 diagonals at bs = 64 (ratio 8) give two full baby chunks over the
    same 8 giant slots (the second accumulating), at even and odd batches."""
    rng = np.random.default_rng(50 + nb)
    slots = pair4.slots
    ks = list(range(512))
    diags = {k: rng.uniform(-0.5, 0.5, slots) for k in ks}
    data = np.concatenate([diags[k] for k in ks])
    lt = pair4.lib.GenerateLinearTransform(ks, data, LEVEL, 8.0, "none")
    plan = W.bsgs_plan(ks, 8.0, slots)
    assert plan["bs"] == 64 and pair4.lib.GetLinearTransformInfo(lt)["bs"] == 64
    for kk in pair4.lib.GetLinearTransformRotationKeys(lt):
        pair4.lib.GenerateLinearTransformRotationKey(kk)
    xs = [rng.uniform(-1, 1, slots) for _ in range(nb)]
    cts = [pair4.encrypt(x) for x in xs]
    outs = pair4.lib.EvaluateLinearTransformBatch(lt, cts)
    pts = [pair4.lib.GetLinearTransformPlaintext(lt, k) for k in ks]
    keys = {pair4.o.galois(d): pair4.key(pair4.o.galois(d)) for d in plan["rotation_keys"]}
    for c, o in zip(cts, outs):
        want = pair4.o.bsgs_lt(pair4.ct_data(c), ks, pts, plan["stride"], keys)
        assert np.array_equal(pair4.ct_data(o), want)
    got = pair4.decrypt(pair4.lib.RescaleNew(outs[-1]))
    assert np.abs(got - W.cleartext_lt(xs[-1], diags, slots)).max() < 1e-3
    pair4.lib.DeleteLinearTransform(lt)

