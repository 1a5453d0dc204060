"""Host side of the end-to-end HE-LRM forward (helrm_b200/helrm.py): the
fit, Orion's prescale rules, the level plan and the cleartext forward,
on a stand-in library that carries only the prime chain (no GPU)."""
import math

import numpy as np
import pytest

from helrm_b200 import helrm as H
from helrm_b200 import library as L
from helrm_b200 import workload as W
from helrm_b200.params import CFG4


class ChainOnly:
    """The library calls the fit and the plan make: the slot count, the
    prime chains and the sign coefficients."""

    def __init__(self, logq, logn, boot=14):
        from oracle import oracle as O
        self.main, _ = O.scheme_primes(list(logq) + [60] * boot, [60] * 6, logn)
        self.usable = len(logq)
        self._default_scale = 2.0 ** 36
        self.slots = 1 << (logn - 1)

    def scheme_info(self):
        return {"slots": self.slots}

    def GetModuliChain(self):
        return self.main[:self.usable]

    def GetAllModuliChain(self):
        return self.main

    def GenerateMinimaxSignCoeffs(self, degrees, *_):
        return L._composite_sign_coeffs(list(degrees), 2.0 ** -6)


@pytest.fixture(scope="module")
def cfg4():
    return H.HELRM(ChainOnly(CFG4.logq, CFG4.logn), build=False)


def test_copy_into_matches_dlrm():
    M = H.copy_into(416, 432, 16)
    x = np.arange(416.0)
    y = M @ x
    assert np.array_equal(y[16:], x) and not y[:16].any()


def test_config4_plan(cfg4):
    """LogN 16, 23 usable levels: the first ReLU fits without a
    bootstrap; every later one bootstraps before its sign (five per
    query), the selector sits two levels above the add."""
    info = cfg4.info()
    assert info["bootstraps_per_query"] == 5
    assert info["boot_slots"] == [256, 64, 16, 512, 256]
    assert info["levels"] == {"dense": 23, "selector": 10, "add": 8, "out": 8}
    for _, _, lin, lout, _ in info["plan"]:
        assert lin >= 1 and lout >= 1


def test_prescales_follow_orion(cfg4):
    for r, (lo, hi, _) in zip(cfg4.relus, cfg4._relu_in):
        a = max(abs(lo), abs(hi)) * H.MARGIN
        assert r.postscale == (math.ceil(a) if a > 1 else 1)
        assert r.prescale == 1.0 / r.postscale
    for r in cfg4.relus:
        if r.boot is not None:  # the prescaled input already lies in [-1, 1]
            assert r.boot.postscale == 1 and abs(r.boot.constant) < 0.5


def test_cleartext_polynomial_relu_close_to_exact(cfg4):
    dense = H.dense_inputs(32, 5)
    sel = cfg4.selectors(W.zipf_queries(cfg4.vocab, 32, seed=9))
    a = cfg4.cleartext(dense, sel)
    b = cfg4.cleartext(dense, sel, poly=False)
    assert a.shape == (32,)
    assert np.abs(a - b).max() < 1e-2


def test_relu_poly_is_a_relu_outside_the_gap():
    stages = H.sign_stages(L._composite_sign_coeffs(list(H.SIGN_DEGREES), 2.0 ** -6))
    x = np.linspace(-4, 4, 4001)
    y = H.relu_poly(x, stages, 0.25, 4)
    far = np.abs(x) * 0.25 > 2.0 ** -6
    assert np.abs(y - np.maximum(x, 0))[far].max() < 1e-3


def test_short_chain_is_refused():
    with pytest.raises(RuntimeError):
        H.HELRM(ChainOnly([50] + [36] * 17, 13), vocab=[50, 3000], bottom=(13, 64, 16), top_hidden=(32,),
                build=False)
