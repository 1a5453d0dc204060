"""The end-to-end HE-LRM forward (helrm_b200/helrm.py, the reference's
examples/criteo/dlrm.py:181-229 HELRM with Orion's ReLU and Bootstrap
layers) on the GPU, at LogN 13 with narrowed widths so that it runs in
seconds: bottom 13-64-16, three tables, top 64-32-1, a 19-level usable
chain over the 14 reserved bootstrapping primes (two bootstraps per
query).  The decrypted logits must match the cleartext forward with the
same composite polynomial activations within 1e-3 (the logit tolerance
of the HE-LRM checks), and the exact-ReLU forward within the composite
sign's own approximation error.
"""
import numpy as np
import pytest

from helrm_b200 import B200Library, CKKSConfig
from helrm_b200 import helrm as H
from helrm_b200 import workload as W

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=13, logq=[50] + [36] * 19, logp=[60] * 6, logscale=36, h=192, boot=True)


@pytest.fixture(scope="module")
def net():
    lib = B200Library(seed=20261206)
    lib.setup_bindings(CFG)
    lib.GenerateSecretKey()
    lib.GenerateRelinearizationKey()
    n = H.HELRM(lib, vocab=[50, 3000, 200000], bottom=(13, 64, 16), top_hidden=(32,), seed=3, boot_chunk=3)
    yield n
    n.close()
    lib.DeleteScheme()


def test_plan(net):
    info = net.info()
    assert info["bootstraps_per_query"] == 2 and info["boot_slots"] == [16, 32]
    assert info["levels"]["selector"] == info["levels"]["add"] + 2


def test_forward_matches_cleartext(net):
    lib = net.lib
    dense = H.dense_inputs(5, 5)
    sel = net.selectors(W.zipf_queries(net.vocab, 5, seed=9))
    d, s = net.encrypt(dense, sel)
    live = lib.GetLiveCiphertexts()
    out = net.forward(d, s)
    assert lib.GetLiveCiphertexts() == live + len(out)  # temporaries freed, inputs kept
    assert all(lib.GetCiphertextScale(o) == net.scale for o in out)
    assert all(lib.GetCiphertextLevel(o) == net.level_out for o in out)
    got = net.decrypt(out)
    want = net.cleartext(dense, sel)
    assert np.abs(got - want).max() < 1e-3
    exact = net.cleartext(dense, sel, poly=False)
    assert np.abs(got - exact).max() < np.abs(want - exact).max() + 1e-3
    for c in out + d + s:
        lib.DeleteCiphertext(c)


def test_forward_rejects_mismatched_inputs(net):
    with pytest.raises(ValueError):
        net.forward([1, 2], [3])
