"""Bootstrapping with the arcsine step (message ratio q0 / scale below
2^10; helrm_b200/bootstrap.py).  Its own module: the library holds one
scheme per process, so this scheme must not live beside another module's.
"""
import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig
from helrm_b200 import bootstrap as BT
from test_gpu_boot import TOP, _decrypt_c, _encrypt_sparse, check_residues_match_oracle

pytestmark = pytest.mark.gpu

# q0 of 44 bits over the 36-bit scale: message ratio 2^8
CFG_ASIN = CKKSConfig(logn=12, logq=[44, 36, 36, 36], logp=[60] * 4, logscale=36, h=64, boot=True)


@pytest.fixture(scope="module")
def pair_asin(oracle_mod):
    p = Pair(CFG_ASIN, dnum=5, seed=20261208, oracle_mod=oracle_mod)
    assert len(p.lib.GetAllModuliChain()) == 4 + BT.boot_levels(44, 36) == 4 + 14
    yield p
    p.close()


def test_bootstrap_with_arcsine_restores_values(pair_asin):
    """sin(2 pi m / q0) is no longer m's linear image within the
    precision at this ratio; the arcsine step corrects it"""
    n = 32
    rng = np.random.default_rng(7)
    z = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    z /= np.abs(z).max()
    ct = _encrypt_sparse(pair_asin, z, n, 0)
    out = pair_asin.lib.Bootstrap(ct, n)
    assert pair_asin.lib._boot[n].asin
    assert pair_asin.lib.GetCiphertextLevel(out) == TOP
    got = _decrypt_c(pair_asin, out)
    assert np.abs(got - np.tile(z, pair_asin.slots // n)).max() < 1e-5


def test_bootstrap_with_arcsine_residues_match_oracle(pair_asin):
    check_residues_match_oracle(pair_asin, padded=False, asin=True)
