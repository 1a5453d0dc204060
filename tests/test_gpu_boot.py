"""Bootstrapping on the GPU path (NewBootstrapper / Bootstrap).

The reference reaches Cheddar's BootContext (orion/backend/cheddar/
bindings.py:1326-1342); Orion's Bootstrap layer scales the slot values
into [-1, 1] first (orion/nn/operations.py:38-115) and expects the result
at the top of the usable chain.  Here: a level-0 ciphertext comes back at
the usable top level with its slot values within 1e-5 (real and complex
values, several sparse slot counts), every residue equal to the oracle's
restatement of the same circuit (oracle/boot.py) on the library's own
keys and transform plaintexts, the message-ratio precondition refused.
"""
import math

import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig
from helrm_b200 import bootstrap as BT

pytestmark = pytest.mark.gpu

# q0 of 50 bits over the 36-bit scale: message ratio 2^14 (no arcsine)
CFG = CKKSConfig(logn=12, logq=[50, 36, 36, 36], logp=[60] * 4, logscale=36, h=64, boot=True)
TOP = 3


@pytest.fixture(scope="module")
def pair(oracle_mod):
    p = Pair(CFG, dnum=5, seed=20261205, oracle_mod=oracle_mod)
    assert len(p.lib.GetAllModuliChain()) == 4 + BT.boot_levels(50, 36) == 4 + 11
    assert len(p.lib.GetModuliChain()) == 4
    yield p
    p.close()



def _encrypt_sparse(pair, z, n, level, padded=False):
    """n slot values repeated over every slot and tagged as a sparse
    ciphertext of n slots (the reference's sparse ciphertexts), or, with
    padded, in slots [0, n) and zero elsewhere at the full width (what
    Orion's Bootstrap layer hands a non-Cheddar backend)"""
    if padded:
        vals = np.zeros(pair.slots, complex)
        vals[:n] = z
    else:
        vals = np.tile(np.asarray(z, complex), pair.slots // n)
    inter = np.stack([vals.real, vals.imag], axis=-1).ravel()
    pt = pair.lib.EncodeComplex(inter, level, pair.scale)
    ct = pair.lib.Encrypt(pt)
    pair.lib.DeletePlaintext(pt)
    if not padded:
        pair.lib.SetCiphertextSlots(ct, n)
    return ct


def _decrypt_c(pair, ct):
    pt = pair.lib.Decrypt(ct)
    v = np.array(pair.lib.DecodeComplex(pt))
    pair.lib.DeletePlaintext(pt)
    return v[0::2] + 1j * v[1::2]


@pytest.mark.parametrize("n", [16, 64])
def test_bootstrap_restores_values(pair, n):
    rng = np.random.default_rng(n)
    z = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    z /= np.abs(z).max()
    ct = _encrypt_sparse(pair, z, n, 0)
    pair.lib.NewBootstrapper(None, n)
    out = pair.lib.Bootstrap(ct, n)
    assert pair.lib.GetCiphertextLevel(out) == TOP
    assert pair.lib.GetCiphertextScale(out) == pytest.approx(pair.scale, rel=1e-9)
    got = _decrypt_c(pair, out)
    assert np.abs(got - np.tile(z, pair.slots // n)).max() < 1e-5


def test_bootstrap_zero_padded_input_from_a_higher_level(pair):
    """Orion's real activations as its Bootstrap layer hands them to a
    non-Cheddar backend: the first n slots, zeros after them, at the full
    width and above level 0 (dropped first); the values come back in the
    first n slots (repeated over the rest)."""
    n = 32
    x = np.linspace(-1, 1, n)
    ct = _encrypt_sparse(pair, x, n, 2, padded=True)
    out = pair.lib.Bootstrap(ct, n)
    got = _decrypt_c(pair, out)
    assert np.abs(got.real - np.tile(x, pair.slots // n)).max() < 1e-5
    assert np.abs(got.imag).max() < 1e-5
    # and a second pass on the (periodic) output, tagged sparse
    low = pair.lib.AlignToLevelNew(out, 0)
    pair.lib.SetCiphertextSlots(low, n)
    again = pair.lib.Bootstrap(low, n)
    assert np.abs(_decrypt_c(pair, again).real - np.tile(x, pair.slots // n)).max() < 2e-5


def check_residues_match_oracle(pair, padded, asin):
    """The bootstrap's output residues against oracle/boot.py on the
    library's own keys and transform plaintexts (also used by the arcsine
    module)."""
    from oracle import boot as OB
    n = 16
    rng = np.random.default_rng(3)
    z = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)) * 0.7
    ct = _encrypt_sparse(pair, z, n, 0, padded=padded)
    pair.lib.NewBootstrapper(None, n)
    ctx = pair.lib._boot[n]
    assert ctx.asin == asin
    out = pair.lib.Bootstrap(ct, n)
    lib, o = pair.lib, pair.o
    info_c, info_s = lib.GetLinearTransformInfo(ctx.cts), lib.GetLinearTransformInfo(ctx.stc)
    gal = {o.galois(k) for k in ctx.subsum_steps} | {2 * pair.N - 1}
    for lt in (ctx.cts, ctx.stc):
        gal |= {o.galois(k) for k in lib.GetLinearTransformRotationKeys(lt)}
    keys = {g: pair.key(g) for g in sorted(gal)}
    c = {"n": n, "R": ctx.R, "B": ctx.B, "q0": ctx.q0, "s_u": ctx.s_u, "s_cos": ctx.s_cos,
         "s_evalmod": ctx.s_evalmod, "s_stc": ctx.s_stc, "subsum_steps": ctx.subsum_steps,
         "cts_bs": info_c["bs"], "stc_bs": info_s["bs"], "top": ctx.top, "double_angles": BT.DOUBLE_ANGLES,
         "cos_coeffs": BT.cos_coeffs(ctx.B, BT.DOUBLE_ANGLES, BT.COS_DEGREE),
         "asin_coeffs": BT.ASIN_COEFFS if ctx.asin else None}
    cts_pts = [lib.GetLinearTransformPlaintext(ctx.cts, k) for k in range(n)]
    stc_pts = [lib.GetLinearTransformPlaintext(ctx.stc, k) for k in range(2 * n)]
    want, s_out = OB.bootstrap(o, pair.ct_data(ct), pair.scale, c, keys, pair.key(0), cts_pts, stc_pts,
                               replicate=padded)
    assert np.array_equal(pair.ct_data(out), want)
    assert lib.GetCiphertextScale(out) == pytest.approx(s_out, rel=1e-12)


@pytest.mark.parametrize("padded", [False, True])
def test_bootstrap_residues_match_oracle(pair, padded):
    check_residues_match_oracle(pair, padded, asin=False)


def test_bootstrap_keeps_a_drifted_scale(pair):
    """The reference snaps a drifted input scale to the default one before
    Cheddar's fixed-scale Boot and multiplies by 1/r afterwards
    (cheddar_pybind.cu:2156-2185, one level).  This circuit reads the input
    at whatever scale it carries: the output keeps that scale exactly, at
    full precision, with no level spent."""
    n = 16
    rng = np.random.default_rng(11)
    z = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)) * 0.7
    drifted = pair.scale * 1.0123
    vals = np.tile(z, pair.slots // n)
    pt = pair.lib.EncodeComplex(np.stack([vals.real, vals.imag], axis=-1).ravel(), 0, drifted)
    ct = pair.lib.Encrypt(pt)
    pair.lib.DeletePlaintext(pt)
    pair.lib.SetCiphertextSlots(ct, n)
    out = pair.lib.Bootstrap(ct, n)
    assert pair.lib.GetCiphertextScale(out) == pytest.approx(drifted, rel=1e-12)
    assert pair.lib.GetCiphertextLevel(out) == TOP
    assert np.abs(_decrypt_c(pair, out) - vals).max() < 1e-5


def test_bootstrap_batch_equals_single(pair):
    """BootstrapBatch runs the circuit through the batched entry points
    (folds, transforms, rescales, polynomials, products); each output must
    equal Bootstrap of that input residue for residue, mixed sparse and
    zero-padded inputs included."""
    n = 16
    rng = np.random.default_rng(21)
    cts = []
    for i in range(3):
        z = (rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)) * 0.6
        cts.append(_encrypt_sparse(pair, z, n, 0, padded=(i == 1)))
    batch = pair.lib.BootstrapBatch(cts, n)
    for c, b in zip(cts, batch):
        one = pair.lib.Bootstrap(c, n)
        assert np.array_equal(pair.ct_data(b), pair.ct_data(one))
        assert pair.lib.GetCiphertextScale(b) == pair.lib.GetCiphertextScale(one)


def test_message_ratio_is_checked(pair):
    n = 16
    pt = pair.lib.Encode(list(np.zeros(pair.slots)), 0, 2.0 ** 48)
    ct = pair.lib.Encrypt(pt)
    with pytest.raises(RuntimeError, match="message ratio"):
        pair.lib.Bootstrap(ct, n)
    with pytest.raises(ValueError, match="power of two"):
        pair.lib.NewBootstrapper(None, 24)
