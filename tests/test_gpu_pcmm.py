"""The HE-LRM embedding PCMM end to end on the B200 path.

cfg1: single 1024 x 16 table, base-32 digits,
LogN 13 -- bit-exact against the oracle and within tolerance of the
cleartext lookup.  cfg2: the 26-table block-diagonal
416 x 4224 matrix at LogN 16, 24 limbs + 4 special primes, dnum 4, the
whole step (LT, rescale, fold) on a batch of two -- every residue against
the oracle, and the decrypted embedding slots against the cleartext matrix
product.  cfg3 primitives at that size, bit-exact: NTT/INTT on
a batch of 16 ciphertexts, the hoisted key switch for 32 rotations, MAC
and rescale.

Tolerance on embedding slots: the error of every
output slot is at most 2^-15 relative to the largest embedding magnitude.
"""
import ctypes

import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import workload as W
from helrm_b200.params import CFG1, CFG2, CFG2_DNUM

pytestmark = pytest.mark.gpu

REL_TOL = 2.0 ** -15


def _pcmm(pair, M, xs, level, ratio=2.0):
    slots = pair.slots
    d, rot = W.diagonalize(M, slots, "hybrid")
    diags = d[(0, 0)]
    ks = sorted(diags)
    data = np.concatenate([diags[k].astype(np.float64) for k in ks])
    lt = pair.lib.GenerateLinearTransform(ks, data, level, ratio, "none")
    for k in pair.lib.GetLinearTransformRotationKeys(lt):
        pair.lib.GenerateLinearTransformRotationKey(k)
    for i in range(1, rot + 1):
        pair.lib.AddRotationKey(slots >> i)
    cts = []
    for x in xs:
        v = np.zeros(slots)
        v[:len(x)] = x
        cts.append(pair.encrypt(v, level))
    outs = pair.lib.EvaluateLinearTransformBatch(lt, cts)
    pair.lib.RescaleBatch(outs)
    pair.lib.HybridFoldBatch(outs, rot)
    return lt, ks, diags, rot, cts, outs


@pytest.fixture(scope="module")
def cfg1(oracle_mod):
    p = Pair(CFG1, dnum=5, seed=101, oracle_mod=oracle_mod)
    yield p
    p.close()


def test_cfg1_pcmm(cfg1):
    M = W.cfg1_matrix()
    idx, sel = W.cfg1_queries(3)
    lt, ks, diags, rot, cts, outs = _pcmm(cfg1, M, sel, cfg1.info["max_level"])
    assert len(ks) == 16 and rot == 8
    for x, o in zip(sel, outs):
        got = cfg1.decrypt(o)[:16]
        ref = M.astype(np.float64) @ x
        assert np.abs(got - ref).max() <= REL_TOL * np.abs(ref).max()


def test_cfg1_lt_bit_exact(cfg1):
    M = W.cfg1_matrix()
    _, sel = W.cfg1_queries(1, seed=5)
    level = cfg1.info["max_level"]
    d, rot = W.diagonalize(M, cfg1.slots, "hybrid")
    ks = sorted(d[(0, 0)])
    data = np.concatenate([d[(0, 0)][k].astype(np.float64) for k in ks])
    lt = cfg1.lib.GenerateLinearTransform(ks, data, level, 2.0, "none")
    plan = W.bsgs_plan(ks, 2.0, cfg1.slots)
    for k in plan["rotation_keys"]:
        cfg1.lib.AddRotationKey(k)
    v = np.zeros(cfg1.slots)
    v[:64] = sel[0]
    ct = cfg1.encrypt(v, level)
    out = cfg1.lib.EvaluateLinearTransform(lt, ct)
    pts = [cfg1.lib.GetLinearTransformPlaintext(lt, k) for k in ks]
    keys = {cfg1.o.galois(k): cfg1.key(cfg1.o.galois(k)) for k in plan["rotation_keys"]}
    want = cfg1.o.bsgs_lt(cfg1.ct_data(ct), ks, pts, plan["stride"], keys)
    assert np.array_equal(cfg1.ct_data(out), want)


@pytest.fixture(scope="module")
def cfg2(oracle_mod):
    p = Pair(CFG2, dnum=CFG2_DNUM, seed=202, oracle_mod=oracle_mod)
    assert p.info["alpha"] == 6 and p.info["dnum"] == 4 and p.info["L"] == 24 and p.info["K"] == 4
    yield p
    p.close()


def test_cfg3_ntt_bit_exact(cfg2):
    import torch
    from helrm_b200 import _capi
    lib = _capi.load()
    rng = np.random.default_rng(3)
    nq, K, N = 24, 4, cfg2.N
    primes = cfg2.o.primes
    rows = nq + K
    host = np.stack([rng.integers(0, primes[i if i < nq else 24 + i - nq], N, dtype=np.uint64)
                     for i in range(rows)])
    dev = torch.from_numpy(host.view(np.int64).copy()).cuda()
    _capi.check(lib.helrm_kernel_ntt(ctypes.c_void_p(dev.data_ptr()), rows, rows, nq, 0, None))
    _capi.check(lib.helrm_Synchronize())
    fwd = dev.cpu().numpy().view(np.uint64)
    for r in range(rows):
        p = r if r < nq else 24 + r - nq
        assert np.array_equal(fwd[r], cfg2.o.ntt(p, host[r])), r
    _capi.check(lib.helrm_kernel_ntt(ctypes.c_void_p(dev.data_ptr()), rows, rows, nq, 1, None))
    _capi.check(lib.helrm_Synchronize())
    assert np.array_equal(dev.cpu().numpy().view(np.uint64), host)


def test_cfg3_hoisted_keyswitch_bit_exact(cfg2):
    ct = cfg2.encrypt(np.cos(np.arange(cfg2.slots) / 100.0))
    ks = [1, 31]
    outs = cfg2.lib.RotateBatchNew(ct, ks)
    data = cfg2.ct_data(ct)
    for k, o in zip(ks, outs):
        g = cfg2.o.galois(k)
        assert np.array_equal(cfg2.ct_data(o), cfg2.o.rotate(data, cfg2.key(g), g)), k


def test_cfg3_rescale_and_mac_bit_exact(cfg2):
    rng = np.random.default_rng(6)
    cts = [cfg2.encrypt(rng.uniform(-1, 1, cfg2.slots)) for _ in range(2)]
    pts = [cfg2.lib.Encode(list(rng.uniform(-1, 1, cfg2.slots)), 23, cfg2.scale) for _ in range(2)]
    m = cfg2.lib.MulPlaintextAccumNew(cts, pts)
    want = cfg2.o.mac([cfg2.ct_data(c) for c in cts], [cfg2.lib.GetPlaintextData(p) for p in pts])
    assert np.array_equal(cfg2.ct_data(m), want)
    r = cfg2.lib.RescaleNew(m)
    assert np.array_equal(cfg2.ct_data(r), cfg2.o.rescale(want))


@pytest.fixture(scope="module")
def cfg2_pcmm(cfg2):
    """The headline step at its own shape on a batch of two ciphertexts:
    the 512-diagonal block-diagonal LT (bs 32, 16 giant groups), the
    rescale and the six hybrid-fold rotations, through the batch entry
    points the bench times."""
    V = W.cfg2_vocab()
    M = W.block_diag_matrix(V, 64, 16, 0.05, seed=0)
    q = W.zipf_queries(V, 2)
    xs = [W.selector(qq, V) for qq in q]
    lt, ks, diags, rot, cts, outs = _pcmm(cfg2, M, xs, cfg2.info["max_level"])
    return M, xs, lt, ks, rot, cts, outs


def test_cfg2_pcmm_embedding_slots(cfg2, cfg2_pcmm):
    M, xs, lt, ks, rot, cts, outs = cfg2_pcmm
    info = cfg2.lib.GetLinearTransformInfo(lt)
    assert info["bs"] == 32 and info["n_diags"] == 512 and info["n_giant"] == 16
    for x, o in zip(xs, outs):
        got = cfg2.decrypt(o)[:416]
        ref = M.astype(np.float64) @ x
        err = np.abs(got - ref).max()
        assert err <= REL_TOL * np.abs(ref).max(), err
        assert cfg2.lib.GetCiphertextLevel(o) == 22


def test_cfg2_pcmm_residues_bit_exact(cfg2, cfg2_pcmm):
    """Every residue of the headline step (LogN 16, 24 q + 4 special primes,
    dnum 4, 512 diagonals, batch of two) equals the oracle's LT -> rescale ->
    fold on the same ciphertexts, plaintext diagonals and switching keys:
    the fixed-shape fused kernels (four digits, full 32-baby chunks, giant
    steps three per key multiplication, the fold's add inside ModDown) at
    the size the bench times."""
    import os
    M, xs, lt, ks, rot, cts, outs = cfg2_pcmm
    o = cfg2.o
    cfg2.om.set_threads(os.cpu_count() or 1)
    try:
        plan = W.bsgs_plan(ks, 2.0, cfg2.slots)
        gal = {o.galois(d) for d in plan["rotation_keys"]} | {o.galois(cfg2.slots >> i) for i in range(1, rot + 1)}
        keys = {g: cfg2.key(g) for g in sorted(gal)}
        pts = [cfg2.lib.GetLinearTransformPlaintext(lt, k) for k in ks]
        for c, out in zip(cts, outs):
            want = o.pcmm(cfg2.ct_data(c), ks, pts, plan["stride"], keys, rot)
            got = cfg2.ct_data(out)
            assert got.shape == want.shape == (2, 23, cfg2.N)
            assert np.array_equal(got, want)
    finally:
        cfg2.om.set_threads(1)


def test_cfg3_hoisted_keyswitch_r32_bit_exact(cfg2):
    """The config-3 hoisted key switch at its own size: 32 rotations of one
    ciphertext sharing one ModUp, every output residue against the oracle."""
    import os
    ct = cfg2.encrypt(np.sin(np.arange(cfg2.slots) / 77.0))
    ks = list(range(1, 33))
    outs = cfg2.lib.RotateBatchNew(ct, ks)
    data = cfg2.ct_data(ct)
    gs = [cfg2.o.galois(k) for k in ks]
    cfg2.om.set_threads(os.cpu_count() or 1)
    try:
        want = cfg2.o.rotate_hoisted(data, [cfg2.key(g) for g in gs], gs)
    finally:
        cfg2.om.set_threads(1)
    for i, o in enumerate(outs):
        assert np.array_equal(cfg2.ct_data(o), want[i]), ks[i]


def test_cfg3_ntt_batch16_bit_exact(cfg2):
    """Forward and inverse NTT on a config-3 batch of 16 ciphertexts
    (768 limbs of 2^16 residues, the microbenchmark's layout) against the
    oracle's NTT of every limb."""
    import torch
    from helrm_b200 import _capi
    lib = _capi.load()
    B, nq, N = 16, 24, cfg2.N
    primes = cfg2.o.primes
    rng = np.random.default_rng(16)
    host = np.empty((B, 2, nq, N), dtype=np.uint64)
    for i in range(nq):
        host[:, :, i] = rng.integers(0, primes[i], (B, 2, N), dtype=np.uint64)
    dev = torch.from_numpy(host.view(np.int64).copy()).cuda()
    rows = B * 2 * nq
    _capi.check(lib.helrm_kernel_ntt(ctypes.c_void_p(dev.data_ptr()), rows, nq, nq, 0, None))
    _capi.check(lib.helrm_Synchronize())
    fwd = dev.cpu().numpy().view(np.uint64).reshape(B, 2, nq, N)
    for b in range(B):
        for pl in range(2):
            for i in range(nq):
                assert np.array_equal(fwd[b, pl, i], cfg2.o.ntt(i, host[b, pl, i])), (b, pl, i)
    _capi.check(lib.helrm_kernel_ntt(ctypes.c_void_p(dev.data_ptr()), rows, nq, nq, 1, None))
    _capi.check(lib.helrm_Synchronize())
    assert np.array_equal(dev.cpu().numpy().view(np.uint64).reshape(B, 2, nq, N), host)


def test_cfg2_pcmm_bench_ratio_bit_exact(cfg2):
    """The headline step as the bench runs it (bsgs_ratio 8: bs 64, two full
    baby chunks over 8 giant slots, the paired-item MAC kernel), batch of
    two, every residue against the oracle at the same split."""
    import os
    V = W.cfg2_vocab()
    M = W.block_diag_matrix(V, 64, 16, 0.05, seed=0)
    xs = [W.selector(qq, V) for qq in W.zipf_queries(V, 2, seed=5)]
    lt, ks, diags, rot, cts, outs = _pcmm(cfg2, M, xs, cfg2.info["max_level"], ratio=8.0)
    info = cfg2.lib.GetLinearTransformInfo(lt)
    assert info["bs"] == 64 and info["n_giant"] == 8
    o = cfg2.o
    cfg2.om.set_threads(os.cpu_count() or 1)
    try:
        plan = W.bsgs_plan(ks, 8.0, cfg2.slots)
        gal = {o.galois(d) for d in plan["rotation_keys"]} | {o.galois(cfg2.slots >> i) for i in range(1, rot + 1)}
        keys = {g: cfg2.key(g) for g in sorted(gal)}
        pts = [cfg2.lib.GetLinearTransformPlaintext(lt, k) for k in ks]
        for x, c, out in zip(xs, cts, outs):
            want = o.pcmm(cfg2.ct_data(c), ks, pts, plan["stride"], keys, rot)
            assert np.array_equal(cfg2.ct_data(out), want)
            got = cfg2.decrypt(out)[:416]
            ref = M.astype(np.float64) @ x
            assert np.abs(got - ref).max() <= REL_TOL * np.abs(ref).max()
    finally:
        cfg2.om.set_threads(1)
    cfg2.lib.DeleteLinearTransform(lt)
