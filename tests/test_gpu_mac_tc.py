"""Bit-exact parity of the tensor-core baby-step MAC (hb_bsgs_tc.cuh).

With HELRM_B200_MAC=tc set when the scheme is created and every q prime
below 2^37, the double-hoisted BSGS transform runs the diagonal MAC of the
q rows on the tcgen05 tensor cores: the baby rotations and the plaintexts
are split into byte planes, multiplied as int8 matrices with int32
accumulators in TMEM, and recombined exactly modulo q.  The result must
equal the oracle's residue for residue.  These cases cover the kernel's
shapes: a full 32-baby chunk with four digits, a partial chunk, a chunk of
40 babies (two baby groups, the second accumulating into the inner sums the
first wrote), inputs below the transform's level (three, two and one
digit), and batches that span two 32-ciphertext passes.  Each test also
checks from the library's profiler that the tensor-core kernel is the one
that ran.
"""
import ctypes
import os

import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig, _capi
from helrm_b200 import workload as W

pytestmark = pytest.mark.gpu

# every q prime near 2^36 (below 2^37); dnum 4 -> alpha 2, four digits at level 7
CFGT = CKKSConfig(logn=12, logq=[36] * 8, logp=[60, 60], logscale=36, h=64)


@pytest.fixture(scope="module")
def pair(oracle_mod):
    old = os.environ.get("HELRM_B200_MAC")
    os.environ["HELRM_B200_MAC"] = "tc"
    try:
        p = Pair(CFGT, dnum=4, seed=20261210, oracle_mod=oracle_mod)
    finally:
        if old is None:
            os.environ.pop("HELRM_B200_MAC", None)
        else:
            os.environ["HELRM_B200_MAC"] = old
    assert p.info["alpha"] == 2 and p.info["dnum"] == 4
    assert max(p.lib.GetModuliChain()) < 2 ** 37
    yield p
    p.close()


def _mma_launches(run):
    """launches of the tensor-core MAC class while `run()` executes"""
    capi = _capi.load()
    _capi.check(capi.helrm_ProfileEnable(1))
    try:
        run()
        K = 16
        ms, by, wk = (ctypes.c_double * K)(), (ctypes.c_double * K)(), (ctypes.c_double * K)()
        n = (ctypes.c_uint64 * K)()
        nc = ctypes.c_int(0)
        _capi.check(capi.helrm_ProfileRead(ms, by, wk, n, K, ctypes.byref(nc)))
        buf = ctypes.create_string_buffer(64)
        for i in range(nc.value):
            capi.helrm_KernelClassName(i, buf, 64)
            if buf.value.decode() == "bsgs_mac_mma":
                return int(n[i])
        return 0
    finally:
        _capi.check(capi.helrm_ProfileEnable(0))


def _check_lt(pair, ks, ratio, level_lt, level_in, nbatch, seed, expect_passes):
    rng = np.random.default_rng(seed)
    slots = pair.slots
    diags = {k: rng.uniform(-0.5, 0.5, slots) for k in ks}
    lt = pair.lib.GenerateLinearTransform(ks, np.concatenate([diags[k] for k in ks]), level_lt, ratio, "none")
    plan = W.bsgs_plan(ks, ratio, slots)
    for kk in pair.lib.GetLinearTransformRotationKeys(lt):
        pair.lib.GenerateLinearTransformRotationKey(kk)
    xs = [rng.uniform(-1, 1, slots) for _ in range(nbatch)]
    cts = [pair.encrypt(x, level_in) for x in xs]
    holder = {}
    launches = _mma_launches(lambda: holder.setdefault("outs", pair.lib.EvaluateLinearTransformBatch(lt, cts)))
    outs = holder["outs"]
    assert launches == expect_passes, launches
    # the oracle takes plaintexts over the input's own q rows + the special rows
    nq = level_in + 1
    pts = [pair.lib.GetLinearTransformPlaintext(lt, k) for k in ks]
    pts = [np.concatenate([p[:nq], p[level_lt + 1:]]) for p in pts]
    keys = {pair.o.galois(d): pair.key(pair.o.galois(d)) for d in plan["rotation_keys"]}
    for c, o in zip(cts, outs):
        want = pair.o.bsgs_lt(pair.ct_data(c), ks, pts, plan["stride"], keys)
        assert np.array_equal(pair.ct_data(o), want)
    got = pair.decrypt(pair.lib.RescaleNew(outs[0]))
    assert np.abs(got - W.cleartext_lt(xs[0], diags, slots)).max() < 1e-3
    pair.lib.DeleteLinearTransform(lt)


def test_tc_full_chunk_four_digits_two_passes(pair):
    # babies 0..31 all present, giants 0, 1, 3, 4 (bs 32); 33 ciphertexts:
    # a pass of 32 and a pass of 1
    ks = list(range(64)) + [96, 97, 130]
    _check_lt(pair, ks, 15.2, 7, 7, 33, seed=1, expect_passes=2)


def test_tc_partial_chunk_three_digits(pair):
    # 64 diagonals, ratio 2: bs 12, six giant slots; input at level 4 (three digits)
    _check_lt(pair, list(range(64)), 2.0, 7, 4, 3, seed=2, expect_passes=1)


def test_tc_two_baby_groups_two_digits(pair):
    # bs 40: babies 0..39 in two groups of the same chunk, the second adding
    # into the inner sums the first wrote; input at level 2 (two digits)
    _check_lt(pair, list(range(80)), 20.0, 7, 2, 2, seed=3, expect_passes=2)


def test_tc_one_digit(pair):
    # input at level 1: two q limbs, one digit
    _check_lt(pair, [0, 1, 2, 3, 5, 8], 2.0, 7, 1, 4, seed=4, expect_passes=1)
