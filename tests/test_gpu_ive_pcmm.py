"""The IVE lookup's one-pass table products on the GPU path.

The reference's Cheddar backend gives IVE (examples/criteo/ive_selector.py)
a plaintext-matrix x ciphertext-vector product in one pass over the inputs
(ConstMatMulKernel / PlaintextMatMulKernel, cheddar_pybind.cu:1044-1569;
bindings.py:621-706).  Here: broadcast constants (one word per prime),
constant and plaintext tables, and MulConstantMatMulNew /
MulPlaintextMatMulNew / MulConstantAccumNew.  Every output row must equal
the oracle's multiply-accumulate of the same inputs residue for residue,
and decrypt to the cleartext product.
"""
import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=12, logq=[36] * 5, logp=[60, 60], logscale=36, h=64)
LEVEL = 4


@pytest.fixture(scope="module")
def pair(oracle_mod):
    p = Pair(CFG, dnum=3, seed=20261230, oracle_mod=oracle_mod)
    yield p
    p.close()


def _inputs(pair, p, seed):
    rng = np.random.default_rng(seed)
    xs = [rng.uniform(-1, 1, pair.slots) for _ in range(p)]
    return xs, [pair.encrypt(x, LEVEL) for x in xs]


def test_constant_table_matmul_bit_exact(pair):
    rows, cols, cscale = 20, 12, 2.0 ** 20
    rng = np.random.default_rng(1)
    C = rng.uniform(-1, 1, (rows, cols))
    xs, cts = _inputs(pair, cols, 2)
    kids = [pair.lib.EncodeConstantNew(float(c), LEVEL, cscale) for c in C.ravel()]
    tab = pair.lib.PackConstantTableNew(kids, rows)
    outs = pair.lib.MulConstantMatMulNew(cts, tab)
    assert len(outs) == rows
    q = pair.o.primes[:LEVEL + 1]
    data = [pair.ct_data(c) for c in cts]
    for r in range(rows):
        words = [[int(round(C[r, k] * cscale)) % qi for qi in q] for k in range(cols)]
        pts = [np.repeat(np.array(w, dtype=np.uint64)[:, None], pair.N, axis=1) for w in words]
        assert np.array_equal(pair.ct_data(outs[r]), pair.o.mac(data, pts)), r
        assert pair.lib.GetCiphertextScale(outs[r]) == pytest.approx(pair.scale * cscale)
    got = pair.decrypt(outs[7])
    ref = sum(C[7, k] * xs[k] for k in range(cols))
    assert np.abs(got - ref).max() < 1e-4
    # the one-row form
    acc = pair.lib.MulConstantAccumNew(cts, kids[3 * cols:4 * cols])
    assert np.array_equal(pair.ct_data(acc), pair.ct_data(outs[3]))
    pair.lib.DeleteConstantTable(tab)
    for k in kids:
        pair.lib.DeleteConstant(k)


def test_plaintext_table_matmul_bit_exact(pair):
    rows, cols = 5, 7
    rng = np.random.default_rng(3)
    vals = rng.uniform(-1, 1, (rows, cols, pair.slots))
    xs, cts = _inputs(pair, cols, 4)
    pids = [pair.lib.Encode(list(vals[r, k]), LEVEL, pair.scale) for r in range(rows) for k in range(cols)]
    tab = pair.lib.PackPlaintextTableNew(pids, rows)
    outs = pair.lib.MulPlaintextMatMulNew(cts, tab)
    data = [pair.ct_data(c) for c in cts]
    for r in range(rows):
        pts = [pair.lib.GetPlaintextData(pids[r * cols + k]) for k in range(cols)]
        assert np.array_equal(pair.ct_data(outs[r]), pair.o.mac(data, pts)), r
    got = pair.decrypt(pair.lib.RescaleNew(outs[2]))
    ref = sum(vals[2, k] * xs[k] for k in range(cols))
    assert np.abs(got - ref).max() < 1e-4
    pair.lib.DeletePlaintextTable(tab)


def test_table_level_above_ciphertexts_is_refused(pair):
    xs, cts = _inputs(pair, 2, 5)
    low = [pair.lib.AlignToLevelNew(c, 2) for c in cts]
    kids = [pair.lib.EncodeConstantNew(0.5, LEVEL, 2.0 ** 10) for _ in range(2)]
    tab = pair.lib.PackConstantTableNew(kids, 1)
    with pytest.raises(RuntimeError, match="below the table's level"):
        pair.lib.MulConstantMatMulNew(low, tab)
    with pytest.raises(ValueError, match="expected 2 ciphertexts"):
        pair.lib.MulConstantMatMulNew(cts[:1], tab)
    pair.lib.DeleteConstantTable(tab)
