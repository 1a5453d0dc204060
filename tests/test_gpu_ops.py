"""The reference's backend oracle tests, replayed against the B200 backend.

Restates the cases of the reference's tests/oracle/ suite (run there with
--backend=<name>) on the Cheddar-style configuration of
tests/oracle/conftest.py:40-55 (LogN 13, LogQ [29,26,26,26], LogP [29],
scale 2^26, Standard ring), with the same cleartext expectations and
tolerances.
"""
import numpy as np
import pytest

from conftest import assert_fhe_close
from helrm_b200 import B200Library
from helrm_b200.params import TEST_CONFIG

pytestmark = pytest.mark.gpu


class S:
    """Minimal stand-in for the reference's Scheme fixture."""

    def __init__(self):
        self.backend = B200Library(seed=77, device=0)
        self.backend.setup_bindings(TEST_CONFIG)
        for f in ("NewKeyGenerator", "GenerateSecretKey", "GeneratePublicKey", "GenerateRelinearizationKey",
                  "GenerateEvaluationKeys"):
            getattr(self.backend, f)()
        self.slots = TEST_CONFIG.get_slots()
        self.max_level = TEST_CONFIG.get_max_level()
        self.scale = TEST_CONFIG.get_default_scale()

    def enc(self, values, level=None):
        level = self.max_level if level is None else level
        vals = list(values) + [0.0] * (self.slots - len(values))
        return self.backend.Encrypt(self.backend.Encode(vals, level, self.scale))

    def dec(self, ct):
        return np.array(self.backend.Decode(self.backend.Decrypt(ct)))


@pytest.fixture(scope="module")
def s():
    sc = S()
    yield sc
    sc.backend.DeleteScheme()


def test_encode_decode(s):
    vals = np.linspace(-4, 4, s.slots)
    pt = s.backend.Encode(list(vals), s.max_level, s.scale)
    assert_fhe_close(s.backend.Decode(pt), vals, atol=1e-3, msg="encode/decode")
    assert s.backend.GetPlaintextLevel(pt) == s.max_level
    assert s.backend.GetPlaintextScale(pt) == s.scale


def test_encrypt_decrypt_levels(s):
    for level in range(s.max_level + 1):
        vals = np.cos(np.arange(s.slots) + level)
        ct = s.enc(vals, level)
        assert s.backend.GetCiphertextLevel(ct) == level
        assert_fhe_close(s.dec(ct), vals, atol=1e-2, msg=f"level {level}")


def test_add_sub(s):
    a, b = np.linspace(0, 1, s.slots), np.linspace(1, 3, s.slots)
    ca, cb = s.enc(a), s.enc(b)
    assert_fhe_close(s.dec(s.backend.AddCiphertextNew(ca, cb)), a + b, msg="add")
    assert_fhe_close(s.dec(s.backend.SubCiphertextNew(ca, cb)), a - b, msg="sub")
    pb = s.backend.Encode(list(b), s.max_level, s.scale)
    assert_fhe_close(s.dec(s.backend.AddPlaintextNew(ca, pb)), a + b, msg="add pt")
    assert_fhe_close(s.dec(s.backend.SubPlaintextNew(ca, pb)), a - b, msg="sub pt")
    c = s.enc(a)
    s.backend.AddCiphertext(c, cb)
    assert_fhe_close(s.dec(c), a + b, msg="add in place")
    assert_fhe_close(s.dec(s.backend.Negate(s.enc(a))), -a, msg="negate")


def test_add_aligns_levels(s):
    a, b = np.linspace(0, 1, s.slots), np.linspace(1, 3, s.slots)
    ca, cb = s.enc(a, 3), s.enc(b, 1)
    out = s.backend.AddCiphertextNew(ca, cb)
    assert s.backend.GetCiphertextLevel(out) == 1
    assert_fhe_close(s.dec(out), a + b, msg="level alignment")


def test_scalar_ops(s):
    """reference tests/oracle/test_eval_scalar.py and test_eval_rescale.py:19-26,83-89"""
    a = np.linspace(-1, 1, s.slots)
    ca = s.enc(a)
    assert_fhe_close(s.dec(s.backend.AddScalarNew(ca, 2.5)), a + 2.5, msg="add scalar")
    assert_fhe_close(s.dec(s.backend.SubScalarNew(ca, 0.5)), a - 0.5, msg="sub scalar")
    mi = s.backend.MulScalarIntNew(ca, 3)
    assert s.backend.GetCiphertextLevel(mi) == s.max_level
    assert_fhe_close(s.dec(mi), 3 * a, msg="mul int")
    mf = s.backend.Rescale(s.backend.MulScalarFloatNew(ca, 0.25))
    assert s.backend.GetCiphertextLevel(mf) == s.max_level - 1
    assert_fhe_close(s.dec(mf), 0.25 * a, msg="mul float")


def test_mul_plaintext_consumes_a_level(s):
    """reference tests/oracle/test_eval_plaintext.py:76-114"""
    a, b = np.linspace(-1, 1, s.slots), np.linspace(2, -2, s.slots)
    ct = s.enc(a)
    pt = s.backend.Encode(list(b), s.max_level, s.scale)
    out = s.backend.Rescale(s.backend.MulPlaintextNew(ct, pt))
    assert s.backend.GetCiphertextLevel(out) == s.max_level - 1
    assert_fhe_close(s.dec(out), a * b, msg="ct x pt")


def test_mul_ciphertext(s):
    a, b = np.linspace(-1, 1, s.slots), np.linspace(2, -2, s.slots)
    out = s.backend.Rescale(s.backend.MulRelinCiphertextNew(s.enc(a), s.enc(b)))
    assert_fhe_close(s.dec(out), a * b, msg="ct x ct")


@pytest.mark.parametrize("k", [1, 2, 5, -1, -7])
def test_rotation_direction(s, k):
    """reference tests/oracle/test_eval_rotate.py:29-91: +k is a left shift."""
    vals = np.arange(1, s.slots + 1, dtype=np.float64)
    out = s.backend.RotateNew(s.enc(vals), k)
    assert_fhe_close(s.dec(out), np.roll(vals, -k), atol=1e-1, msg=f"rotate {k}")


def test_rotate_batch(s):
    vals = np.arange(s.slots, dtype=np.float64) / s.slots
    ct = s.enc(vals)
    outs = s.backend.RotateBatchNew(ct, [0, 1, 3, 3])
    for k, o in zip([0, 1, 3, 3], outs):
        assert_fhe_close(s.dec(o), np.roll(vals, -k), msg=f"batch {k}")


def test_polynomial_horner(s):
    a = np.linspace(-1, 1, s.slots)
    pid = s.backend.GenerateMonomial([0.5, -1.0, 2.0])  # ascending: 0.5 - x + 2x^2
    out = s.backend.EvaluatePolynomial(s.enc(a), pid, s.scale)
    assert_fhe_close(s.dec(out), 0.5 - a + 2 * a * a, atol=5e-2, msg="poly")


def _lt(s, diags_idxs, diags_data, level, ratio):
    lt = s.backend.GenerateLinearTransform(diags_idxs, diags_data, level, ratio, "none")
    for key in s.backend.GetLinearTransformRotationKeys(lt):
        s.backend.GenerateLinearTransformRotationKey(key)
    return lt


def _run(s, lt, ct):
    out = s.backend.EvaluateLinearTransform(lt, ct)
    if not getattr(s.backend, "lt_output_prerescaled", False):
        out = s.backend.Rescale(out)
    return s.dec(out)


def test_lt_identity(s):
    values = [float(i + 1) for i in range(s.slots)]
    lt = _lt(s, [0], [1.0] * s.slots, s.max_level, 1.0)
    assert_fhe_close(_run(s, lt, s.enc(values)), values, atol=1e-1, msg="identity transform")


def test_lt_scale(s):
    values = [float(i + 1) for i in range(s.slots)]
    lt = _lt(s, [0], [3.0] * s.slots, s.max_level, 1.0)
    assert_fhe_close(_run(s, lt, s.enc(values)), [3 * v for v in values], atol=5e-1, msg="scale transform")


def test_lt_cyclic_permutation(s):
    values = [float(i + 1) for i in range(s.slots)]
    lt = _lt(s, [3], [1.0] * s.slots, s.max_level, 1.0)
    exp = [values[(i + 3) % s.slots] for i in range(s.slots)]
    assert_fhe_close(_run(s, lt, s.enc(values)), exp, atol=1e-1, msg="permute by 3")


def test_lt_multi_diagonal(s):
    values = [float(i + 1) for i in range(s.slots)]
    lt = _lt(s, [0, 1], [1.0] * s.slots * 2, s.max_level, 1.0)
    exp = [values[i] + values[(i + 1) % s.slots] for i in range(s.slots)]
    assert_fhe_close(_run(s, lt, s.enc(values)), exp, atol=5e-1, msg="multi-diagonal")


def test_lt_input_above_transform_level(s):
    values = [float(i % 7) - 3.0 for i in range(s.slots)]
    lt = _lt(s, [0, 1], [2.0] * s.slots + [1.0] * s.slots, 1, 1.0)
    exp = [2.0 * values[i] + values[(i + 1) % s.slots] for i in range(s.slots)]
    assert_fhe_close(_run(s, lt, s.enc(values)), exp, atol=5e-1, msg="input above transform level")


def test_lt_input_above_transform_level_bsgs(s):
    values = [float((i * 5) % 11) - 5.0 for i in range(s.slots)]
    idx = [0, 1, 2, 5, 8]
    data = []
    for d in idx:
        data += [float(d + 1)] * s.slots
    lt = _lt(s, idx, data, 1, 2.0)
    exp = [sum((d + 1.0) * values[(i + d) % s.slots] for d in idx) for i in range(s.slots)]
    assert_fhe_close(_run(s, lt, s.enc(values)), exp, atol=5e-1, msg="input above transform level (bsgs)")


@pytest.mark.parametrize("num_diags", [50, 100, 144])
def test_bsgs_stress(s, num_diags):
    """reference tests/test_bsgs_linear_transform.py:195-235"""
    rng = np.random.default_rng(seed=42 + num_diags)
    values = [float(i % 17) * 0.1 for i in range(s.slots)]
    idx = sorted(rng.choice(s.slots, size=num_diags, replace=False).tolist())
    w = rng.uniform(-0.5, 0.5, size=num_diags).tolist()
    data = []
    for wi in w:
        data.extend([wi] * s.slots)
    lt = _lt(s, idx, data, s.max_level, 2)
    exp = [sum(wi * values[(i + d) % s.slots] for d, wi in zip(idx, w)) for i in range(s.slots)]
    assert_fhe_close(_run(s, lt, s.enc(values)), exp, atol=1.0, msg=f"BSGS stress {num_diags} diagonals")
    s.backend.DeleteLinearTransform(lt)


def test_bsgs_vs_naive(s):
    rng = np.random.default_rng(seed=99)
    values = [float(i % 13) * 0.2 for i in range(s.slots)]
    idx = sorted(rng.choice(s.slots, size=30, replace=False).tolist())
    w = rng.uniform(-0.3, 0.3, size=30).tolist()
    data = []
    for wi in w:
        data.extend([wi] * s.slots)
    a = _run(s, _lt(s, idx, data, s.max_level, 2), s.enc(values))
    b = _run(s, _lt(s, idx, data, s.max_level, "none"), s.enc(values))
    assert_fhe_close(a, b, atol=1.0, msg="BSGS vs naive consistency")


def test_errors_are_exceptions(s):
    with pytest.raises(IndexError):
        s.backend.GetCiphertextLevel(987654)
    ct0 = s.enc([1.0], 0)
    with pytest.raises(RuntimeError):
        s.backend.RescaleNew(ct0)
    a = s.enc([1.0])
    b = s.enc([1.0])
    s.backend.SetCiphertextScale(b, s.scale * 1.5)
    with pytest.raises(RuntimeError):
        s.backend.AddCiphertextNew(a, b)
    with pytest.raises(ValueError):
        s.backend.Encode([0.0] * (s.slots + 1), 0, s.scale)
    with pytest.raises(NotImplementedError):
        s.backend.SerializeDiagonal(1, 0)


def test_live_counts_and_memory(s):
    n0 = s.backend.GetLiveCiphertexts()
    ct = s.enc([1.0])
    assert s.backend.GetLiveCiphertexts() == n0 + 1
    s.backend.DeleteCiphertext(ct)
    assert s.backend.GetLiveCiphertexts() == n0
    assert s.backend.GetKeyMemoryMB() > 0
    assert s.backend.GetPeakLiveMemoryMB() >= s.backend.GetLiveMemoryMB()


def test_mul_relin_batch_equals_per_pair(s):
    """MulRelinCiphertextBatchNew: the pairs of each level in one batched
    tensor product and relinearisation, residue for residue what
    MulRelinCiphertextNew gives pair by pair (mixed levels, a squaring,
    operands at different levels)."""
    lib = s.backend
    rng = np.random.default_rng(31)
    top = s.max_level
    cts = [s.enc(rng.uniform(-1, 1, s.slots), lvl) for lvl in (top, top, top - 1, top, top - 1)]
    a_ids = [cts[0], cts[1], cts[2], cts[3], cts[0]]
    b_ids = [cts[1], cts[1], cts[4], cts[2], cts[0]]
    got = lib.MulRelinCiphertextBatchNew(a_ids, b_ids)
    assert len(set(got)) == len(got)
    for a, b, g in zip(a_ids, b_ids, got):
        want = lib.MulRelinCiphertextNew(a, b)
        assert np.array_equal(lib.GetCiphertextData(g), lib.GetCiphertextData(want))
        assert lib.GetCiphertextScale(g) == lib.GetCiphertextScale(want)
        assert lib.GetCiphertextLevel(g) == lib.GetCiphertextLevel(want)
        lib.DeleteCiphertext(want)
        lib.DeleteCiphertext(g)
    assert lib.MulRelinCiphertextBatchNew([], []) == []
    with pytest.raises(ValueError):
        lib.MulRelinCiphertextBatchNew([cts[0]], [])
