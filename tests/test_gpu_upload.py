"""The upload side of the path on the GPU: device encoding, the imaginary
unit, and complex-lane unpacking.

Reference: Encode / EncodeComplex (cheddar_pybind.cu:538-580, the encoder
Orion calls per ciphertext), MulImaginaryUnit (cheddar_pybind.cu:1825-1837)
and the HE-LRM selector upload's lane packing (orion/core/lane_packing.py:
60-115, examples/criteo/bench_sweep.py:355-420), with the seeded upload
(EncryptSeeded -> DropAx -> ExpandSeededAx) in front of it.
Encoding must agree with the oracle's canonical embedding to +-1 per
coefficient (two FFTs may round a .5 coefficient differently) and decode
back within 1e-8; the imaginary unit and the lane split must equal the
oracle residue for residue; the fused UnpackLanes must equal the
reference's op-by-op sequence through this backend, residue for residue.
"""
import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig, lanes

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=12, logq=[40, 36, 36, 36, 36], logp=[60, 60], logscale=36, h=64)


@pytest.fixture(scope="module")
def pair(oracle_mod):
    p = Pair(CFG, dnum=2, seed=20261203, oracle_mod=oracle_mod)
    yield p
    p.close()


def _close_coeffs(pair, got, want, rows):
    for i in range(rows):
        q = pair.o.primes[i] if i < pair.o.L else None
        assert q is not None
        d = (pair.o.intt(i, got[i]).astype(object) - pair.o.intt(i, want[i]).astype(object)) % q
        d = np.where(d > q // 2, d - q, d)
        assert np.abs(d.astype(np.int64)).max() <= 1, i


@pytest.mark.parametrize("level,scale_bits", [(4, 36), (2, 40), (0, 30)])
def test_device_encode_matches_oracle(pair, level, scale_bits):
    rng = np.random.default_rng(level)
    vals = rng.uniform(-4, 4, pair.slots)
    scale = 2.0 ** scale_bits
    pt = pair.lib.Encode(list(vals), level, scale)
    got = pair.lib.GetPlaintextData(pt)
    want = pair.o.encode(vals, level + 1, scale)
    _close_coeffs(pair, got, want, level + 1)
    assert np.abs(np.array(pair.lib.Decode(pt)) - vals).max() < 1e-7


def test_device_encode_complex_and_partial(pair):
    rng = np.random.default_rng(9)
    n = 300  # fewer values than slots: the rest are zero
    z = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    inter = np.stack([z.real, z.imag], axis=-1).ravel()
    pt = pair.lib.EncodeComplex(inter, 4, pair.scale)
    full = np.zeros(pair.slots, complex)
    full[:n] = z
    _close_coeffs(pair, pair.lib.GetPlaintextData(pt), pair.o.encode(full, 5, pair.scale), 5)
    back = np.array(pair.lib.DecodeComplex(pt))
    back = back[0::2] + 1j * back[1::2] if back.dtype != complex else back
    assert np.abs(back[:pair.slots] - full).max() < 1e-8


def test_encode_batch_equals_single(pair):
    rng = np.random.default_rng(4)
    vals = rng.uniform(-1, 1, (5, pair.slots))
    ids = pair.lib.EncodeBatch(vals, 3, pair.scale)
    for row, pid in zip(vals, ids):
        one = pair.lib.Encode(list(row), 3, pair.scale)
        assert np.array_equal(pair.lib.GetPlaintextData(pid), pair.lib.GetPlaintextData(one))


def _iunit(pair, nq):
    """NTT of X^(N/2) per prime, from the oracle's own NTT."""
    rows = []
    for i in range(nq):
        mono = np.zeros(pair.N, dtype=np.uint64)
        mono[pair.N // 2] = 1
        rows.append(pair.o.ntt(i, mono))
    return np.array(rows, dtype=object)


def _mul_rows(a, m, qs):
    return ((a.astype(object) * m[None]) % qs).astype(np.uint64)


def test_imaginary_unit_bit_exact(pair):
    rng = np.random.default_rng(2)
    x = rng.uniform(-1, 1, pair.slots)
    ct = pair.encrypt(x, 4)
    out = pair.lib.MulImaginaryUnitNew(ct)
    qs = np.array(pair.o.primes[:5], dtype=object)[None, :, None]
    assert np.array_equal(pair.ct_data(out), _mul_rows(pair.ct_data(ct), _iunit(pair, 5), qs))
    assert pair.lib.GetCiphertextLevel(out) == 4
    got = np.array(pair.lib.DecodeComplex(pair.lib.Decrypt(out)))
    assert np.abs(got[0::2]).max() < 1e-6 and np.abs(got[1::2] - x).max() < 1e-6


def _reference_unpack(lib, packed, num_real):
    """orion/core/lane_packing.py:84-115, op by op through this backend."""
    out = []
    for pid in packed:
        conj = lib.ConjugateNew(pid)
        even = lib.AddCiphertextNew(pid, conj)
        diff = lib.SubCiphertextNew(pid, conj)
        lib.MulImaginaryUnit(diff)
        odd = lib.Negate(diff)
        lib.DeleteCiphertext(conj)
        lib.DeleteCiphertext(diff)
        out.extend([even, odd])
    for s in out[num_real:]:
        lib.DeleteCiphertext(s)
    return out[:num_real]


@pytest.mark.parametrize("num_elements", [3 * 2048, 4 * 2048 - 100])
def test_unpack_lanes(pair, num_elements):
    rng = np.random.default_rng(num_elements)
    values = rng.uniform(-1, 1, num_elements)
    packed_vec, num_real = lanes.pack_lanes(values, pair.slots)
    assert (num_real, len(packed_vec) // pair.slots) == lanes.plan_packing(num_elements, pair.slots)
    pts = lanes.encode_packed(pair.lib, packed_vec, pair.slots, 4, pair.scale)
    packed = [pair.lib.Encrypt(p) for p in pts]
    fused = lanes.unpack_lanes(pair.lib, packed, num_real)
    ref = _reference_unpack(pair.lib, packed, num_real)
    assert len(fused) == len(ref) == num_real
    # the oracle: conjugation with the same key, then p + c and i (c - p)
    g = 2 * pair.N - 1
    key = pair.key(g)
    assert np.array_equal(key, pair.o.rotation_key(pair.sk, pair.seed, g))
    qs = np.array(pair.o.primes[:5], dtype=object)[None, :, None]
    iu = _iunit(pair, 5)
    flat = np.concatenate([values, np.zeros(num_real * pair.slots - num_elements)])
    for m, pid in enumerate(packed):
        p = pair.ct_data(pid)
        c = pair.o.rotate(p, key, g)
        even = ((p.astype(object) + c.astype(object)) % qs).astype(np.uint64)
        odd = _mul_rows((c.astype(object) - p.astype(object)) % qs, iu, qs)
        for lane, want in enumerate([even, odd]):
            r = 2 * m + lane
            if r >= num_real:
                continue
            assert np.array_equal(pair.ct_data(fused[r]), want)
            assert np.array_equal(pair.ct_data(ref[r]), want)
            assert pair.lib.GetCiphertextScale(fused[r]) == pair.lib.GetCiphertextScale(pid)
            got = pair.decrypt(fused[r])
            assert np.abs(got - flat[r * pair.slots:(r + 1) * pair.slots]).max() < 1e-5


def test_seeded_packed_upload(pair):
    """The selector upload of bench_sweep.py:366-420: lane-packed, seeded
    (only b crosses the wire), a rebuilt by ExpandSeededAx, then unpacked."""
    rng = np.random.default_rng(12)
    values = rng.uniform(-1, 1, 2 * pair.slots)
    packed_vec, num_real = lanes.pack_lanes(values, pair.slots)
    pts = lanes.encode_packed(pair.lib, packed_vec, pair.slots, 4, pair.scale)
    seeds = [int(s) for s in rng.integers(1, 2 ** 62, len(pts))]
    cts = [pair.lib.EncryptSeeded(p, s) for p, s in zip(pts, seeds)]
    for c in cts:
        pair.lib.DropAx(c)
    for c, s in zip(cts, seeds):
        pair.lib.ExpandSeededAx(c, s)
    outs = lanes.unpack_lanes(pair.lib, cts, num_real)
    for r, o in enumerate(outs):
        assert np.abs(pair.decrypt(o) - values[r * pair.slots:(r + 1) * pair.slots]).max() < 1e-5


def test_unpack_errors(pair):
    a = pair.encrypt(np.zeros(pair.slots), 4)
    b = pair.encrypt(np.zeros(pair.slots), 3)
    with pytest.raises(RuntimeError, match="share one level"):
        pair.lib.UnpackLanes([a, b], 4)
    with pytest.raises(ValueError):
        pair.lib.UnpackLanes([a], 3)


@pytest.mark.parametrize("level,scale_bits", [(0, 30), (1, 60), (3, 100), (4, 120)])
def test_device_decode_multilimb(pair, level, scale_bits):
    """Decoding runs on the device: Garner's CRT over the first min(l+1, 4)
    limbs, centred, then the special FFT.  Large scales put the
    coefficients beyond the first limbs (40- and 36-bit primes here), so
    the mixed radix and its sign decision are exercised; negative and
    complex values too."""
    rng = np.random.default_rng(scale_bits)
    z = rng.uniform(-3, 3, pair.slots) + 1j * rng.uniform(-3, 3, pair.slots)
    scale = 2.0 ** scale_bits
    # the coefficients round(scale * values) through the oracle's encoder,
    # which handles any scale exactly (integer arithmetic)
    want = pair.o.encode(z, level + 1, scale)
    pt = pair.lib.NewPlaintextFromData(want, level, False, scale)
    got = np.array(pair.lib.DecodeComplex(pt))
    got = got[0::2] + 1j * got[1::2]
    # the encoding's own rounding (half a unit per coefficient, about
    # sqrt(N) / 2 / scale in a slot) plus the FP64 transform's error
    tol = 256.0 / scale + 1e-12
    assert np.abs(got - z).max() < tol
    real = np.array(pair.lib.Decode(pt))
    assert np.abs(real - z.real).max() < tol
