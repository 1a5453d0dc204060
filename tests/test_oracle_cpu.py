"""The CPU oracle, pinned before anything is compared against it.

Pins: the O(N^2) negacyclic definition of the NTT; the reference's own
prime rule and diagonal extraction (golden fixtures made by
tests/golden/make_golden.py from the reference's Python); and the
reference's cleartext-tolerance linear-transform tests
(tests/oracle/test_linear_transform.py, tests/test_bsgs_linear_transform.py
of the reference), replayed through the oracle's CKKS at small N.
"""
import math

import numpy as np
import pytest

from conftest import assert_fhe_close


def test_gen_primes_matches_reference(oracle_mod, golden_primes):
    for name, g in golden_primes.items():
        main, aux = oracle_mod.scheme_primes(g["logq"], g["logp"], g["logn"])
        assert main == g["main"], name
        assert aux == g["aux"], name
        for p in main + aux:
            assert p % (2 << g["logn"]) == 1


@pytest.fixture(scope="module")
def small(oracle_mod):
    logn = 10
    main, aux = oracle_mod.scheme_primes([40, 36, 36, 36], [50, 50], logn)
    o = oracle_mod.Oracle(logn, main, aux, dnum=2)
    s = o.sample_secret(7, 64)
    sk = o.secret_ntt(s)
    return o, s, sk


@pytest.mark.parametrize("logn", [4, 7, 10])
def test_ntt_matches_naive_definition(oracle_mod, logn):
    main, aux = oracle_mod.scheme_primes([36, 40], [50], logn)
    o = oracle_mod.Oracle(logn, main, aux, dnum=1)
    rng = np.random.default_rng(logn)
    for p in range(3):
        a = rng.integers(0, o.primes[p], o.N, dtype=np.uint64)
        assert np.array_equal(o.ntt(p, a), o.ntt_naive(p, a))
        assert np.array_equal(o.intt(p, o.ntt(p, a)), a)


def test_ntt_is_negacyclic_convolution(small):
    o, _, _ = small
    rng = np.random.default_rng(3)
    q = o.primes[1]
    a = rng.integers(0, 50, o.N).astype(object)
    b = rng.integers(0, 50, o.N).astype(object)
    c = [0] * o.N
    for i in range(o.N):
        for j in range(o.N):
            k = i + j
            if k < o.N:
                c[k] += a[i] * b[j]
            else:
                c[k - o.N] -= a[i] * b[j]
    c = np.array([x % q for x in c], dtype=np.uint64)
    A = o.ntt(1, np.array(a, dtype=np.uint64))
    B = o.ntt(1, np.array(b, dtype=np.uint64))
    prod = np.array([(int(x) * int(y)) % q for x, y in zip(A, B)], dtype=np.uint64)
    assert np.array_equal(o.intt(1, prod), c)


def test_secret_hamming_weight(small):
    o, s, _ = small
    assert np.count_nonzero(s) == 64
    assert set(np.unique(s)) <= {-1, 0, 1}


def test_encode_decode_round_trip(small):
    o, _, _ = small
    rng = np.random.default_rng(5)
    z = rng.uniform(-1, 1, o.N // 2) + 1j * rng.uniform(-1, 1, o.N // 2)
    pt = o.encode(z, 4, 2.0 ** 36)
    back = o.decode(pt, 2.0 ** 36, complex_out=True)
    assert np.abs(back - z).max() < 1e-8


def test_encrypt_decrypt(small):
    o, _, sk = small
    vals = np.linspace(-1, 1, o.N // 2)
    ct = o.encrypt(sk, o.encode(vals, 4, 2.0 ** 36), 99)
    assert_fhe_close(o.decode(o.decrypt(sk, ct), 2.0 ** 36), vals, atol=1e-6, msg="encrypt/decrypt")


@pytest.mark.parametrize("k", [1, 3, -2, 511])
def test_rotation_is_left_shift(small, k):
    """rot(ct,k)[i] = ct[i+k] (reference tests/oracle/assumptions.md:5-9)."""
    o, _, sk = small
    vals = np.arange(o.N // 2, dtype=np.float64) / o.N
    ct = o.encrypt(sk, o.encode(vals, 4, 2.0 ** 36), 1)
    g = o.galois(k)
    out = o.rotate(ct, o.rotation_key(sk, 1234, g), g)
    assert_fhe_close(o.decode(o.decrypt(sk, out), 2.0 ** 36), np.roll(vals, -k), atol=1e-6, msg=f"rot {k}")


def test_conjugation(small):
    o, _, sk = small
    rng = np.random.default_rng(9)
    z = rng.uniform(-1, 1, o.N // 2) + 1j * rng.uniform(-1, 1, o.N // 2)
    ct = o.encrypt(sk, o.encode(z, 4, 2.0 ** 36), 2)
    g = o.conj_galois()
    out = o.rotate(ct, o.rotation_key(sk, 1234, g), g)
    back = o.decode(o.decrypt(sk, out), 2.0 ** 36, complex_out=True)
    assert np.abs(back - np.conj(z)).max() < 1e-6


def test_hoisted_batch_equals_single_rotations(small):
    o, _, sk = small
    vals = np.sin(np.arange(o.N // 2))
    ct = o.encrypt(sk, o.encode(vals, 4, 2.0 ** 36), 3)
    gs = [o.galois(k) for k in (1, 2, 7)]
    keys = [o.rotation_key(sk, 1234, g) for g in gs]
    batch = o.rotate_hoisted(ct, keys, gs)
    for i, g in enumerate(gs):
        assert np.array_equal(batch[i], o.rotate(ct, keys[i], g))


def test_mul_plain_rescale(small):
    """ct x pt consumes one level (reference tests/oracle/test_eval_plaintext.py:76-114)."""
    o, _, sk = small
    vals = np.linspace(-1, 1, o.N // 2)
    ct = o.encrypt(sk, o.encode(vals, 4, 2.0 ** 36), 4)
    pt = o.encode(np.full(o.N // 2, 0.5), 4, o.primes[3])
    out = o.rescale(o.mac([ct], [pt]))
    assert out.shape[1] == 3
    assert_fhe_close(o.decode(o.decrypt(sk, out), 2.0 ** 36), 0.5 * vals, atol=1e-6, msg="mul+rescale")


def test_relinearized_square(small):
    o, _, sk = small
    vals = np.linspace(-1, 1, o.N // 2)
    ct = o.encrypt(sk, o.encode(vals, 4, 2.0 ** 36), 5)
    rl = o.relinearize(o.tensor(ct, ct), o.relin_key(sk, 1234))
    out = o.rescale(rl)
    assert_fhe_close(o.decode(o.decrypt(sk, out), 2.0 ** 72 / o.primes[3]), vals * vals, atol=1e-6, msg="square")


def _oracle_lt(o, sk, vals, diags, ratio, level_nq, scale=2.0 ** 36, seed=11):
    from helrm_b200.workload import bsgs_plan, preroll
    slots = o.N // 2
    ks = sorted(diags)
    plan = bsgs_plan(ks, ratio, slots)
    stride = plan["stride"]
    pts = [o.encode(preroll(diags[k], k // stride if plan["use_bsgs"] else 0, stride), level_nq, scale, ext=True)
           for k in ks]
    keys = {o.galois(d): o.rotation_key(sk, 1234, o.galois(d)) for d in plan["rotation_keys"]}
    ct = o.encrypt(sk, o.encode(vals, level_nq, scale), seed)
    out = o.bsgs_lt(ct, ks, pts, stride, keys)
    rs = o.rescale(out)
    return o.decode(o.decrypt(sk, rs), scale * scale / o.primes[level_nq - 1])


# The reference's linear-transform cases (tests/oracle/test_linear_transform.py:10-199)
LT_CASES = [
    ("identity", {0: 1.0}, 1.0),
    ("scale", {0: 3.0}, 1.0),
    ("permute3", {3: 1.0}, 1.0),
    ("multi", {0: 1.0, 1: 1.0}, 1.0),
    ("bsgs5", {0: 1.0, 1: 2.0, 2: 3.0, 5: 6.0, 8: 9.0}, 2.0),
    ("naive3", {0: 1.0, 2: -1.0, 7: 0.5}, "none"),
]


@pytest.mark.parametrize("name,diag_consts,ratio", LT_CASES)
def test_linear_transform_cases(small, name, diag_consts, ratio):
    o, _, sk = small
    slots = o.N // 2
    vals = np.array([float((i * 5) % 11) - 5.0 for i in range(slots)]) / 8
    diags = {k: np.full(slots, c) for k, c in diag_consts.items()}
    got = _oracle_lt(o, sk, vals, diags, ratio, 4)
    from helrm_b200.workload import cleartext_lt
    assert_fhe_close(got, cleartext_lt(vals, diags, slots), atol=1e-4, msg=name)


@pytest.mark.parametrize("num_diags", [50, 100, 144])
def test_bsgs_stress(small, num_diags):
    """reference tests/test_bsgs_linear_transform.py:195-235 (same seeds)."""
    o, _, sk = small
    slots = o.N // 2
    rng = np.random.default_rng(seed=42 + num_diags)
    vals = np.array([float(i % 17) * 0.1 for i in range(slots)])
    idx = sorted(rng.choice(slots, size=num_diags, replace=False).tolist())
    w = rng.uniform(-0.5, 0.5, size=num_diags)
    diags = {k: np.full(slots, wi) for k, wi in zip(idx, w)}
    got = _oracle_lt(o, sk, vals, diags, 2.0, 4)
    from helrm_b200.workload import cleartext_lt
    assert_fhe_close(got, cleartext_lt(vals, diags, slots), atol=1e-4, msg=f"stress {num_diags}")


def test_bsgs_vs_naive(small):
    """reference tests/test_bsgs_linear_transform.py:237-280."""
    o, _, sk = small
    slots = o.N // 2
    rng = np.random.default_rng(seed=99)
    vals = np.array([float(i % 13) * 0.2 for i in range(slots)])
    idx = sorted(rng.choice(slots, size=30, replace=False).tolist())
    w = rng.uniform(-0.3, 0.3, size=30)
    diags = {k: np.full(slots, wi) for k, wi in zip(idx, w)}
    a = _oracle_lt(o, sk, vals, diags, 2.0, 4)
    b = _oracle_lt(o, sk, vals, diags, "none", 4)
    assert_fhe_close(a, b, atol=1e-4, msg="bsgs vs naive")


def test_slot_varying_diagonals(small):
    o, _, sk = small
    slots = o.N // 2
    rng = np.random.default_rng(21)
    vals = rng.uniform(-1, 1, slots)
    diags = {k: rng.uniform(-0.5, 0.5, slots) for k in (0, 1, 4, 9, 33, 100, 257)}
    got = _oracle_lt(o, sk, vals, diags, 2.0, 4)
    from helrm_b200.workload import cleartext_lt
    assert_fhe_close(got, cleartext_lt(vals, diags, slots), atol=1e-4, msg="slot-varying")
