"""ctypes front-end of the CPU oracle (oracle/ckks_oracle.c).

TEST INFRASTRUCTURE ONLY.  The checker for the CUDA path: tests/,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may use
it; the product package ``helrm_b200`` never does.

Arrays are numpy ``uint64`` in the limb-major layout the CUDA library uses:
a polynomial at level l is ``(l+1, N)``, a ciphertext ``(2, l+1, N)``, an
extended-basis (PQ) polynomial ``(l+1+K, N)`` with the q rows first, a
switching key ``(dnum, 2, L+K, N)`` (b then a).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libckks_oracle.so")

_u64p = ctypes.POINTER(ctypes.c_uint64)
_i32p = ctypes.POINTER(ctypes.c_int)
_f64p = ctypes.POINTER(ctypes.c_double)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i8p = ctypes.POINTER(ctypes.c_int8)


def build() -> str:
    """Compile the oracle with its Makefile (gcc); returns the .so path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "ckks_oracle.c"))):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    sig = {
        "ora_is_prime": ([ctypes.c_uint64], ctypes.c_int),
        "ora_gen_primes": ([_i32p, ctypes.c_int, ctypes.c_int, _u64p, _i32p, ctypes.c_int, _u64p], ctypes.c_int),
        "ora_find_psi": ([ctypes.c_uint64, ctypes.c_int], ctypes.c_uint64),
        "ora_new": ([ctypes.c_int, _u64p, ctypes.c_int, ctypes.c_int, ctypes.c_int], ctypes.c_void_p),
        "ora_free": ([ctypes.c_void_p], None),
        "ora_alpha": ([ctypes.c_void_p], ctypes.c_int),
        "ora_dnum": ([ctypes.c_void_p], ctypes.c_int),
        "ora_ntt": ([ctypes.c_void_p, ctypes.c_int, _u64p], None),
        "ora_intt": ([ctypes.c_void_p, ctypes.c_int, _u64p], None),
        "ora_ntt_naive": ([ctypes.c_void_p, ctypes.c_int, _u64p, _u64p], None),
        "ora_galois_rotation": ([ctypes.c_void_p, ctypes.c_long], ctypes.c_uint64),
        "ora_automorphism_index": ([ctypes.c_void_p, ctypes.c_uint64, _u32p], None),
        "ora_automorphism": ([ctypes.c_void_p, _u64p, _u64p, ctypes.c_int, ctypes.c_uint64], None),
        "ora_rand64": ([ctypes.c_uint64] * 3, ctypes.c_uint64),
        "ora_uniform": ([ctypes.c_uint64] * 4, ctypes.c_uint64),
        "ora_cbd": ([ctypes.c_uint64] * 3, ctypes.c_int),
        "ora_sample_secret": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, _i8p], None),
        "ora_secret_ntt": ([ctypes.c_void_p, _i8p, _u64p], None),
        "ora_key_seed": ([ctypes.c_uint64, ctypes.c_uint64], ctypes.c_uint64),
        "ora_gen_swk": ([ctypes.c_void_p, _u64p, _u64p, ctypes.c_uint64, _u64p], None),
        "ora_gen_rotation_key": ([ctypes.c_void_p, _u64p, ctypes.c_uint64, ctypes.c_uint64, _u64p], None),
        "ora_gen_relin_key": ([ctypes.c_void_p, _u64p, ctypes.c_uint64, _u64p], None),
        "ora_encrypt": ([ctypes.c_void_p, _u64p, _u64p, ctypes.c_int, ctypes.c_uint64, _u64p], None),
        "ora_decrypt": ([ctypes.c_void_p, _u64p, _u64p, ctypes.c_int, _u64p], None),
        "ora_encode": ([ctypes.c_void_p, _f64p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, _u64p], None),
        "ora_decode": ([ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_double, _f64p], None),
        "ora_rescale": ([ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.c_int, _u64p], None),
        "ora_modup": ([ctypes.c_void_p, _u64p, ctypes.c_int, _u64p], None),
        "ora_moddown": ([ctypes.c_void_p, _u64p, ctypes.c_int, _u64p], None),
        "ora_keymult": ([ctypes.c_void_p, _u64p, ctypes.c_int, _u64p, ctypes.c_uint64, _u64p], None),
        "ora_rotate": ([ctypes.c_void_p, _u64p, ctypes.c_int, _u64p, ctypes.c_uint64, _u64p], None),
        "ora_rotate_hoisted": ([ctypes.c_void_p, _u64p, ctypes.c_int, ctypes.POINTER(_u64p), _u64p,
                                ctypes.c_int, _u64p], None),
        "ora_relinearize": ([ctypes.c_void_p, _u64p, ctypes.c_int, _u64p, _u64p], None),
        "ora_tensor": ([ctypes.c_void_p, _u64p, _u64p, ctypes.c_int, _u64p], None),
        "ora_mac": ([ctypes.c_void_p, ctypes.POINTER(_u64p), ctypes.POINTER(_u64p), ctypes.c_int,
                     ctypes.c_int, _u64p], None),
        "ora_set_threads": ([ctypes.c_int], None),
        "ora_num_threads": ([], ctypes.c_int),
        "ora_bsgs_lt": ([ctypes.c_void_p, _u64p, ctypes.c_int, _i32p, ctypes.POINTER(_u64p), ctypes.c_int,
                         ctypes.c_int, _u64p, ctypes.POINTER(_u64p), ctypes.c_int, _u64p], ctypes.c_int),
    }
    for name, (argt, rest) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = argt
        fn.restype = rest
    return lib


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(_u64p)


def gen_primes(bit_sizes, logn, used=None):
    """Restatement of orion/backend/cheddar/bindings.py:108-132."""
    used = list(used or [])
    cap = len(used) + len(bit_sizes) + 8
    used_arr = np.zeros(cap, dtype=np.uint64)
    used_arr[:len(used)] = used
    nused = ctypes.c_int(len(used))
    bits = (ctypes.c_int * len(bit_sizes))(*bit_sizes)
    out = np.zeros(len(bit_sizes), dtype=np.uint64)
    rc = lib().ora_gen_primes(bits, len(bit_sizes), logn, _p(used_arr), ctypes.byref(nused), cap, _p(out))
    if rc != 0:
        raise ValueError(f"gen_primes failed ({rc})")
    return [int(x) for x in out], [int(x) for x in used_arr[:nused.value]]


def scheme_primes(logq, logp, logn):
    """Main primes (one per LogQ entry) then aux primes, sharing `used`."""
    main, used = gen_primes(logq, logn, [])
    aux, _ = gen_primes(logp, logn, used)
    return main, aux


class Oracle:
    """CPU CKKS restatement bound to one parameter set."""

    def __init__(self, logn, main_primes, aux_primes, dnum):
        self.logn = logn
        self.N = 1 << logn
        self.L = len(main_primes)
        self.K = len(aux_primes)
        self.primes = [int(p) for p in main_primes] + [int(p) for p in aux_primes]
        arr = np.array(self.primes, dtype=np.uint64)
        self._ctx = lib().ora_new(logn, _p(arr), self.L, self.K, dnum)
        if not self._ctx:
            raise ValueError("bad oracle parameters")
        self.alpha = lib().ora_alpha(self._ctx)
        self.dnum = lib().ora_dnum(self._ctx)

    def __del__(self):
        if getattr(self, "_ctx", None):
            lib().ora_free(self._ctx)
            self._ctx = None

    # -- helpers ---------------------------------------------------
    def beta(self, nq):
        return (nq + self.alpha - 1) // self.alpha

    def ext_primes(self, nq):
        return self.primes[:nq] + self.primes[self.L:]

    def galois(self, k):
        return int(lib().ora_galois_rotation(self._ctx, int(k)))

    def conj_galois(self):
        return 2 * self.N - 1

    # -- NTT -------------------------------------------------------
    def ntt(self, prime_idx, a):
        a = np.ascontiguousarray(a, dtype=np.uint64).copy()
        lib().ora_ntt(self._ctx, prime_idx, _p(a))
        return a

    def intt(self, prime_idx, a):
        a = np.ascontiguousarray(a, dtype=np.uint64).copy()
        lib().ora_intt(self._ctx, prime_idx, _p(a))
        return a

    def ntt_rows(self, a, prime_rows):
        out = np.ascontiguousarray(a, dtype=np.uint64).copy()
        for r, p in enumerate(prime_rows):
            lib().ora_ntt(self._ctx, p, _p(out[r]))
        return out

    def intt_rows(self, a, prime_rows):
        out = np.ascontiguousarray(a, dtype=np.uint64).copy()
        for r, p in enumerate(prime_rows):
            lib().ora_intt(self._ctx, p, _p(out[r]))
        return out

    def ntt_naive(self, prime_idx, a):
        a = np.ascontiguousarray(a, dtype=np.uint64)
        out = np.zeros_like(a)
        lib().ora_ntt_naive(self._ctx, prime_idx, _p(a), _p(out))
        return out

    def automorphism_index(self, g):
        idx = np.zeros(self.N, dtype=np.uint32)
        lib().ora_automorphism_index(self._ctx, g, idx.ctypes.data_as(_u32p))
        return idx

    def automorphism(self, a, g):
        a = np.ascontiguousarray(a, dtype=np.uint64)
        rows = a.size // self.N
        out = np.zeros_like(a)
        lib().ora_automorphism(self._ctx, _p(a), _p(out), rows, g)
        return out

    # -- keys ------------------------------------------------------
    def sample_secret(self, seed, h):
        s = np.zeros(self.N, dtype=np.int8)
        lib().ora_sample_secret(self._ctx, seed, h, s.ctypes.data_as(_i8p))
        return s

    def secret_ntt(self, s):
        s = np.ascontiguousarray(s, dtype=np.int8)
        sk = np.zeros((self.L + self.K, self.N), dtype=np.uint64)
        lib().ora_secret_ntt(self._ctx, s.ctypes.data_as(_i8p), _p(sk))
        return sk

    def key_shape(self):
        return (self.dnum, 2, self.L + self.K, self.N)

    def rotation_key(self, sk, master_seed, g):
        swk = np.zeros(self.key_shape(), dtype=np.uint64)
        lib().ora_gen_rotation_key(self._ctx, _p(sk), master_seed, g, _p(swk))
        return swk

    def relin_key(self, sk, master_seed):
        swk = np.zeros(self.key_shape(), dtype=np.uint64)
        lib().ora_gen_relin_key(self._ctx, _p(sk), master_seed, _p(swk))
        return swk

    # -- encode / encrypt -----------------------------------------
    def encode(self, values, nq, scale, ext=False):
        v = np.asarray(values)
        if np.iscomplexobj(v):
            inter = np.stack([v.real, v.imag], axis=-1).astype(np.float64).ravel()
        else:
            inter = np.stack([v.astype(np.float64), np.zeros(len(v))], axis=-1).ravel()
        inter = np.ascontiguousarray(inter)
        rows = nq + (self.K if ext else 0)
        out = np.zeros((rows, self.N), dtype=np.uint64)
        lib().ora_encode(self._ctx, inter.ctypes.data_as(_f64p), len(v), nq, 1 if ext else 0,
                         float(scale), _p(out))
        return out

    def decode(self, pt, scale, complex_out=False):
        pt = np.ascontiguousarray(pt, dtype=np.uint64)
        nq = pt.shape[0]
        out = np.zeros(self.N, dtype=np.float64)
        lib().ora_decode(self._ctx, _p(pt), nq, float(scale), out.ctypes.data_as(_f64p))
        z = out[0::2] + 1j * out[1::2]
        return z if complex_out else z.real.copy()

    def encrypt(self, sk, pt, ct_seed):
        pt = np.ascontiguousarray(pt, dtype=np.uint64)
        nq = pt.shape[0]
        ct = np.zeros((2, nq, self.N), dtype=np.uint64)
        lib().ora_encrypt(self._ctx, _p(sk), _p(pt), nq, ct_seed, _p(ct))
        return ct

    def decrypt(self, sk, ct):
        ct = np.ascontiguousarray(ct, dtype=np.uint64)
        nq = ct.shape[1]
        pt = np.zeros((nq, self.N), dtype=np.uint64)
        lib().ora_decrypt(self._ctx, _p(sk), _p(ct), nq, _p(pt))
        return pt

    # -- evaluation -----------------------------------------------
    def rescale(self, ct):
        ct = np.ascontiguousarray(ct, dtype=np.uint64)
        npoly, nq = ct.shape[0], ct.shape[1]
        out = np.zeros((npoly, nq - 1, self.N), dtype=np.uint64)
        lib().ora_rescale(self._ctx, _p(ct), npoly, nq, _p(out))
        return out

    def modup(self, a):
        a = np.ascontiguousarray(a, dtype=np.uint64)
        nq = a.shape[0]
        D = np.zeros((self.beta(nq), nq + self.K, self.N), dtype=np.uint64)
        lib().ora_modup(self._ctx, _p(a), nq, _p(D))
        return D

    def moddown(self, x):
        x = np.ascontiguousarray(x, dtype=np.uint64)
        nq = x.shape[0] - self.K
        out = np.zeros((nq, self.N), dtype=np.uint64)
        lib().ora_moddown(self._ctx, _p(x), nq, _p(out))
        return out

    def keymult(self, D, swk, g):
        D = np.ascontiguousarray(D, dtype=np.uint64)
        ne = D.shape[1]
        nq = ne - self.K
        acc = np.zeros((2, ne, self.N), dtype=np.uint64)
        lib().ora_keymult(self._ctx, _p(D), nq, _p(swk), g, _p(acc))
        return acc

    def rotate(self, ct, swk, g):
        ct = np.ascontiguousarray(ct, dtype=np.uint64)
        out = np.zeros_like(ct)
        lib().ora_rotate(self._ctx, _p(ct), ct.shape[1], _p(swk), g, _p(out))
        return out

    def rotate_hoisted(self, ct, swks, gs):
        ct = np.ascontiguousarray(ct, dtype=np.uint64)
        n = len(gs)
        outs = np.zeros((n,) + ct.shape, dtype=np.uint64)
        ptrs = (_u64p * n)(*[_p(k) for k in swks])
        garr = np.array(gs, dtype=np.uint64)
        lib().ora_rotate_hoisted(self._ctx, _p(ct), ct.shape[1], ptrs, _p(garr), n, _p(outs))
        return outs

    def tensor(self, a, b):
        a = np.ascontiguousarray(a, dtype=np.uint64)
        b = np.ascontiguousarray(b, dtype=np.uint64)
        nq = a.shape[1]
        out = np.zeros((3, nq, self.N), dtype=np.uint64)
        lib().ora_tensor(self._ctx, _p(a), _p(b), nq, _p(out))
        return out

    def relinearize(self, ct3, rlk):
        ct3 = np.ascontiguousarray(ct3, dtype=np.uint64)
        nq = ct3.shape[1]
        out = np.zeros((2, nq, self.N), dtype=np.uint64)
        lib().ora_relinearize(self._ctx, _p(ct3), nq, _p(rlk), _p(out))
        return out

    def mac(self, cts, pts):
        cts = [np.ascontiguousarray(c, dtype=np.uint64) for c in cts]
        pts = [np.ascontiguousarray(p, dtype=np.uint64) for p in pts]
        nq = cts[0].shape[1]
        out = np.zeros((2, nq, self.N), dtype=np.uint64)
        cp = (_u64p * len(cts))(*[_p(c) for c in cts])
        pp = (_u64p * len(pts))(*[_p(p) for p in pts])
        lib().ora_mac(self._ctx, cp, pp, len(cts), nq, _p(out))
        return out

    def bsgs_lt(self, ct, diag_ks, pts, bs, keys):
        """Double-hoisted BSGS LT.  pts[t]: extended-basis plaintext for
        diag_ks[t] (pre-rolled by g*bs); keys: {galois: swk}."""
        ct = np.ascontiguousarray(ct, dtype=np.uint64)
        nq = ct.shape[1]
        pts = [np.ascontiguousarray(p, dtype=np.uint64) for p in pts]
        kl = list(keys.items())
        ks = (ctypes.c_int * len(diag_ks))(*diag_ks)
        pp = (_u64p * len(pts))(*[_p(p) for p in pts])
        garr = np.array([g for g, _ in kl] or [0], dtype=np.uint64)
        kp = (_u64p * max(1, len(kl)))(*[_p(k) for _, k in kl])
        out = np.zeros((2, nq, self.N), dtype=np.uint64)
        rc = lib().ora_bsgs_lt(self._ctx, _p(ct), nq, ks, pp, len(diag_ks), bs, _p(garr), kp, len(kl), _p(out))
        if rc != 0:
            raise KeyError("missing rotation key for the BSGS linear transform")
        return out

    def fold_add(self, a, b):
        """(a + b) mod q_i, limb by limb (residues below 2^61: no overflow)."""
        qs = np.array(self.primes[:a.shape[1]], dtype=np.uint64)[None, :, None]
        s = a + b
        return np.where(s >= qs, s - qs, s)

    def pcmm(self, ct, diag_ks, pts, bs, keys, fold_rotations):
        """The embedding layer's encrypted step as the reference runs it
        (orion/nn/linear.py:99-140): the BSGS linear transform, the rescale
        (orion/backend/python/lt_evaluator.py:262-273), then the hybrid
        output fold out += rot(out, slots / 2^i) for i = 1..fold_rotations
        (linear.py:115-117).  keys must hold the fold rotations' keys too."""
        out = self.rescale(self.bsgs_lt(ct, diag_ks, pts, bs, keys))
        for i in range(1, fold_rotations + 1):
            g = self.galois((self.N // 2) >> i)
            out = self.fold_add(out, self.rotate(out, keys[g], g))
        return out


def set_threads(n: int) -> None:
    """Worker threads for the oracle's limb-parallel loops (default 1)."""
    lib().ora_set_threads(int(n))
