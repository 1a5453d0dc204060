"""B200Library -- the Orion backend object of the B200-native CKKS backend.

Mirrors the integer-handle surface of the reference's backends so that
``orion/backend/python/*`` and ``CipherTensor``/``PlainTensor`` drive it
unchanged: same method names, argument meaning and error behaviour as
``CheddarLibrary`` (orion/backend/cheddar/bindings.py:135-1342) and
``LattigoLibrary`` (orion/backend/lattigo/bindings.py:99-797).  Every call
goes through the C ABI of ``libhelrm_b200.so`` (include/helrm_b200.h) into
sm_100a kernels (the canonical-embedding encoding and decoding included);
no ciphertext or plaintext arithmetic runs on the CPU.  Compile-time
tables (the composite-sign fit, the bootstrapping matrices) are formed
with numpy on the host.
"""
from __future__ import annotations

import ctypes
import math
import os
from typing import Sequence

import numpy as np

from . import _capi
from ._capi import P, c_double, c_int, c_u64, call

_i32 = ctypes.c_int


def _int_array(vals):
    arr = np.ascontiguousarray(np.asarray(vals, dtype=np.int32))
    return arr, arr.ctypes.data_as(P(c_int))


def _f64_array(vals):
    arr = np.ascontiguousarray(np.asarray(vals, dtype=np.float64))
    return arr, arr.ctypes.data_as(P(c_double))


def _out_int():
    return ctypes.c_int(0)


def _cheb_basis(x: np.ndarray, degree: int) -> np.ndarray:
    """[len(x), degree + 1] matrix of T_0(x) .. T_degree(x), by T_{j+1} = 2 x T_j - T_{j-1}."""
    t = np.empty((len(x), degree + 1))
    t[:, 0] = 1.0
    if degree >= 1:
        t[:, 1] = x
    for j in range(2, degree + 1):
        t[:, j] = 2.0 * x * t[:, j - 1] - t[:, j - 2]
    return t


def _composite_sign_coeffs(degrees, gap):
    lo, hi = -1.0, 1.0
    flat: list[float] = []
    for i, d in enumerate(degrees):
        last = i == len(degrees) - 1
        npts = max(8 * d, 500)
        x = np.concatenate([np.linspace(lo, -gap, npts), np.linspace(gap, hi, npts)])
        target = np.where(x > 0, 1.0, 0.0) if last else np.sign(x)
        c = np.linalg.lstsq(_cheb_basis(x, d), target, rcond=None)[0]
        flat.extend(c[:d + 1].tolist())
        if last:
            break
        grid = np.concatenate([np.linspace(lo, -gap, 2000), np.linspace(gap, hi, 2000)])
        vals = _cheb_basis(grid, d) @ c
        lo, hi = float(vals.min()), float(vals.max())
        edge = _cheb_basis(np.array([gap, -gap]), d) @ c
        gap = max(float(min(abs(edge[0]), abs(edge[1]))), 1e-12)
    return flat


class B200Library:
    """Orion backend over libhelrm_b200.so.

    ``setup_bindings(orion_params)`` is the single entry point
    ``Scheme.setup_backend`` uses; every other method is called per op
    with integer ids, like the reference backends.
    """

    # The LT output is NOT rescaled natively; lt_evaluator rescales it
    # (orion/backend/python/lt_evaluator.py:262-273).
    lt_output_prerescaled = False

    def __init__(self, *, dnum: int | None = None, seed: int | None = None, device: int | None = None):
        self.lib = _capi.load()
        self._dnum = dnum
        self._seed = seed
        self._device = device
        self._polys: dict[int, tuple[list[float], str]] = {}
        self._next_poly = 1
        self._slots = None
        self._max_level = None
        self._default_scale = None
        self._h = 0
        self._boot = {}        # slots -> bootstrap.BootContext

    # ------------------------------------------------------------ setup
    def setup_bindings(self, orion_params) -> None:
        self.setup_scheme(orion_params)
        self.setup_tensor_binds()
        self.setup_key_generator()
        self.setup_encoder()
        self.setup_encryptor()
        self.setup_evaluator()
        self.setup_poly_evaluator()
        self.setup_lt_evaluator()
        self.setup_bootstrapper()

    def setup_scheme(self, orion_params) -> None:
        logn = int(orion_params.get_logn())
        logq = [int(x) for x in orion_params.get_logq()]
        logp = [int(x) for x in orion_params.get_logp()]
        logscale = int(orion_params.get_logscale())
        h = int(orion_params.get_hamming_weight())
        ring = str(getattr(orion_params, "get_ringtype", lambda: "standard")()).lower()
        if ring not in ("standard",):
            # The B200 backend implements the Standard ring only (N/2
            # complex slots), like the reference's Cheddar backend
            # (tests/oracle/conftest.py:34-55).
            pass
        dnum = self._dnum if self._dnum is not None else int(os.environ.get("HELRM_B200_DNUM", "0"))
        seed = self._seed if self._seed is not None else int(os.environ.get("HELRM_B200_SEED", "0"))
        device = self._device if self._device is not None else int(os.environ.get("HELRM_B200_DEVICE", "0"))
        # bootstrapping reserves primes above the usable chain, as the
        # reference's Cheddar setup does when Orion's boot parameters are set
        # (orion/backend/cheddar/bindings.py:262-294); GetModuliChain keeps
        # returning the usable primes only
        boot = getattr(orion_params, "get_boot_num_cts_levels", lambda: None)() is not None or \
            bool(getattr(orion_params, "boot", False))
        from . import bootstrap as _bt
        logq_all = logq + (_bt.boot_prime_bits(logscale, logq[0]) if boot else [])
        qa, qp = _int_array(logq_all)
        pa, pp = _int_array(logp)
        call("helrm_NewScheme", logn, qp, len(logq_all), pp, len(logp), logscale, h, dnum, seed, device)
        self._slots = 1 << (logn - 1)
        self._max_level = len(logq) - 1
        self._default_scale = 1 << logscale
        self._h = h
        self._boot = {}

    def DeleteScheme(self) -> None:
        call("helrm_DeleteScheme")

    def setup_tensor_binds(self):
        """No-op: objects live in the native registries."""

    def setup_key_generator(self):
        """No-op."""

    def setup_encoder(self):
        """No-op."""

    def setup_encryptor(self):
        """No-op."""

    def setup_evaluator(self):
        """No-op."""

    def setup_poly_evaluator(self):
        """No-op."""

    def setup_lt_evaluator(self):
        """No-op."""

    def setup_bootstrapper(self):
        """No-op."""

    # ------------------------------------------------------------ keys
    def NewKeyGenerator(self):
        """No-op: keys are generated by the Generate* calls."""

    def GenerateSecretKey(self):
        call("helrm_GenerateSecretKey")

    def GeneratePublicKey(self):
        call("helrm_GeneratePublicKey")

    def GenerateRelinearizationKey(self):
        call("helrm_GenerateRelinearizationKey")

    def GenerateEvaluationKeys(self):
        call("helrm_GenerateEvaluationKeys")

    def SerializeSecretKey(self):
        self._not_implemented("SerializeSecretKey")

    def LoadSecretKey(self, data):
        self._not_implemented("LoadSecretKey")

    def NewEncoder(self):
        """No-op."""

    def NewEncryptor(self):
        """No-op."""

    def NewDecryptor(self):
        """No-op."""

    def NewEvaluator(self):
        """No-op."""

    def NewPolynomialEvaluator(self):
        """No-op."""

    def NewLinearTransformEvaluator(self):
        """No-op."""

    # ------------------------------------------------------------ encode
    def Encode(self, values, level: int, scale) -> int:
        arr, ptr = _f64_array(list(values))
        out = _out_int()
        call("helrm_Encode", ptr, len(arr), int(level), float(scale), ctypes.byref(out))
        return out.value

    def EncodeBatch(self, values, level: int, scale) -> list[int]:
        """One plaintext per row of ``values`` (count x n reals), encoded on
        the device in one pass."""
        arr = np.ascontiguousarray(np.asarray(values, dtype=np.float64))
        if arr.ndim != 2:
            raise ValueError("EncodeBatch: values must be a 2-D array (count x n)")
        outs = np.zeros(arr.shape[0], dtype=np.int32)
        call("helrm_EncodeBatch", arr.ctypes.data_as(P(c_double)), arr.shape[0], arr.shape[1], int(level),
             float(scale), outs.ctypes.data_as(P(c_int)))
        return [int(v) for v in outs]

    def EncodeComplex(self, interleaved, level: int, scale) -> int:
        arr, ptr = _f64_array(list(interleaved))
        if len(arr) % 2:
            raise ValueError("EncodeComplex: expected interleaved [re, im, ...] pairs.")
        out = _out_int()
        call("helrm_EncodeComplex", ptr, len(arr) // 2, int(level), float(scale), ctypes.byref(out))
        return out.value

    def Decode(self, pt_id: int) -> list[float]:
        buf = np.zeros(self._slots, dtype=np.float64)
        n = _out_int()
        call("helrm_Decode", int(pt_id), buf.ctypes.data_as(P(c_double)), self._slots, ctypes.byref(n))
        return buf[:n.value].tolist()

    def DecodeComplex(self, pt_id: int) -> list[float]:
        buf = np.zeros(2 * self._slots, dtype=np.float64)
        n = _out_int()
        call("helrm_DecodeComplex", int(pt_id), buf.ctypes.data_as(P(c_double)), self._slots, ctypes.byref(n))
        return buf[:2 * n.value].tolist()

    # ------------------------------------------------------------ encrypt
    def Encrypt(self, pt_id: int) -> int:
        out = _out_int()
        call("helrm_Encrypt", int(pt_id), ctypes.byref(out))
        return out.value

    def EncryptSeeded(self, pt_id: int, seed: int) -> int:
        out = _out_int()
        call("helrm_EncryptSeeded", int(pt_id), int(seed) & (2**64 - 1), ctypes.byref(out))
        return out.value

    def DropAx(self, ct_id: int) -> None:
        call("helrm_DropAx", int(ct_id))

    def ExpandSeededAx(self, ct_id: int, seed: int) -> None:
        call("helrm_ExpandSeededAx", int(ct_id), int(seed) & (2**64 - 1))

    def Decrypt(self, ct_id: int) -> int:
        out = _out_int()
        call("helrm_Decrypt", int(ct_id), ctypes.byref(out))
        return out.value

    # ------------------------------------------------------------ arithmetic helpers
    def _new2(self, name, a, b):
        out = _out_int()
        call(name, int(a), int(b), ctypes.byref(out))
        return out.value

    def AddCiphertextNew(self, a, b):
        return self._new2("helrm_AddCiphertextNew", a, b)

    def AddCiphertext(self, a, b):
        call("helrm_AddCiphertext", int(a), int(b))
        return int(a)

    def SubCiphertextNew(self, a, b):
        return self._new2("helrm_SubCiphertextNew", a, b)

    def SubCiphertext(self, a, b):
        call("helrm_SubCiphertext", int(a), int(b))
        return int(a)

    def MulRelinCiphertextNew(self, a, b):
        return self._new2("helrm_MulRelinCiphertextNew", a, b)

    def MulRelinCiphertextBatchNew(self, a_ids: Sequence[int], b_ids: Sequence[int]) -> list[int]:
        """[MulRelinCiphertextNew(a, b) for a, b in pairs], the pairs of one
        level computed in batched kernels (residue-identical)."""
        if len(a_ids) != len(b_ids):
            raise ValueError("MulRelinCiphertextBatchNew: a_ids and b_ids differ in length")
        aa, ap = _int_array(a_ids)
        ba, bp = _int_array(b_ids)
        outs = np.zeros(len(aa), dtype=np.int32)
        call("helrm_MulRelinCiphertextBatchNew", ap, bp, len(aa), outs.ctypes.data_as(P(c_int)))
        return outs.tolist()

    def MulRelinCiphertext(self, a, b):
        call("helrm_MulRelinCiphertext", int(a), int(b))
        return int(a)

    def Negate(self, ct_id):
        """A new ciphertext holding -ct (the input is left as it is), like
        every reference backend's Negate."""
        out = _out_int()
        call("helrm_Negate", int(ct_id), ctypes.byref(out))
        return out.value

    def MulPlaintextNew(self, ct_id, pt_id):
        return self._new2("helrm_MulPlaintextNew", ct_id, pt_id)

    def MulPlaintext(self, ct_id, pt_id):
        call("helrm_MulPlaintext", int(ct_id), int(pt_id))
        return int(ct_id)

    def MulPlaintextAccumNew(self, ct_ids: Sequence[int], pt_ids: Sequence[int]) -> int:
        if len(ct_ids) == 0 or len(ct_ids) != len(pt_ids):
            raise RuntimeError("MulPlaintextAccumNew: ct_ids/pt_ids must be equal-length and non-empty.")
        ca, cp = _int_array(ct_ids)
        pa, pp = _int_array(pt_ids)
        out = _out_int()
        call("helrm_MulPlaintextAccumNew", cp, pp, len(ca), ctypes.byref(out))
        return out.value

    def AddPlaintextNew(self, ct_id, pt_id):
        return self._new2("helrm_AddPlaintextNew", ct_id, pt_id)

    def AddPlaintext(self, ct_id, pt_id):
        call("helrm_AddPlaintext", int(ct_id), int(pt_id))
        return int(ct_id)

    def SubPlaintextNew(self, ct_id, pt_id):
        return self._new2("helrm_SubPlaintextNew", ct_id, pt_id)

    def SubPlaintext(self, ct_id, pt_id):
        call("helrm_SubPlaintext", int(ct_id), int(pt_id))
        return int(ct_id)

    def _scalar_new(self, name, ct_id, s):
        out = _out_int()
        call(name, int(ct_id), s, ctypes.byref(out))
        return out.value

    def AddScalarNew(self, ct_id, scalar):
        return self._scalar_new("helrm_AddScalarNew", ct_id, float(scalar))

    def AddScalar(self, ct_id, scalar):
        call("helrm_AddScalar", int(ct_id), float(scalar))
        return int(ct_id)

    def SubScalarNew(self, ct_id, scalar):
        return self._scalar_new("helrm_SubScalarNew", ct_id, float(scalar))

    def SubScalar(self, ct_id, scalar):
        call("helrm_SubScalar", int(ct_id), float(scalar))
        return int(ct_id)

    def MulScalarIntNew(self, ct_id, scalar):
        return self._scalar_new("helrm_MulScalarIntNew", ct_id, int(scalar))

    def MulScalarInt(self, ct_id, scalar):
        call("helrm_MulScalarInt", int(ct_id), int(scalar))
        return int(ct_id)

    def MulScalarFloatNew(self, ct_id, scalar):
        return self._scalar_new("helrm_MulScalarFloatNew", ct_id, float(scalar))

    def MulScalarFloat(self, ct_id, scalar):
        call("helrm_MulScalarFloat", int(ct_id), float(scalar))
        return int(ct_id)

    def RescaleNew(self, ct_id):
        out = _out_int()
        call("helrm_RescaleNew", int(ct_id), ctypes.byref(out))
        return out.value

    def Rescale(self, ct_id):
        call("helrm_Rescale", int(ct_id))
        return int(ct_id)

    def AlignToLevelNew(self, ct_id, level):
        out = _out_int()
        call("helrm_AlignToLevelNew", int(ct_id), int(level), ctypes.byref(out))
        return out.value

    # ------------------------------------------------------------ rotations
    def AddRotationKey(self, k: int) -> None:
        call("helrm_AddRotationKey", int(k))

    def RotateNew(self, ct_id, k):
        out = _out_int()
        call("helrm_RotateNew", int(ct_id), int(k), ctypes.byref(out))
        return out.value

    def Rotate(self, ct_id, k):
        call("helrm_Rotate", int(ct_id), int(k))
        return int(ct_id)

    def RotateBatchNew(self, ct_id, ks: Sequence[int]) -> list[int]:
        ka, kp = _int_array(ks)
        outs = np.zeros(len(ka), dtype=np.int32)
        call("helrm_RotateBatchNew", int(ct_id), kp, len(ka), outs.ctypes.data_as(P(c_int)))
        return outs.tolist()

    def ConjugateNew(self, ct_id):
        out = _out_int()
        call("helrm_ConjugateNew", int(ct_id), ctypes.byref(out))
        return out.value

    def Conjugate(self, ct_id):
        call("helrm_Conjugate", int(ct_id))
        return int(ct_id)

    def ModRaiseNew(self, ct_id):
        """A level-0 ciphertext lifted (centred) to every main prime: it
        decrypts to m + q_0 I (bootstrapping's first step)."""
        out = _out_int()
        call("helrm_ModRaiseNew", int(ct_id), ctypes.byref(out))
        return out.value

    def MulImaginaryUnitNew(self, ct_id):
        """Slot-wise multiply by sqrt(-1): key-free, no level consumed."""
        out = _out_int()
        call("helrm_MulImaginaryUnitNew", int(ct_id), ctypes.byref(out))
        return out.value

    def MulImaginaryUnit(self, ct_id):
        call("helrm_MulImaginaryUnit", int(ct_id))
        return int(ct_id)

    def UnpackLanes(self, packed_ids: Sequence[int], num_real: int) -> list[int]:
        """Server side of complex-lane packing (orion/core/lane_packing.py:
        84-115): packed[m] = (x_2m + i x_2m+1) / 2 -> [x_0, x_1, ...], the
        first num_real of them, one batched conjugation for all inputs."""
        pa, pp = _int_array(packed_ids)
        outs = np.zeros(max(1, int(num_real)), dtype=np.int32)
        call("helrm_UnpackLanes", pp, len(pa), int(num_real), outs.ctypes.data_as(P(c_int)))
        return [int(v) for v in outs[:int(num_real)]]

    # ------------------------------------------------------------ lifecycle
    def DeleteCiphertext(self, ct_id):
        call("helrm_DeleteCiphertext", int(ct_id))

    def DeletePlaintext(self, pt_id):
        call("helrm_DeletePlaintext", int(pt_id))

    # ------------------------------------------------------------ linear transforms
    def GenerateLinearTransform(self, diags_idxs, diags_data, level, bsgs_ratio, io_mode="none") -> int:
        n = len(diags_idxs)
        if n == 0:
            raise ValueError("GenerateLinearTransform: no diagonals")
        data = np.ascontiguousarray(np.asarray(diags_data, dtype=np.float64))
        width = data.size // n
        if width * n != data.size:
            raise ValueError("GenerateLinearTransform: diagonal data is not n_diags x width")
        ia, ip = _int_array(diags_idxs)
        ratio = -1.0 if bsgs_ratio in ("none", None) else float(bsgs_ratio)
        out = _out_int()
        call("helrm_GenerateLinearTransform", ip, n, data.ctypes.data_as(P(c_double)), width, int(level), ratio,
             ctypes.byref(out))
        return out.value

    def GenerateLinearTransformEx(self, diag_idxs, diags_data, width: int, level: int, bsgs_ratio,
                                  cplx: bool, scale: float) -> int:
        """A transform with complex diagonals (interleaved re, im pairs,
        `width` pairs each when cplx) at an explicit plaintext scale."""
        ia, ip = _int_array(diag_idxs)
        data = np.ascontiguousarray(np.asarray(diags_data, dtype=np.float64).ravel())
        per = 2 if cplx else 1
        if data.size != len(ia) * int(width) * per:
            raise ValueError("GenerateLinearTransformEx: data size does not match the diagonals")
        out = _out_int()
        call("helrm_GenerateLinearTransformEx", ip, len(ia), data.ctypes.data_as(P(c_double)), int(width), int(level),
             float(bsgs_ratio), 1 if cplx else 0, float(scale), ctypes.byref(out))
        return out.value

    def GetLinearTransformRotationKeys(self, lt_id) -> list[int]:
        n = _out_int()
        call("helrm_GetLinearTransformRotationKeys", int(lt_id), None, 0, ctypes.byref(n))
        buf = np.zeros(max(1, n.value), dtype=np.int32)
        call("helrm_GetLinearTransformRotationKeys", int(lt_id), buf.ctypes.data_as(P(c_int)), n.value,
             ctypes.byref(n))
        return buf[:n.value].tolist()

    def GetLinearTransformInfo(self, lt_id) -> dict:
        bs, nd, ng, lv = (_out_int() for _ in range(4))
        call("helrm_GetLinearTransformInfo", int(lt_id), ctypes.byref(bs), ctypes.byref(nd), ctypes.byref(ng),
             ctypes.byref(lv))
        return {"bs": bs.value or None, "n_diags": nd.value, "n_giant": ng.value, "level": lv.value}

    def GenerateLinearTransformRotationKey(self, k):
        self.AddRotationKey(int(k))

    def EvaluateLinearTransform(self, lt_id, ct_id) -> int:
        out = _out_int()
        call("helrm_EvaluateLinearTransform", int(lt_id), int(ct_id), ctypes.byref(out))
        return out.value

    def EvaluateLinearTransformBatch(self, lt_id, ct_ids: Sequence[int]) -> list[int]:
        ca, cp = _int_array(ct_ids)
        outs = np.zeros(len(ca), dtype=np.int32)
        call("helrm_EvaluateLinearTransformBatch", int(lt_id), cp, len(ca), outs.ctypes.data_as(P(c_int)))
        return outs.tolist()

    def HybridFoldBatch(self, ct_ids: Sequence[int], rotations: int) -> None:
        """In place: ct += rot(ct, slots/2^i) for i = 1..rotations
        (orion/nn/linear.py:115-117), batched over ciphertexts."""
        ca, cp = _int_array(ct_ids)
        call("helrm_HybridFoldBatch", cp, len(ca), int(rotations))

    # ------------------------------------------------ IVE lookup: constants and tables
    # (orion/backend/cheddar/bindings.py:621-706; the one-pass kernels of
    # cheddar_pybind.cu:1044-1569)
    def EncodeConstantNew(self, scalar: float, level: int, scale) -> int:
        """A broadcast scalar in RNS form, one word per prime."""
        out = _out_int()
        call("helrm_EncodeConstantNew", float(scalar), int(level), float(scale), ctypes.byref(out))
        return out.value

    def DeleteConstant(self, const_id: int) -> None:
        call("helrm_DeleteConstant", int(const_id))

    def MulConstantAccumNew(self, ct_ids: Sequence[int], const_ids: Sequence[int]) -> int:
        """sum_i const_i * ct_i in one pass; scale ct * constant, not rescaled."""
        ca, cp = _int_array(ct_ids)
        ka, kp = _int_array(const_ids)
        if len(ca) != len(ka):
            raise ValueError("MulConstantAccumNew: ct_ids and const_ids differ in length")
        out = _out_int()
        call("helrm_MulConstantAccumNew", cp, kp, len(ca), ctypes.byref(out))
        return out.value

    def PackConstantTableNew(self, const_ids: Sequence[int], rows: int) -> int:
        """A rows x cols table of constants, row-major, for MulConstantMatMulNew."""
        ka, kp = _int_array(const_ids)
        out = _out_int()
        call("helrm_PackConstantTableNew", kp, len(ka), int(rows), ctypes.byref(out))
        return out.value

    def DeleteConstantTable(self, table_id: int) -> None:
        call("helrm_DeleteTable", int(table_id))

    def PackPlaintextTableNew(self, pt_ids: Sequence[int], rows: int) -> int:
        """A rows x cols table of plaintexts (kept by id: keep them alive)."""
        pa, pp = _int_array(pt_ids)
        out = _out_int()
        call("helrm_PackPlaintextTableNew", pp, len(pa), int(rows), ctypes.byref(out))
        return out.value

    def DeletePlaintextTable(self, table_id: int) -> None:
        call("helrm_DeleteTable", int(table_id))

    def _table_matmul(self, ct_ids, table_id) -> list[int]:
        rows = _out_int()
        call("helrm_GetTableShape", int(table_id), ctypes.byref(rows), None, None)
        ca, cp = _int_array(ct_ids)
        outs = np.zeros(rows.value, dtype=np.int32)
        call("helrm_MulTableMatMulNew", cp, len(ca), int(table_id), outs.ctypes.data_as(P(c_int)))
        return outs.tolist()

    def MulConstantMatMulNew(self, ct_ids: Sequence[int], table_id: int) -> list[int]:
        """The whole constant table against the ciphertext vector in one
        pass: one id per row, scale ct * constant, not rescaled."""
        return self._table_matmul(ct_ids, table_id)

    def MulPlaintextMatMulNew(self, ct_ids: Sequence[int], table_id: int) -> list[int]:
        """The slot-varying twin: one id per row, scale ct * plaintext."""
        return self._table_matmul(ct_ids, table_id)

    def CiphertextsToDevice(self, ct_ids: Sequence[int], dev_ptr: int, words_each: int) -> None:
        """Copy the ciphertexts' residues into a device buffer of the
        scheme's GPU (item i at i * words_each words), e.g. the tensor an
        NCCL reduce sums next.  Returns after the copies have finished."""
        ca, cp = _int_array(ct_ids)
        call("helrm_CiphertextsToDevice", cp, len(ca), ctypes.c_void_p(int(dev_ptr)), int(words_each))

    def NewCiphertextsFromDeviceSum(self, dev_ptr: int, n: int, level: int, npoly: int, scale: float) -> list[int]:
        """New ciphertexts from a device buffer of per-limb 64-bit sums of
        residues (partial ciphertexts of several ranks added as integers),
        each word reduced modulo its limb's prime on import."""
        outs = np.zeros(int(n), dtype=np.int32)
        call("helrm_NewCiphertextsFromDeviceSum", ctypes.c_void_p(int(dev_ptr)), int(n), int(level), int(npoly),
             float(scale), outs.ctypes.data_as(P(c_int)))
        return outs.tolist()

    def RescaleBatch(self, ct_ids: Sequence[int]) -> None:
        ca, cp = _int_array(ct_ids)
        call("helrm_RescaleBatch", cp, len(ca))

    def DeleteLinearTransform(self, lt_id):
        call("helrm_DeleteLinearTransform", int(lt_id))

    def RemoveRotationKeys(self):
        """No-op: rotation keys stay cached natively (like Cheddar)."""

    def RemovePlaintextDiagonals(self, lt_id):
        """No-op: diagonals stay resident until DeleteLinearTransform."""

    def GenerateAndSerializeRotationKey(self, k):
        self._not_implemented("GenerateAndSerializeRotationKey")

    def LoadRotationKey(self, byte_data, k=None):
        self._not_implemented("LoadRotationKey")

    def SerializeDiagonal(self, lt_id, diag_idx):
        self._not_implemented("SerializeDiagonal")

    def LoadPlaintextDiagonal(self, byte_data, lt_id, diag_idx):
        self._not_implemented("LoadPlaintextDiagonal")

    # ------------------------------------------------------------ polynomials
    def GenerateMonomial(self, coeffs) -> int:
        pid = self._next_poly
        self._next_poly += 1
        self._polys[pid] = (list(coeffs), "monomial")
        return pid

    def GenerateChebyshev(self, coeffs) -> int:
        pid = self._next_poly
        self._next_poly += 1
        self._polys[pid] = (list(coeffs), "chebyshev")
        return pid

    def EvaluatePolynomial(self, ct_id, poly_id, scale=None) -> int:
        """f(ct) for a polynomial from GenerateMonomial / GenerateChebyshev,
        at scale ``scale`` (the default scale when None), as the reference
        backends do (cheddar bindings.py:1102-1116): degree >= 2 runs the
        native log-depth evaluation (ceil(log2(d+1)) levels, the depth
        orion/nn/activation.py plans with), below that Horner's rule."""
        coeffs, kind = self._polys[poly_id]
        if len(coeffs) - 1 >= 2:
            return self._eval_native([ct_id], coeffs, kind, scale)[0]
        if kind == "chebyshev":
            # degree <= 1: T0 = 1, T1 = x, the conversion is exact
            coeffs = np.polynomial.chebyshev.cheb2poly(coeffs).tolist()
        return self._eval_horner(ct_id, coeffs)

    def EvaluatePolynomialBatch(self, ct_ids: Sequence[int], poly_id, scale=None) -> list[int]:
        """EvaluatePolynomial over all ciphertexts of a CipherTensor
        (poly_evaluator.py:29-31 calls it once per id) in batched kernels."""
        coeffs, kind = self._polys[poly_id]
        if len(coeffs) - 1 >= 2:
            return self._eval_native(list(ct_ids), coeffs, kind, scale)
        return [self.EvaluatePolynomial(c, poly_id, scale) for c in ct_ids]

    def _eval_native(self, ct_ids, coeffs, kind, scale):
        ca, cp = _int_array(ct_ids)
        co, pp = _f64_array(coeffs)
        s = float(self._default_scale if scale is None else scale)
        outs = np.zeros(len(ca), dtype=np.int32)
        call("helrm_EvaluatePolynomialBatch", cp, len(ca), pp, len(co), 1 if kind == "chebyshev" else 0, s,
             outs.ctypes.data_as(P(c_int)))
        return [int(v) for v in outs]

    def _eval_horner(self, ct_id, coeffs):
        """Horner's rule over MulRelin + Rescale (ascending coefficients)."""
        n = len(coeffs) - 1
        if n < 0:
            raise ValueError("EvaluatePolynomial: empty coefficient list.")
        acc = self.Rescale(self.MulScalarFloatNew(ct_id, coeffs[n] if n > 0 else 0.0))
        if n == 0:
            return self.AddScalar(acc, coeffs[0])
        acc = self.AddScalar(acc, coeffs[n - 1])
        for i in range(n - 2, -1, -1):
            prod = self.MulRelinCiphertextNew(acc, ct_id)
            self.DeleteCiphertext(acc)
            acc = self.Rescale(prod)
            acc = self.AddScalar(acc, coeffs[i])
        return acc

    def GetPolyDepth(self, poly_id) -> int:
        """Levels EvaluatePolynomial consumes (poly_evaluator.py:58-59):
        ceil(log2(d+1)) natively, one for the Horner path's degree 0 or 1."""
        coeffs, _ = self._polys[poly_id]
        d = len(coeffs) - 1
        return max(1, math.ceil(math.log2(d + 1))) if d >= 2 else 1

    def PolynomialPlanInfo(self, poly_id, level: int, in_scale: float, scale=None) -> dict:
        """The native evaluation plan for an input at ``level`` and
        ``in_scale``: levels consumed, ciphertext products, rescales and
        the baby-step count."""
        coeffs, kind = self._polys[poly_id]
        co, pp = _f64_array(coeffs)
        info = (c_int * 4)()
        s = float(self._default_scale if scale is None else scale)
        call("helrm_PolynomialPlanInfo", int(level) + 1, float(in_scale), pp, len(co),
             1 if kind == "chebyshev" else 0, s, info)
        return {"depth": info[0], "products": info[1], "rescales": info[2], "bs": info[3]}

    def GenerateMinimaxSignCoeffs(self, degrees, prec, logalpha, logerr, debug) -> list[float]:
        """Coefficients of a composite sign approximation, the stages'
        Chebyshev coefficients concatenated (the host computation of the
        reference's Cheddar backend, bindings.py:1164-1230).  Stage i is the
        least-squares fit, in the standard Chebyshev basis, of sign(x) --
        the last stage of the step x > 0 -> 1, else 0 (ReLU = x * step(x))
        -- on max(8 d, 500) evenly spaced points on each of [lo, -gap] and
        [gap, hi].  The first stage covers [-1, 1] with gap 2^-logalpha; each
        later one the previous stage's output range over 2000-point grids of
        its intervals, with gap the smaller magnitude of its output at
        +-gap.  prec, logerr and debug do not change the fit."""
        return _composite_sign_coeffs([int(d) for d in degrees], 2.0 ** (-float(logalpha)))

    # ------------------------------------------------------------ bootstrap (out of this backend's scope)
    def NewBootstrapper(self, logPs, slots: int) -> None:
        """Prepare the bootstrapping circuit for `slots` (its transforms,
        polynomials and keys; helrm_b200/bootstrap.py).  logPs is accepted
        for the interface, as the reference's Cheddar backend does
        (bindings.py:1326-1339).  Idempotent per slot count."""
        from . import bootstrap as _bt
        n = int(slots)
        if n not in self._boot:
            self._boot[n] = _bt.BootContext(self, n)

    def Bootstrap(self, ct_id, slots) -> int:
        """A fresh ciphertext at the top of the usable chain holding the
        slot values of ct_id (|values| <= 1 as Orion's Bootstrap layer
        scales them, orion/nn/operations.py:38-115)."""
        from . import bootstrap as _bt
        n = int(slots)
        if n not in self._boot:
            self.NewBootstrapper(None, n)
        return _bt.bootstrap(self, self._boot[n], int(ct_id))

    def BootstrapBatch(self, ct_ids: Sequence[int], slots) -> list[int]:
        """Bootstrap over a batch of ciphertexts of one slot count; each
        output equals Bootstrap of that input residue for residue."""
        from . import bootstrap as _bt
        n = int(slots)
        if n not in self._boot:
            self.NewBootstrapper(None, n)
        return _bt.bootstrap_batch(self, self._boot[n], [int(c) for c in ct_ids])

    def DeleteBootstrappers(self):
        """Release the bootstrapping transforms (keys stay cached)."""
        for ctx in self._boot.values():
            self.DeleteLinearTransform(ctx.cts)
            self.DeleteLinearTransform(ctx.stc)
        self._boot = {}

    # ------------------------------------------------------------ metadata
    def _get(self, name, obj_id, ctype=c_int):
        v = ctype(0)
        call(name, int(obj_id), ctypes.byref(v))
        return v.value

    def GetModuliChain(self) -> list[int]:
        """The usable primes q_0..q_max_level (the bootstrapping primes
        reserved above them are left out, as the reference does)."""
        return self.GetAllModuliChain()[:self._max_level + 1]

    def GetAllModuliChain(self) -> list[int]:
        """Every main prime, the reserved bootstrapping primes included."""
        n = _out_int()
        buf = np.zeros(64, dtype=np.uint64)
        call("helrm_GetModuliChain", buf.ctypes.data_as(P(c_u64)), 64, ctypes.byref(n))
        return [int(x) for x in buf[:n.value]]

    def GetAuxModuliChain(self) -> list[int]:
        n = _out_int()
        buf = np.zeros(64, dtype=np.uint64)
        call("helrm_GetAuxModuliChain", buf.ctypes.data_as(P(c_u64)), 64, ctypes.byref(n))
        return [int(x) for x in buf[:n.value]]

    def GetCiphertextLevel(self, ct_id):
        return self._get("helrm_GetCiphertextLevel", ct_id)

    def GetPlaintextLevel(self, pt_id):
        return self._get("helrm_GetPlaintextLevel", pt_id)

    def GetCiphertextScale(self, ct_id):
        return self._get("helrm_GetCiphertextScale", ct_id, c_double)

    def GetPlaintextScale(self, pt_id):
        return self._get("helrm_GetPlaintextScale", pt_id, c_double)

    def SetCiphertextScale(self, ct_id, scale):
        call("helrm_SetCiphertextScale", int(ct_id), float(scale))

    def SetPlaintextScale(self, pt_id, scale):
        call("helrm_SetPlaintextScale", int(pt_id), float(scale))

    def GetCiphertextSlots(self, ct_id):
        return self._get("helrm_GetCiphertextSlots", ct_id)

    def GetPlaintextSlots(self, pt_id):
        return self._get("helrm_GetPlaintextSlots", pt_id)

    def SetCiphertextSlots(self, ct_id, slots):
        call("helrm_SetCiphertextSlots", int(ct_id), int(slots))

    def GetCiphertextDegree(self, ct_id):
        return self._get("helrm_GetCiphertextDegree", ct_id)

    def GetLivePlaintexts(self):
        c, p = _out_int(), _out_int()
        call("helrm_GetLiveCounts", ctypes.byref(c), ctypes.byref(p))
        return p.value

    def GetLiveCiphertexts(self):
        c, p = _out_int(), _out_int()
        call("helrm_GetLiveCounts", ctypes.byref(c), ctypes.byref(p))
        return c.value

    def GetCiphertextBytes(self, ct_id):
        return self._get("helrm_GetCiphertextBytes", ct_id, c_double)

    def GetCiphertextBxBytes(self, ct_id):
        return self.GetCiphertextBytes(ct_id) / (self.GetCiphertextDegree(ct_id) + 1)

    def _mem(self):
        a, b, c = c_double(0), c_double(0), c_double(0)
        call("helrm_GetMemoryMB", ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    def GetLiveMemoryMB(self):
        return self._mem()[0]

    def GetPeakLiveMemoryMB(self):
        return self._mem()[1]

    def GetPeakDeviceMemoryMB(self):
        return self._mem()[1]

    def GetKeyMemoryMB(self):
        return self._mem()[2]

    # ------------------------------------------------------------ raw residues
    def scheme_info(self) -> dict:
        vals = [_out_int() for _ in range(5)]
        call("helrm_GetSchemeInfo", *[ctypes.byref(v) for v in vals])
        logn, slots, maxl, alpha, dnum = (v.value for v in vals)
        return {"logn": logn, "N": 1 << logn, "slots": slots, "max_level": maxl, "alpha": alpha, "dnum": dnum,
                "K": len(self.GetAuxModuliChain()), "L": maxl + 1}

    def GetCiphertextData(self, ct_id) -> np.ndarray:
        info = self.scheme_info()
        nq = self.GetCiphertextLevel(ct_id) + 1
        npoly = self.GetCiphertextDegree(ct_id) + 1
        buf = np.zeros((npoly, nq, info["N"]), dtype=np.uint64)
        call("helrm_GetCiphertextData", int(ct_id), buf.ctypes.data_as(P(c_u64)), buf.size)
        return buf

    def NewCiphertextFromData(self, data: np.ndarray, scale: float) -> int:
        data = np.ascontiguousarray(data, dtype=np.uint64)
        out = _out_int()
        call("helrm_NewCiphertextFromData", data.ctypes.data_as(P(c_u64)), data.shape[1] - 1, data.shape[0],
             float(scale), ctypes.byref(out))
        return out.value

    def GetPlaintextData(self, pt_id, ext=False) -> np.ndarray:
        info = self.scheme_info()
        nq = self.GetPlaintextLevel(pt_id) + 1
        rows = nq + (info["K"] if ext else 0)
        buf = np.zeros((rows, info["N"]), dtype=np.uint64)
        call("helrm_GetPlaintextData", int(pt_id), buf.ctypes.data_as(P(c_u64)), buf.size)
        return buf

    def NewPlaintextFromData(self, data: np.ndarray, level: int, ext: bool, scale: float) -> int:
        data = np.ascontiguousarray(data, dtype=np.uint64)
        out = _out_int()
        call("helrm_NewPlaintextFromData", data.ctypes.data_as(P(c_u64)), int(level), 1 if ext else 0,
             float(scale), ctypes.byref(out))
        return out.value

    def GetKeyData(self, galois: int) -> np.ndarray:
        info = self.scheme_info()
        shape = (info["dnum"], 2, info["L"] + info["K"], info["N"])
        buf = np.zeros(shape, dtype=np.uint64)
        call("helrm_GetKeyData", int(galois), buf.ctypes.data_as(P(c_u64)), buf.size)
        return buf

    def GetSecretKeyData(self) -> np.ndarray:
        info = self.scheme_info()
        buf = np.zeros((info["L"] + info["K"], info["N"]), dtype=np.uint64)
        call("helrm_GetSecretKeyData", buf.ctypes.data_as(P(c_u64)), buf.size)
        return buf

    def GetLinearTransformPlaintext(self, lt_id, k) -> np.ndarray:
        info = self.scheme_info()
        lv = self.GetLinearTransformInfo(lt_id)["level"]
        buf = np.zeros((lv + 1 + info["K"], info["N"]), dtype=np.uint64)
        call("helrm_GetLinearTransformPlaintext", int(lt_id), int(k), buf.ctypes.data_as(P(c_u64)), buf.size)
        return buf

    def Synchronize(self):
        call("helrm_Synchronize")

    # ------------------------------------------------------------ misc
    def _not_implemented(self, name: str):
        raise NotImplementedError(
            f"B200Library.{name}() is not implemented by the B200 backend "
            "(outside the embedding-PCMM path it accelerates).")
