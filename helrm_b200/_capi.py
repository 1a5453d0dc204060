"""ctypes binding of libhelrm_b200.so (the C ABI in include/helrm_b200.h).

Loading fails loudly when the library is missing or was built without the
CUDA kernels: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhelrm_b200.so")

c_int, c_double, c_u64, c_size = ctypes.c_int, ctypes.c_double, ctypes.c_uint64, ctypes.c_size_t
P = ctypes.POINTER
c_void = ctypes.c_void_p

# name -> argtypes (every entry point returns int status)
SIGNATURES = {
    "helrm_NewScheme": [c_int, P(c_int), c_int, P(c_int), c_int, c_int, c_int, c_int, c_u64, c_int],
    "helrm_DeleteScheme": [],
    "helrm_GetModuliChain": [P(c_u64), c_int, P(c_int)],
    "helrm_GetAuxModuliChain": [P(c_u64), c_int, P(c_int)],
    "helrm_GetSchemeInfo": [P(c_int)] * 5,
    "helrm_GenPrimes": [c_int, P(c_int), c_int, P(c_u64), c_int, P(c_u64)],
    "helrm_GenerateSecretKey": [],
    "helrm_GeneratePublicKey": [],
    "helrm_GenerateRelinearizationKey": [],
    "helrm_GenerateEvaluationKeys": [],
    "helrm_AddRotationKey": [c_int],
    "helrm_Encode": [P(c_double), c_int, c_int, c_double, P(c_int)],
    "helrm_EncodeComplex": [P(c_double), c_int, c_int, c_double, P(c_int)],
    "helrm_Decode": [c_int, P(c_double), c_int, P(c_int)],
    "helrm_DecodeComplex": [c_int, P(c_double), c_int, P(c_int)],
    "helrm_Encrypt": [c_int, P(c_int)],
    "helrm_Decrypt": [c_int, P(c_int)],
    "helrm_EncryptSeeded": [c_int, c_u64, P(c_int)],
    "helrm_DropAx": [c_int],
    "helrm_ExpandSeededAx": [c_int, c_u64],
    "helrm_AddCiphertextNew": [c_int, c_int, P(c_int)],
    "helrm_AddCiphertext": [c_int, c_int],
    "helrm_SubCiphertextNew": [c_int, c_int, P(c_int)],
    "helrm_SubCiphertext": [c_int, c_int],
    "helrm_MulRelinCiphertextNew": [c_int, c_int, P(c_int)],
    "helrm_MulRelinCiphertext": [c_int, c_int],
    "helrm_Negate": [c_int, P(c_int)],
    "helrm_AddPlaintextNew": [c_int, c_int, P(c_int)],
    "helrm_AddPlaintext": [c_int, c_int],
    "helrm_SubPlaintextNew": [c_int, c_int, P(c_int)],
    "helrm_SubPlaintext": [c_int, c_int],
    "helrm_MulPlaintextNew": [c_int, c_int, P(c_int)],
    "helrm_MulPlaintext": [c_int, c_int],
    "helrm_MulPlaintextAccumNew": [P(c_int), P(c_int), c_int, P(c_int)],
    "helrm_AddScalarNew": [c_int, c_double, P(c_int)],
    "helrm_AddScalar": [c_int, c_double],
    "helrm_SubScalarNew": [c_int, c_double, P(c_int)],
    "helrm_SubScalar": [c_int, c_double],
    "helrm_MulScalarIntNew": [c_int, ctypes.c_int64, P(c_int)],
    "helrm_MulScalarInt": [c_int, ctypes.c_int64],
    "helrm_MulScalarFloatNew": [c_int, c_double, P(c_int)],
    "helrm_MulScalarFloat": [c_int, c_double],
    "helrm_RescaleNew": [c_int, P(c_int)],
    "helrm_Rescale": [c_int],
    "helrm_AlignToLevelNew": [c_int, c_int, P(c_int)],
    "helrm_RotateNew": [c_int, c_int, P(c_int)],
    "helrm_Rotate": [c_int, c_int],
    "helrm_RotateBatchNew": [c_int, P(c_int), c_int, P(c_int)],
    "helrm_ConjugateNew": [c_int, P(c_int)],
    "helrm_Conjugate": [c_int],
    "helrm_GenerateLinearTransform": [P(c_int), c_int, P(c_double), c_int, c_int, c_double, P(c_int)],
    "helrm_EvaluateLinearTransform": [c_int, c_int, P(c_int)],
    "helrm_EvaluateLinearTransformBatch": [c_int, P(c_int), c_int, P(c_int)],
    "helrm_DeleteLinearTransform": [c_int],
    "helrm_GetLinearTransformRotationKeys": [c_int, P(c_int), c_int, P(c_int)],
    "helrm_GetLinearTransformInfo": [c_int, P(c_int), P(c_int), P(c_int), P(c_int)],
    "helrm_HybridFoldBatch": [P(c_int), c_int, c_int],
    "helrm_RescaleBatch": [P(c_int), c_int],
    "helrm_MulRelinCiphertextBatchNew": [P(c_int), P(c_int), c_int, P(c_int)],
    "helrm_DeleteCiphertext": [c_int],
    "helrm_DeletePlaintext": [c_int],
    "helrm_GetCiphertextLevel": [c_int, P(c_int)],
    "helrm_GetPlaintextLevel": [c_int, P(c_int)],
    "helrm_GetCiphertextScale": [c_int, P(c_double)],
    "helrm_GetPlaintextScale": [c_int, P(c_double)],
    "helrm_SetCiphertextScale": [c_int, c_double],
    "helrm_SetPlaintextScale": [c_int, c_double],
    "helrm_GetCiphertextSlots": [c_int, P(c_int)],
    "helrm_GetPlaintextSlots": [c_int, P(c_int)],
    "helrm_SetCiphertextSlots": [c_int, c_int],
    "helrm_GetCiphertextDegree": [c_int, P(c_int)],
    "helrm_GetLiveCounts": [P(c_int), P(c_int)],
    "helrm_GetCiphertextBytes": [c_int, P(c_double)],
    "helrm_GetMemoryMB": [P(c_double), P(c_double), P(c_double)],
    "helrm_GetCiphertextData": [c_int, P(c_u64), c_size],
    "helrm_NewCiphertextFromData": [P(c_u64), c_int, c_int, c_double, P(c_int)],
    "helrm_GetPlaintextData": [c_int, P(c_u64), c_size],
    "helrm_NewPlaintextFromData": [P(c_u64), c_int, c_int, c_double, P(c_int)],
    "helrm_GetKeyData": [c_u64, P(c_u64), c_size],
    "helrm_GetSecretKeyData": [P(c_u64), c_size],
    "helrm_GetLinearTransformPlaintext": [c_int, c_int, P(c_u64), c_size],
    "helrm_UploadCiphertextsAsync": [P(c_void), c_int, c_int, c_int, c_double, P(c_int)],
    "helrm_DownloadCiphertextsAsync": [P(c_int), c_int, P(c_void), c_size],
    "helrm_TransferSync": [],
    "helrm_EncodeConstantNew": [c_double, c_int, c_double, P(c_int)],
    "helrm_DeleteConstant": [c_int],
    "helrm_MulConstantAccumNew": [P(c_int), P(c_int), c_int, P(c_int)],
    "helrm_PackConstantTableNew": [P(c_int), c_int, c_int, P(c_int)],
    "helrm_PackPlaintextTableNew": [P(c_int), c_int, c_int, P(c_int)],
    "helrm_DeleteTable": [c_int],
    "helrm_GetTableShape": [c_int, P(c_int), P(c_int), P(c_int)],
    "helrm_MulTableMatMulNew": [P(c_int), c_int, c_int, P(c_int)],
    "helrm_ModRaiseNew": [c_int, P(c_int)],
    "helrm_GenerateLinearTransformEx": [P(c_int), c_int, P(c_double), c_int, c_int, c_double, c_int, c_double,
                                        P(c_int)],
    "helrm_EncodeBatch": [P(c_double), c_int, c_int, c_int, c_double, P(c_int)],
    "helrm_MulImaginaryUnitNew": [c_int, P(c_int)],
    "helrm_MulImaginaryUnit": [c_int],
    "helrm_UnpackLanes": [P(c_int), c_int, c_int, P(c_int)],
    "helrm_EvaluatePolynomial": [c_int, P(c_double), c_int, c_int, c_double, P(c_int)],
    "helrm_EvaluatePolynomialBatch": [P(c_int), c_int, P(c_double), c_int, c_int, c_double, P(c_int)],
    "helrm_PolynomialPlanInfo": [c_int, c_double, P(c_double), c_int, c_int, c_double, P(c_int)],
    "helrm_CiphertextsToDevice": [P(c_int), c_int, c_void, c_size],
    "helrm_NewCiphertextsFromDeviceSum": [c_void, c_int, c_int, c_int, c_double, P(c_int)],
    "helrm_kernel_ntt": [c_void, c_int, c_int, c_int, c_int, c_void],
    "helrm_kernel_automorphism": [c_void, c_void, c_int, c_u64, c_void],
    "helrm_kernel_rescale": [c_void, c_void, c_int, c_int, c_void],
    "helrm_kernel_rescale_noalloc": [c_void, c_void, c_int, c_int, c_void],
    "helrm_kernel_mac": [P(c_void), P(c_void), c_int, c_int, c_void, c_void],
    "helrm_kernel_rotate_hoisted": [c_void, c_int, c_int, P(c_int), c_int, c_void, c_void],
    "helrm_Synchronize": [],
    "helrm_TimerStart": [],
    "helrm_TimerStop": [P(c_double)],
    "helrm_ProfileEnable": [c_int],
    "helrm_ProfileRead": [P(c_double), P(c_double), P(c_double), P(c_u64), c_int, P(c_int)],
    "helrm_KernelClassName": [c_int, ctypes.c_char_p, c_int],
    "helrm_GetLaunchCount": [P(c_u64)],
    "helrm_GetAllocCount": [P(c_u64)],
    "helrm_ProfilerRange": [c_int],
}

ERRORS = {
    -1: ValueError,
    -2: IndexError,
    -3: RuntimeError,
    -4: RuntimeError,
    -5: MemoryError,
    -6: NotImplementedError,
}

_lib = None


def load(path: str | None = None):
    """Load the shared library (built by helrm_b200.build) and bind types."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python -m helrm_b200.build` "
            "(the B200 backend has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, argt in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argt
        fn.restype = c_int
    lib.helrm_LastError.argtypes = []
    lib.helrm_LastError.restype = ctypes.c_char_p
    _lib = lib
    return lib


def check(rc: int):
    if rc != 0:
        msg = _lib.helrm_LastError().decode("utf-8", "replace")
        raise ERRORS.get(rc, RuntimeError)(msg)


def call(name, *args):
    check(getattr(_lib, name)(*args))
