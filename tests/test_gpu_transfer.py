"""Asynchronous batch transfers through the C ABI: helrm_UploadCiphertextsAsync,
helrm_DownloadCiphertextsAsync and helrm_TransferSync move ciphertexts
between pinned host buffers and the device on the library's transfer
streams; arithmetic issued in between is ordered after the upload and before
the download by the library.  Results must equal the synchronous entry
points' bit for bit, also when the ciphertexts are deleted right after the
download is issued."""
import ctypes

import numpy as np
import pytest

from helrm_b200 import B200Library, CKKSConfig, _capi

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=12, logq=[40, 36, 36, 36, 36], logp=[60, 60], logscale=36, h=64)


@pytest.fixture(scope="module")
def scheme():
    lib = B200Library(dnum=2, seed=21, device=0)
    lib.setup_bindings(CFG)
    lib.GenerateSecretKey()
    yield lib
    lib.DeleteScheme()


def test_async_upload_compute_download_round_trip(scheme):
    import torch
    capi = _capi.load()
    primes = scheme.GetModuliChain()
    N = scheme.scheme_info()["N"]
    level, nb = 4, 6
    nq = level + 1
    rng = np.random.default_rng(5)
    host = torch.empty((nb, 2 * nq * N), dtype=torch.int64, pin_memory=True)
    for b in range(nb):
        rows = np.stack([rng.integers(0, primes[i % nq], N, dtype=np.uint64) for i in range(2 * nq)])
        host[b].copy_(torch.from_numpy(rows.reshape(-1).view(np.int64)))
    back = torch.zeros((nb, 2 * nq * N), dtype=torch.int64, pin_memory=True)
    ptrs = (ctypes.c_void_p * nb)(*[host[b].data_ptr() for b in range(nb)])
    bptrs = (ctypes.c_void_p * nb)(*[back[b].data_ptr() for b in range(nb)])
    ids = (ctypes.c_int * nb)()
    q = np.array([primes[i % nq] for i in range(2 * nq)], dtype=np.uint64)[:, None]
    for rep in range(2):  # twice in a row, reusing the host buffers
        back.zero_()
        _capi.check(capi.helrm_UploadCiphertextsAsync(ptrs, nb, level, 2, 2.0 ** 36, ids))
        sums = [scheme.AddCiphertextNew(ids[b], ids[b]) for b in range(nb)]  # x + x on the device
        sa = (ctypes.c_int * nb)(*sums)
        _capi.check(capi.helrm_DownloadCiphertextsAsync(sa, nb, bptrs, 2 * nq * N))
        want = [np.asarray(scheme.GetCiphertextData(s)).reshape(2 * nq, N) for s in sums]
        for b in range(nb):  # delete while the download may be in flight
            scheme.DeleteCiphertext(ids[b])
            scheme.DeleteCiphertext(sums[b])
        _capi.check(capi.helrm_TransferSync())
        got = back.numpy().view(np.uint64).reshape(nb, 2 * nq, N)
        x = host.numpy().view(np.uint64).reshape(nb, 2 * nq, N)
        for b in range(nb):
            assert np.array_equal(got[b], want[b])
            assert np.array_equal(got[b], (x[b] + x[b]) % q)


def test_async_transfer_argument_errors(scheme):
    capi = _capi.load()
    ids = (ctypes.c_int * 1)()
    with pytest.raises(ValueError):
        _capi.check(capi.helrm_UploadCiphertextsAsync(None, 1, 0, 2, 1.0, ids))
    with pytest.raises(ValueError):
        _capi.check(capi.helrm_DownloadCiphertextsAsync(None, 1, None, 0))
