"""helrm_kernel_rescale_noalloc: the rescale entry point whose temporaries
live in a fixed array inside the library instead of the device pool.

Its output must equal helrm_kernel_rescale's on the same input (integer
residues: the tolerance is zero), on two calls issued back to back, and the
calls must make no device-pool allocation: the library's allocation count
(helrm_GetAllocCount, every cudaMallocAsync the scheme makes) stays put.
Requests above the fixed array's size must be refused before any work.
This file is named to be collected last, so it also runs after every other
GPU test in the same process; it needs nothing from them.
"""
import ctypes

import numpy as np
import pytest

from helrm_b200 import B200Library, CKKSConfig, _capi

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=12, logq=[40, 36, 36, 36, 36], logp=[60, 60], logscale=36, h=64)
SCRATCH_WORDS = 4 << 20  # HELRM_RESCALE_SCRATCH_WORDS


@pytest.fixture(scope="module")
def scheme():
    lib = B200Library(dnum=2, seed=11, device=0)
    lib.setup_bindings(CFG)
    yield lib
    lib.DeleteScheme()


def _residues(primes, nb, nq, N, gen):
    import torch
    t = torch.empty((nb, 2, nq, N), dtype=torch.int64, device="cuda")
    for i in range(nq):
        t[:, :, i].random_(0, primes[i], generator=gen)
    return t


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _peak_mb(capi):
    live, peak, keys = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
    _capi.check(capi.helrm_GetMemoryMB(ctypes.byref(live), ctypes.byref(peak), ctypes.byref(keys)))
    return peak.value


def _allocs(capi):
    n = ctypes.c_uint64(0)
    _capi.check(capi.helrm_GetAllocCount(ctypes.byref(n)))
    return n.value


def test_noalloc_rescale_matches_allocating_entry_point(scheme):
    import torch
    capi = _capi.load()
    primes = scheme.GetModuliChain()
    N = scheme.scheme_info()["N"]
    gen = torch.Generator(device="cuda").manual_seed(3)
    cases = [(5, 3), (4, 2)]  # (limbs, ciphertexts) of the two calls
    xs = [_residues(primes, nb, nq, N, gen) for nq, nb in cases]
    got = [torch.full((nb, 2, nq - 1, N), -1, dtype=torch.int64, device="cuda") for nq, nb in cases]
    want = [torch.full_like(g, -2) for g in got]
    torch.cuda.synchronize()

    n0 = _allocs(capi)
    for (nq, nb), x, g in zip(cases, xs, got):  # two calls in a row, no sync between
        _capi.check(capi.helrm_kernel_rescale_noalloc(_ptr(x), _ptr(g), nq, nb, None))
    _capi.check(capi.helrm_Synchronize())
    assert _allocs(capi) == n0, "the no-allocation entry point drew on the device pool"

    for (nq, nb), x, w in zip(cases, xs, want):
        _capi.check(capi.helrm_kernel_rescale(_ptr(x), _ptr(w), nq, nb, None))
    _capi.check(capi.helrm_Synchronize())
    # the counter does see the allocating entry point's temporaries
    assert _allocs(capi) > n0
    for g, w in zip(got, want):
        assert torch.equal(g.cpu(), w.cpu())  # tolerance 0: exact residues


def test_noalloc_rescale_size_limit(scheme):
    import torch
    capi = _capi.load()
    primes = scheme.GetModuliChain()
    N = scheme.scheme_info()["N"]
    nq = 5
    nb_max = SCRATCH_WORDS // (2 * nq * N)
    gen = torch.Generator(device="cuda").manual_seed(4)
    x = _residues(primes, nb_max + 1, nq, N, gen)
    out = torch.empty((nb_max + 1, 2, nq - 1, N), dtype=torch.int64, device="cuda")
    # the largest batch that fits runs and matches the allocating path
    _capi.check(capi.helrm_kernel_rescale_noalloc(_ptr(x), _ptr(out), nq, nb_max, None))
    _capi.check(capi.helrm_Synchronize())
    got = out[:nb_max].cpu()
    _capi.check(capi.helrm_kernel_rescale(_ptr(x), _ptr(out), nq, nb_max, None))
    _capi.check(capi.helrm_Synchronize())
    assert torch.equal(got, out[:nb_max].cpu())
    # one more ciphertext is refused on the host before any work
    with pytest.raises(ValueError, match="static limit"):
        _capi.check(capi.helrm_kernel_rescale_noalloc(_ptr(x), _ptr(out), nq, nb_max + 1, None))
    assert np.isfinite(_peak_mb(capi))
