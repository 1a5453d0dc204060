"""The opt-in one-pass 2^16 NTT (thread-block clusters holding a limb in
distributed shared memory, HELRM_B200_NTT=cluster) must equal the oracle
residue for residue, forward and inverse, on q limbs (FP64 butterflies) and
special-prime limbs (integer butterflies), and through the out-of-place
inverse the key switch uses.  The switch is read once per process, so the
check runs in a child process with the variable set.
"""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import ctypes, sys
    import numpy as np
    import torch
    sys.path.insert(0, sys.argv[1])
    from helrm_b200 import B200Library, _capi
    from helrm_b200.params import CFG2, CFG2_DNUM
    from oracle import oracle as om
    lib = B200Library(dnum=CFG2_DNUM, seed=3, device=0)
    lib.setup_bindings(CFG2)
    main, aux = lib.GetModuliChain(), lib.GetAuxModuliChain()
    o = om.Oracle(16, main, aux, CFG2_DNUM)
    capi = _capi.load()
    rng = np.random.default_rng(11)
    nq, K, N = 24, 4, 1 << 16
    rows = nq + K
    host = np.stack([rng.integers(0, o.primes[r if r < nq else 24 + r - nq], N, dtype=np.uint64)
                     for r in range(rows)])
    dev = torch.from_numpy(host.view(np.int64).copy()).cuda()
    _capi.check(capi.helrm_kernel_ntt(ctypes.c_void_p(dev.data_ptr()), rows, rows, nq, 0, None))
    _capi.check(capi.helrm_Synchronize())
    fwd = dev.cpu().numpy().view(np.uint64)
    for r in range(rows):
        assert np.array_equal(fwd[r], o.ntt(r if r < nq else 24 + r - nq, host[r])), r
    _capi.check(capi.helrm_kernel_ntt(ctypes.c_void_p(dev.data_ptr()), rows, rows, nq, 1, None))
    _capi.check(capi.helrm_Synchronize())
    assert np.array_equal(dev.cpu().numpy().view(np.uint64), host)
    # the key switch (out-of-place inverse inside ModUp / ModDown)
    lib.GenerateSecretKey()
    pt = lib.Encode(list(np.sin(np.arange(N // 2) / 50.0)), 23, float(1 << 36))
    ct = lib.Encrypt(pt)
    out = lib.RotateNew(ct, 5)
    g = o.galois(5)
    assert np.array_equal(lib.GetCiphertextData(out), o.rotate(lib.GetCiphertextData(ct), lib.GetKeyData(g), g))
    lib.DeleteScheme()
    print("cluster ntt ok")
""")


def test_cluster_ntt_bit_exact():
    env = dict(os.environ, HELRM_B200_NTT="cluster")
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "cluster ntt ok" in r.stdout
