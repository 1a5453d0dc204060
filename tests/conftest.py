"""Shared test configuration.

``-m "not gpu"`` runs on any host: the CPU oracle against the golden
fixtures made from the reference, the host logic, and the C-ABI library's
load/export checks.  ``-m gpu`` runs the parity tests proper on a B200,
calling the CUDA path through the C ABI and checking it against the
oracle bit for bit (residues) or within the stated tolerances (decrypted
values).
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA) -- parity tests of the sm_100a path")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def golden_primes():
    import json
    with open(os.path.join(GOLDEN, "primes.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def golden_diag():
    return dict(np.load(os.path.join(GOLDEN, "diagonalize.npz")))


@pytest.fixture(scope="session")
def golden_bsgs():
    import json
    with open(os.path.join(GOLDEN, "bsgs_calls.json")) as f:
        return json.load(f)


def assert_fhe_close(actual, expected, atol=1e-2, msg=""):
    """Restates tests/oracle/fhe_test_utils.py:6-48 of the reference."""
    a = np.asarray(actual, dtype=np.float64).ravel()
    e = np.asarray(expected, dtype=np.float64).ravel()
    n = min(len(a), len(e))
    a, e = a[:n], e[:n]
    diff = np.abs(a - e)
    bad = diff > atol
    if bad.any():
        i = int(diff.argmax())
        raise AssertionError(f"{msg}: max error {diff[i]:.6e} at {i} (actual={a[i]:.6f}, expected={e[i]:.6f}); "
                             f"{int(bad.sum())}/{n} slots exceeded atol={atol}")
