"""The C-ABI library without a GPU: it loads, exports every symbol the
header declares, runs its host-only prime rule, and reports errors as
status codes (no compute call is made here)."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def capi():
    from helrm_b200 import build, _capi
    build.build()
    return _capi, _capi.load()


def _declared():
    txt = open(os.path.join(ROOT, "include", "helrm_b200.h")).read()
    return sorted(set(re.findall(r"\b(helrm_\w+)\s*\(", txt)))


def test_header_symbols_exported(capi):
    _, lib = capi
    names = _declared()
    assert len(names) > 80
    for n in names:
        assert hasattr(lib, n), n


def test_bindings_cover_header(capi):
    mod, _ = capi
    declared = set(_declared()) - {"helrm_LastError"}
    assert declared == set(mod.SIGNATURES), declared ^ set(mod.SIGNATURES)


def test_library_is_sm100a_build(capi):
    """The shared object embeds sm_100a device code (fatbin ELF note)."""
    data = open(os.path.join(ROOT, "helrm_b200", "libhelrm_b200.so"), "rb").read()
    assert b"sm_100a" in data or b"compute_100a" in data


def test_host_prime_rule_matches_reference(capi, golden_primes):
    mod, lib = capi
    for name, g in golden_primes.items():
        used = np.zeros(1, dtype=np.uint64)
        bits = (ctypes.c_int * len(g["logq"]))(*g["logq"])
        out = np.zeros(len(g["logq"]), dtype=np.uint64)
        mod.check(lib.helrm_GenPrimes(g["logn"], bits, len(g["logq"]), used.ctypes.data_as(mod.P(mod.c_u64)), 0,
                                      out.ctypes.data_as(mod.P(mod.c_u64))))
        assert [int(x) for x in out] == g["main"], name
        ub = np.array(g["main"], dtype=np.uint64)
        bits = (ctypes.c_int * len(g["logp"]))(*g["logp"])
        out = np.zeros(len(g["logp"]), dtype=np.uint64)
        mod.check(lib.helrm_GenPrimes(g["logn"], bits, len(g["logp"]), ub.ctypes.data_as(mod.P(mod.c_u64)), len(ub),
                                      out.ctypes.data_as(mod.P(mod.c_u64))))
        assert [int(x) for x in out] == g["aux"], name


def test_errors_without_scheme(capi):
    mod, lib = capi
    out = ctypes.c_int(0)
    vals = (ctypes.c_double * 4)(1, 2, 3, 4)
    rc = lib.helrm_Encode(vals, 4, 0, 1.0, ctypes.byref(out))
    assert rc == -3
    assert b"not initialised" in lib.helrm_LastError()
    with pytest.raises(RuntimeError):
        mod.check(rc)
    bad = (ctypes.c_int * 1)(70)
    o = np.zeros(1, dtype=np.uint64)
    assert lib.helrm_GenPrimes(13, bad, 1, None, 0, o.ctypes.data_as(mod.P(mod.c_u64))) == -1


def test_product_path_has_no_oracle_dependency():
    """The product package never imports or loads the checker."""
    pkg = os.path.join(ROOT, "helrm_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".hpp")):
                txt = open(os.path.join(dirpath, f), errors="ignore").read()
                assert "ckks_oracle" not in txt and "from oracle" not in txt and "import oracle" not in txt, f


def test_orion_trace_methods_exist_on_backend():
    """Every backend method the reference's Orion called in the recorded
    flows (tests/golden/orion_trace.json) exists on B200Library."""
    import json
    import os
    from helrm_b200 import B200Library
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "orion_trace.json")
    with open(path) as f:
        trace = json.load(f)
    methods = {c["m"] for t in trace.values() for c in t["calls"]}
    assert {"GenerateLinearTransform", "EvaluateLinearTransform", "RescaleNew", "AddPlaintext"} <= methods
    assert [m for m in methods if not hasattr(B200Library, m)] == []
