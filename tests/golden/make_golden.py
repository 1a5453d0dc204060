"""Generate the golden fixtures under tests/golden/ from the REFERENCE.

Run in the build container (where the read-only reference checkout exists):

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own Python (orion) with its four absent optional
dependencies stubbed, and records:

* ``primes.json``  -- ``_gen_primes`` (orion/backend/cheddar/bindings.py:108-132)
  for the test, cfg1 and cfg2 parameter sets;
* ``diagonalize.npz`` -- ``packing.diagonalize`` (orion/core/packing.py:626-865)
  on the docstring example, the cfg1 table stack and a 26-table
  block-diagonal matrix at 2048 slots, plus a digest of the full cfg2
  (416 x 4224 at 32768 slots) diagonals;
* ``bsgs_calls.json`` -- the call sequence of the reference's Python BSGS
  orchestration (``CheddarLibrary.GenerateLinearTransform`` /
  ``GetLinearTransformRotationKeys`` / ``_eval_lt_bsgs``,
  bindings.py:833-1032) recorded through a fake native module, for the
  diagonal sets of the reference's own LT tests.

Nothing at test time reads the reference; only these files are used.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_root):
    sys.path.insert(0, ref_root)
    for name in ["matplotlib", "matplotlib.pyplot", "h5py", "opt_einsum", "desilofhe"]:
        sys.modules.setdefault(name, types.ModuleType(name))
    fake = _FakeNative()
    sys.modules["orion.backend.cheddar._cheddar_native"] = fake
    from orion.core import packing  # noqa: E402
    from orion.backend.cheddar import bindings as cb  # noqa: E402
    return packing, cb, fake


class _FakeNative(types.ModuleType):
    """Stands in for _cheddar_native: hands out ids and records calls."""

    def __init__(self):
        super().__init__("orion.backend.cheddar._cheddar_native")
        self.calls = []
        self.next_id = 1
        self.pt_values = {}
        self.levels = {}

    def _new(self):
        i = self.next_id
        self.next_id += 1
        return i

    def Encode(self, values, level, scale):
        i = self._new()
        self.pt_values[i] = list(values)
        self.calls.append(["Encode", i, level])
        return i

    def RotateBatchNew(self, ct, ks, mode):
        out = [self._new() for _ in ks]
        self.calls.append(["RotateBatchNew", ct, list(ks), out])
        return out

    def RotateNew(self, ct, k):
        i = self._new()
        self.calls.append(["RotateNew", ct, k, i])
        return i

    def MulPlaintextAccumNew(self, cts, pts):
        i = self._new()
        self.calls.append(["MulPlaintextAccumNew", list(cts), list(pts), i])
        return i

    def MulPlaintextNew(self, ct, pt):
        i = self._new()
        self.calls.append(["MulPlaintextAccumNew", [ct], [pt], i])
        return i

    def AddCiphertextNew(self, a, b):
        i = self._new()
        self.calls.append(["AddCiphertextNew", a, b, i])
        return i

    def DeleteCiphertext(self, i):
        self.calls.append(["DeleteCiphertext", i])

    def DeletePlaintext(self, i):
        pass

    def GetCiphertextLevel(self, i):
        return self.levels.get(i, 99)

    def AlignToLevelNew(self, ct, level):
        i = self._new()
        self.calls.append(["AlignToLevelNew", ct, level, i])
        return i

    def delete_scheme(self):
        pass


PARAM_SETS = {
    # tests/oracle/conftest.py:40-55 (Cheddar-style Standard ring)
    "test": {"logn": 13, "logq": [29, 26, 26, 26], "logp": [29]},
    # BASELINE.json configs[0]
    "cfg1": {"logn": 13, "logq": [40] * 5, "logp": [60]},
    # BASELINE.json configs[1]/[2]
    "cfg2": {"logn": 16, "logq": [36] * 24, "logp": [60] * 4},
}


def make_primes(cb):
    out = {}
    for name, p in PARAM_SETS.items():
        used: set[int] = set()
        main = cb._gen_primes(p["logq"], p["logn"], used)
        aux = cb._gen_primes(p["logp"], p["logn"], used)
        out[name] = {**p, "main": main, "aux": aux}
    with open(os.path.join(HERE, "primes.json"), "w") as f:
        json.dump(out, f, indent=1)


def cfg1_matrix(seed=1):
    """cfg1: V=1024 x 16 table, base 32, 2 digits -> the 16 x 64 stack."""
    rng = np.random.default_rng(seed)
    digit_tables = [rng.normal(0.0, 0.1, size=(32, 16)) for _ in range(2)]
    return np.concatenate(digit_tables, axis=0).T.astype(np.float32)  # (16, 64)


def block_diag_matrix(vocab, base, dim, std, seed):
    rng = np.random.default_rng(seed)
    widths = [base * math.ceil(math.log(int(v), base)) for v in vocab]
    M = np.zeros((dim * len(vocab), sum(widths)), dtype=np.float32)
    r = c = 0
    for w in widths:
        M[r:r + dim, c:c + w] = rng.normal(0.0, std, size=(dim, w))
        r += dim
        c += w
    return M


def cfg2_vocab(seed=0):
    rng = np.random.default_rng(seed)
    return np.floor(np.exp(rng.uniform(np.log(3), np.log(1e7), 26))).astype(np.int64)


def _diag_arrays(diags_by_block):
    (blk,) = list(diags_by_block.keys())
    d = diags_by_block[blk]
    ks = np.array(sorted(d.keys()), dtype=np.int64)
    vals = np.array([d[k] for k in ks], dtype=np.float32)
    return ks, vals


def make_diagonalize(packing):
    import scipy.sparse as sp
    res = {}
    m = np.arange(16, dtype=np.float32).reshape(4, 4)
    ks, vals = _diag_arrays(packing.diagonalize(sp.csr_matrix(m), 4, "hybrid", True)[0])
    res["doc_ks"], res["doc_vals"] = ks, vals

    M1 = cfg1_matrix()
    d, rots, _ = packing.diagonalize(sp.csr_matrix(M1), 4096, "hybrid", False)
    res["cfg1_matrix"] = M1
    res["cfg1_ks"], res["cfg1_vals"] = _diag_arrays(d)
    res["cfg1_output_rotations"] = np.array(rots)

    vocab_small = np.array([3, 40, 70, 5000, 9, 200] * 4 + [64, 65], dtype=np.int64)
    Ms = block_diag_matrix(vocab_small, 8, 4, 0.05, seed=3)
    d, rots, _ = packing.diagonalize(sp.csr_matrix(Ms), 2048, "hybrid", False)
    res["small_matrix"] = Ms
    res["small_ks"], res["small_vals"] = _diag_arrays(d)
    res["small_output_rotations"] = np.array(rots)

    V = cfg2_vocab()
    M2 = block_diag_matrix(V, 64, 16, 0.05, seed=0)
    d, rots, _ = packing.diagonalize(sp.csr_matrix(M2), 32768, "hybrid", False)
    ks, vals = _diag_arrays(d)
    res["cfg2_vocab"] = V
    res["cfg2_shape"] = np.array(M2.shape)
    res["cfg2_ks"] = ks
    res["cfg2_output_rotations"] = np.array(rots)
    res["cfg2_sha256"] = np.frombuffer(hashlib.sha256(vals.tobytes()).digest(), dtype=np.uint8)
    res["cfg2_sample"] = vals[:, ::997].copy()
    np.savez_compressed(os.path.join(HERE, "diagonalize.npz"), **res)


def make_bsgs_calls(cb, fake):
    cases = []
    slots = 64
    specs = [
        ("identity", [0], 1.0),
        ("permute", [3], 1.0),
        ("multi", [0, 1], 1.0),
        ("bsgs5", [0, 1, 2, 5, 8], 2.0),
        ("naive3", [0, 2, 7], "none"),
    ]
    rng = np.random.default_rng(42 + 50)
    specs.append(("stress50", sorted(rng.choice(slots, size=50, replace=False).tolist()), 2.0))
    for name, ks, ratio in specs:
        lib = cb.CheddarLibrary(hoist_mode="single")
        lib._default_scale = 1 << 26
        fake.calls.clear()
        data = []
        for k in ks:
            data.extend([float(k + 1 + i / 100.0) for i in range(slots)])
        lt = lib.GenerateLinearTransform(ks, data, 3, ratio, "none")
        encodes = [c for c in fake.calls if c[0] == "Encode"]
        pt_vals = {int(c[1]): fake.pt_values[c[1]] for c in encodes}
        t = lib._transforms[lt]
        keys = lib.GetLinearTransformRotationKeys(lt)
        fake.calls.clear()
        fake.levels[1000] = 3
        lib.EvaluateLinearTransform(lt, 1000)
        cases.append({
            "name": name, "ks": [int(k) for k in ks], "ratio": ratio, "slots": slots,
            "bs": t["bs"], "use_bsgs": t["use_bsgs"],
            "pt_ids": {str(k): int(v) for k, v in t["pt_ids"].items()},
            "pt_values": {str(k): v for k, v in pt_vals.items()},
            "rotation_keys": [int(k) for k in keys],
            "eval_calls": fake.calls[:],
        })
    with open(os.path.join(HERE, "bsgs_calls.json"), "w") as f:
        json.dump(cases, f)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HELRM_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_golden.py <reference checkout>")
    packing, cb, fake = _import_reference(ref)
    make_primes(cb)
    make_diagonalize(packing)
    make_bsgs_calls(cb, fake)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
