"""Golden composite sign-polynomial coefficients from the reference.

Runs the reference's own ``CheddarLibrary.GenerateMinimaxSignCoeffs``
(orion/backend/cheddar/bindings.py:1164-1230, pure numpy) for the degree
lists Orion's ReLU and sign layers use (orion/nn/activation.py:201-300,
defaults [15, 15, 27] with logalpha 6) and the reference's own test cases
(tests/oracle/test_poly_eval.py:100-116), and writes minimax_sign.json.
The native Cheddar module and a few plotting/IO packages are absent here:
empty stand-in modules take their import slots (the coefficient generator
never calls them).

    python tests/golden/make_minimax_sign.py /path/to/reference
"""
from __future__ import annotations

import json
import os
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    ([15, 15, 27], 128, 6, 12),
    ([15, 15, 27], 128, 12, 12),
    ([7], 64, 6, 6),
    ([3, 5], 64, 6, 6),
    ([7, 15], 128, 8, 12),
]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    os.environ.pop("ORION_CHEDDAR_WORD32", None)  # the 64-bit word build's fit
    # modules the orion package imports that this image does not have
    for name in ["matplotlib", "matplotlib.pyplot", "h5py", "opt_einsum", "desilofhe"]:
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules.setdefault("orion.backend.cheddar._cheddar_native",
                           types.ModuleType("orion.backend.cheddar._cheddar_native"))
    from orion.backend.cheddar.bindings import CheddarLibrary

    lib = object.__new__(CheddarLibrary)
    out = []
    for degrees, prec, logalpha, logerr in CASES:
        coeffs = lib.GenerateMinimaxSignCoeffs(list(degrees), prec, logalpha, logerr, 0)
        out.append({"degrees": degrees, "prec": prec, "logalpha": logalpha, "logerr": logerr,
                    "coeffs": [float(c) for c in coeffs]})
    with open(os.path.join(HERE, "minimax_sign.json"), "w") as f:
        json.dump({"source": "orion/backend/cheddar/bindings.py:1164-1230", "cases": out}, f, indent=1)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HELRM_REFERENCE", ""))
