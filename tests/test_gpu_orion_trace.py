"""The reference's Orion driving the B200 backend, replayed on the GPU.

tests/golden/make_orion_trace.py ran the reference's own flow (init_scheme,
fit, compile, encode, encrypt, the encrypted forward of an ``on.Linear``
and of an ``on.Embedding`` layer, decrypt, decode; orion/core/orion.py,
orion/nn/linear.py:99-140, orion/backend/python/lt_evaluator.py:224-275),
and of a Linear -> ReLU -> Linear network whose ReLU is Orion's composite
minimax sign [15, 15, 27] (orion/nn/activation.py:201-300: the sign
coefficients from GenerateMinimaxSignCoeffs, three EvaluatePolynomial
stages at the levels Orion's compiler placed, x * step(x)), and of a
network with two ReLUs over a chain too short for both, where Orion's own
bootstrap placement (orion/core/auto_bootstrap.py) inserted two
NewBootstrapper / Bootstrap calls (orion/nn/operations.py:38-115), and
of the reference's own HE-LRM model (examples/criteo/dlrm.py:181-229:
bottom MLP with ReLUs, the block-diagonal embedding, the two copy-into
layers, the add, the top MLP; module widths narrowed to fit LogN 13),
two encrypted inputs and three Orion-placed bootstraps,
with ``backend: b200`` registered through helrm_b200.orion_adapter and
recorded every backend call, in order, with its arguments.  The reference
cannot travel to the GPU box, so the calls are replayed here on the real
B200Library: the same methods, the same arguments (the diagonals and bias
vectors Orion's compiler produced), handles mapped from the recording.
The decrypted outputs must match the cleartext forward of the same
networks (recorded with the trace) within the north star's 1e-3 bound, and
every handle the replay returns must be of the kind the recording saw.
"""
import json
import os

import numpy as np
import pytest

from helrm_b200 import B200Library, CKKSConfig

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load():
    with open(os.path.join(GOLDEN, "orion_trace.json")) as f:
        trace = json.load(f)
    arrays = dict(np.load(os.path.join(GOLDEN, "orion_trace.npz")))
    return trace, arrays


def _replay(kind):
    trace, arrays = _load()
    t = trace[kind]
    p = t["params"]
    lib = B200Library(seed=17, device=0)
    lib.setup_bindings(CKKSConfig(logn=p["logn"], logq=p["logq"], logp=p["logp"], logscale=p["logscale"],
                                  h=p["h"], boot=bool(p.get("boot", False))))
    handles = {}
    decoded = {}
    try:
        def arg(a):
            if isinstance(a, dict) and "array" in a:
                return list(arrays[f"{kind}/{a['array']}"])
            if isinstance(a, dict):
                (k, v), = a.items()
                return handles[(k, v)]
            return a

        for i, c in enumerate(t["calls"]):
            res = getattr(lib, c["m"])(*[arg(a) for a in c["a"]])
            r = c["r"]
            if isinstance(r, dict):
                (k, v), = r.items()
                assert isinstance(res, int) and res > 0, (c["m"], res)
                handles[(k, v)] = res
            elif c["m"] == "GetLinearTransformRotationKeys":
                assert sorted(res) == sorted(r)  # the same key set the recording planned
            elif c["m"] == "GenerateMinimaxSignCoeffs":
                assert np.allclose(res, r, rtol=0, atol=1e-12)
            if c["m"] == "Decode":
                decoded[i] = np.asarray(res)
        out = decoded[t["output_decode_calls"][0]]
        return out, np.asarray(t["cleartext_output"])
    finally:
        lib.DeleteScheme()


@pytest.mark.parametrize("kind", ["linear", "embedding", "mlp_relu", "mlp_boot", "helrm"])
def test_orion_flow_replayed_on_b200(kind):
    out, clear = _replay(kind)
    n = len(clear)
    assert np.abs(out[:n] - clear).max() <= 1e-3
