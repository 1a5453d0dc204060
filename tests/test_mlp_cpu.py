"""MLP linear-layer semantics on CPU (helrm_b200/mlp.py).

The encrypted layer's output slots, computed on cleartext from the layer's
own diagonals, fold and tiled bias, must equal W x + b in the first
out_features slots, repeat with the fold's period (hybrid method), and
leave the square method's output unfolded (the network's last transform,
orion/core/orion.py:258-272).  A recording stand-in replaces the GPU
library: the test exercises the host logic only.
"""
import numpy as np
import pytest

from helrm_b200 import mlp


class RecordingLib:
    def __init__(self, slots):
        self.slots = slots
        self.calls = []

    def scheme_info(self):
        return {"slots": self.slots, "N": 2 * self.slots}

    def GenerateLinearTransform(self, ks, data, level, ratio, io):
        self.calls.append(("lt", len(ks), level, ratio))
        return 1

    def GetLinearTransformRotationKeys(self, lt):
        return []

    def GenerateLinearTransformRotationKey(self, k):
        pass

    def AddRotationKey(self, k):
        self.calls.append(("key", k))

    def DeleteLinearTransform(self, lt):
        pass


@pytest.mark.parametrize("shape", [(512, 13), (256, 512), (64, 256), (16, 64), (512, 432)])
def test_hybrid_layer_matches_matrix_product(shape):
    slots = 2048
    rng = np.random.default_rng(shape[0] + shape[1])
    (w, b), = mlp.random_mlp([shape[1], shape[0]], seed=shape[0])
    lib = RecordingLib(slots)
    layer = mlp.LinearLayer(lib, w, b, level=5)
    x = rng.normal(0, 1, shape[1])
    y = layer.cleartext(x)
    ref = w.astype(np.float64) @ x + b
    assert np.allclose(y[:shape[0]], ref, atol=1e-9)
    P = layer.period
    assert P == 2 ** int(np.ceil(np.log2(shape[0]))) and layer.rot == int(np.log2(slots // P))
    assert np.allclose(y.reshape(-1, P), y[:P][None, :])  # periodic after the fold
    assert layer.folded_slots == P
    assert ("key", slots >> 1) in lib.calls  # fold keys requested


def test_square_last_layer_has_no_fold():
    slots = 2048
    (w, b), = mlp.random_mlp([256, 1], seed=9)
    lib = RecordingLib(slots)
    layer = mlp.LinearLayer(lib, w, b, level=3, last=True)
    assert layer.rot == 0 and layer.folded_slots is None and len(layer.ks) == 256
    x = np.random.default_rng(1).normal(0, 1, 256)
    y = layer.cleartext(x)
    assert abs(y[0] - (w.astype(np.float64) @ x + b)[0]) < 1e-9
