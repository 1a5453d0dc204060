"""The HE-LRM MLP linear layers on the GPU path (helrm_b200/mlp.py).

The bottom MLP's four linear layers (13-512-256-64-16, BASELINE config 4,
without the activations, which are the polynomial evaluator's part) run
through the same BSGS kernels as the embedding PCMM: transform, rescale,
hybrid fold, fold-retag narrowing and bias add.  Checked:

* one layer bit-exact against the oracle's transform -> rescale -> fold
  followed by the bias plaintext's add;
* the four-layer chain decrypted against the cleartext chain within the
  north star's logit tolerance (max abs error 1e-3);
* the square method of the network's last transform (256 -> 1, no fold);
* the narrowing retag: the folded output reports the fold's period.
"""
import numpy as np
import pytest

from gpu_helpers import Pair
from helrm_b200 import CKKSConfig, mlp
from helrm_b200 import workload as W

pytestmark = pytest.mark.gpu

CFG = CKKSConfig(logn=12, logq=[40] + [36] * 6, logp=[60, 60], logscale=36, h=64)


@pytest.fixture(scope="module")
def pair(oracle_mod):
    p = Pair(CFG, dnum=3, seed=20261220, oracle_mod=oracle_mod)
    yield p
    p.close()


def _dense(n, seed):
    rng = np.random.default_rng(seed)
    return np.log1p(rng.lognormal(0.0, 1.0, n))  # config 4's dense features


def _enc(pair, x, level):
    v = np.zeros(pair.slots)
    v[:len(x)] = x
    return pair.encrypt(v, level)


def test_layer_bit_exact_vs_oracle(pair):
    level = pair.info["max_level"]
    (w, b), = mlp.random_mlp([13, 512], seed=1)
    layer = mlp.LinearLayer(pair.lib, w, b, level)
    ct = _enc(pair, _dense(13, 2), level)
    out = layer.forward([ct])[0]
    assert pair.lib.GetCiphertextSlots(out) == layer.period == 512
    o = pair.o
    plan = W.bsgs_plan(layer.ks, 2.0, pair.slots)
    gal = {o.galois(d) for d in plan["rotation_keys"]} | {o.galois(pair.slots >> i) for i in range(1, layer.rot + 1)}
    keys = {g: pair.key(g) for g in gal}
    pts = [pair.lib.GetLinearTransformPlaintext(layer.lt, k) for k in layer.ks]
    y = o.pcmm(pair.ct_data(ct), layer.ks, pts, plan["stride"], keys, layer.rot)
    bias_pt = layer._bias_for(pair.lib.GetCiphertextScale(out))
    bres = pair.lib.GetPlaintextData(bias_pt)
    y[0] = o.fold_add(y[:1], bres[None])[0]
    assert np.array_equal(pair.ct_data(out), y)
    layer.close()


def test_bottom_mlp_chain_within_logit_tolerance(pair):
    level = pair.info["max_level"]
    layers = mlp.random_mlp([13, 512, 256, 64, 16], seed=3)
    xs = [_dense(13, 10 + i) for i in range(3)]
    cts = [_enc(pair, x, level) for x in xs]
    enc_layers = []
    for i, (w, b) in enumerate(layers):
        layer = mlp.LinearLayer(pair.lib, w, b, level - i)
        enc_layers.append(layer)
        cts = layer.forward(cts)
    for x, c in zip(xs, cts):
        ref = x
        for w, b in layers:
            ref = w.astype(np.float64) @ ref + b
        got = pair.decrypt(c)[:16]
        assert np.abs(got - ref).max() <= 1e-3
        assert pair.lib.GetCiphertextLevel(c) == level - 4
    for layer in enc_layers:
        layer.close()


def test_square_last_layer(pair):
    level = 3
    (w, b), = mlp.random_mlp([256, 1], seed=5)
    layer = mlp.LinearLayer(pair.lib, w, b, level, last=True)
    assert layer.rot == 0 and layer.folded_slots is None
    x = np.random.default_rng(6).normal(0, 0.5, 256)
    out = layer.forward([_enc(pair, x, level)])[0]
    ref = (w.astype(np.float64) @ x + b)[0]
    assert abs(pair.decrypt(out)[0] - ref) <= 1e-3
    layer.close()
