"""Linear layers of the HE-LRM bottom and top MLPs through the same
linear-transform kernels as the embedding PCMM.

Restates the reference's encrypted Linear layer:

* compile (orion/nn/linear.py:189-209, orion/core/packing.py:495-533): the
  weight matrix (one input row per ciphertext here, so the Kronecker
  product with eye(N) is the matrix itself) is diagonalised with the
  hybrid method, or with the square method for the network's last linear
  transform (orion/core/orion.py:258-272), and handed to
  GenerateLinearTransform; the bias is encoded one level below the
  transform;
* forward (orion/nn/linear.py:99-140, lt_evaluator.py:262-273): the BSGS
  transform, the rescale, the hybrid fold out += rot(out, slots / 2^i)
  for i = 1..output_rotations, the fold-retag narrowing to the fold's
  period (SetCiphertextSlots, metadata only), then the bias add.

The backend works on full-width ciphertexts: after the fold the output is
periodic with period bh (the block height), and the bias is tiled with
the same period, so the full-width and the narrowed views agree.  The
bias plaintext is encoded at the exact scale the rescaled output carries
(the input's: the diagonals sit at the dropped prime), so the add needs no
scale-drift absorption.
"""
from __future__ import annotations

import numpy as np

from . import workload as W


class LinearLayer:
    """One encrypted Linear layer (weight out x in, bias out) on a
    B200Library scheme, evaluated on a batch of ciphertexts that each hold
    one input vector in slots 0..in-1 (any period-replicated copies beyond
    are ignored: the diagonals read only the first copy).  narrow retags
    the folded output to its period; ratio None picks the BSGS split with
    32 baby steps (64 above 512 diagonals)."""

    def __init__(self, lib, weight: np.ndarray, bias, level: int, last: bool = False, ratio: float | None = 2.0,
                 narrow: bool = True):
        self.lib = lib
        info = lib.scheme_info()
        self.slots = info["slots"]
        self.weight = np.asarray(weight, dtype=np.float32)
        H, Wd = self.weight.shape
        if max(H, Wd) > self.slots:
            raise ValueError("layer wider than the ciphertext's slots")
        self.has_bias = bias is not None  # Orion's Linear(bias=False) adds nothing
        self.bias = np.zeros(H) if bias is None else np.asarray(bias, dtype=np.float64)
        self.level, self.last = level, last
        d, self.rot = W.diagonalize(self.weight, self.slots, "hybrid", last=last)
        self.diags = d[(0, 0)]
        self.ks = sorted(self.diags)
        data = np.concatenate([self.diags[k].astype(np.float64) for k in self.ks])
        if ratio is None:  # 32 baby steps (64 above 512 diagonals): the fused MAC's full chunks
            bs = 64 if len(self.ks) > 512 else 32
            ratio = bs * bs / float(len(self.ks))
        # the diagonals at q_level (GenerateLinearTransform's rule): the
        # rescaled output keeps the input's scale exactly
        self.lt = lib.GenerateLinearTransform(self.ks, data, level, ratio, "none")
        for k in lib.GetLinearTransformRotationKeys(self.lt):
            lib.GenerateLinearTransformRotationKey(k)
        for i in range(1, self.rot + 1):
            lib.AddRotationKey(self.slots >> i)
        self.period = self.slots >> self.rot
        self.folded_slots = self.period if (narrow and self.rot) else None
        self._bias_pt = {}

    def _bias_for(self, scale: float) -> int:
        key = float(scale)
        if key not in self._bias_pt:
            tiled = np.zeros(self.slots)
            for start in range(0, self.slots, self.period):
                tiled[start:start + len(self.bias)] = self.bias
            self._bias_pt[key] = self.lib.Encode(list(tiled), self.level - 1, key)
        return self._bias_pt[key]

    def forward(self, cts) -> list[int]:
        """New ciphertexts (one level down): W x + b for every input."""
        lib = self.lib
        outs = lib.EvaluateLinearTransformBatch(self.lt, cts)
        lib.RescaleBatch(outs)
        if self.rot:
            lib.HybridFoldBatch(outs, self.rot)
        for o in outs:
            if self.folded_slots and self.folded_slots < lib.GetCiphertextSlots(o):
                lib.SetCiphertextSlots(o, self.folded_slots)
            if self.has_bias:
                lib.AddPlaintext(o, self._bias_for(lib.GetCiphertextScale(o)))
        return outs

    def cleartext(self, x) -> np.ndarray:
        """The layer's output slots on cleartext (tests): the folded
        transform of the padded input plus the tiled bias."""
        v = np.zeros(self.slots)
        v[:len(x)] = x
        y = W.hybrid_fold(W.cleartext_lt(v, self.diags, self.slots), self.slots, self.rot)
        tiled = np.zeros(self.slots)
        for start in range(0, self.slots, self.period):
            tiled[start:start + len(self.bias)] = self.bias
        return y + tiled

    def close(self):
        self.lib.DeleteLinearTransform(self.lt)
        for p in self._bias_pt.values():
            self.lib.DeletePlaintext(p)
        self._bias_pt.clear()


def random_mlp(widths, seed: int = 0):
    """Weights ~ N(0, 1/fan_in) and biases ~ N(0, 0.01) for the widths
    chain (bottom 13-512-256-64-16, top 432-512-256-1)."""
    rng = np.random.default_rng(seed)
    layers = []
    for a, b in zip(widths[:-1], widths[1:]):
        layers.append((rng.normal(0.0, 1.0 / np.sqrt(a), size=(b, a)).astype(np.float32),
                       rng.normal(0.0, 0.1, size=b)))
    return layers
