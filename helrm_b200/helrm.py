"""The end-to-end HE-LRM forward on the B200 backend.

Restates the reference's encrypted recommendation model,
examples/criteo/dlrm.py:181-229 (HELRM): the bottom MLP
13-512-256-64-16 with a ReLU after every layer (dlrm.py:131-143,
last_relu=True), `bottom_to_top` copying its 16 outputs into slots 0..15
of the 432-wide top input, the block-diagonal embedding product over the
concatenated one-hot digits with `sparse_to_top` copying its 416 outputs
into slots 16..431 (dlrm.py:173-178 copy_into), their sum, and the top MLP
432-512-256-1 (ReLUs between its layers only).  One ciphertext carries
one query; a batch of ciphertexts goes through every layer together.

The encrypted layers follow Orion's modules:

* Linear (orion/nn/linear.py:99-140): the BSGS transform, rescale, hybrid
  fold and bias add of helrm_b200.mlp.LinearLayer;
* ReLU (orion/nn/activation.py:246-300): x <- x * prescale (a level when
  the prescale is not 1), the composite minimax sign [15, 15, 27] stage by
  stage with the last stage's output scale set to the prime of its output
  level, x * step(x) and its rescale, the integer postscale; prescale =
  1 / ceil(margin * max |input|) when that exceeds 1 (activation.py:
  263-270);
* Bootstrap (orion/nn/operations.py:38-115): shift by the fitted centre,
  multiply by a plaintext holding the prescale in the first `elements`
  slots and zeros after them (encoded at the input level's prime), the
  bootstrap over 2^ceil(log2 elements) slots, then the integer postscale
  and the shift back; placed, as Orion's placement does for a ReLU whose
  sign no longer fits the remaining levels, after the ReLU's prescale and
  before its sign (the order a recorded Orion trace shows).

Ranges come from a cleartext forward over a seeded calibration batch
(Orion's fit, orion/core/orion.py: fit) with margin 2.  Every ciphertext
keeps exactly the input scale through the network: the transforms'
diagonals and the prescale plaintexts are encoded at the prime their
rescale drops, so the two branches meet at the add with equal scales.
"""
from __future__ import annotations

import math

import numpy as np
from numpy.polynomial import chebyshev as _cheb

from . import workload as W
from .mlp import LinearLayer, random_mlp

DENSE = 13
EMB = W.EMB_DIM
BOTTOM = (DENSE, 512, 256, 64, EMB)
TOP_HIDDEN = (512, 256)
SIGN_DEGREES = (15, 15, 27)
SIGN_DEPTH = sum(math.ceil(math.log2(d + 1)) for d in SIGN_DEGREES)
MARGIN = 2


def dense_inputs(n: int, seed: int) -> np.ndarray:
    """n x 13 dense features ~ lognormal(0, 1), then log1p."""
    rng = np.random.default_rng(seed)
    return np.log1p(rng.lognormal(0.0, 1.0, size=(n, DENSE)))


def copy_into(width: int, out: int, start: int) -> np.ndarray:
    """dlrm.py:173-178: an (out x width) matrix with eye(width) at rows
    start..start+width-1."""
    M = np.zeros((out, width), dtype=np.float32)
    M[start:start + width, :width] = np.eye(width, dtype=np.float32)
    return M


def sign_stages(coeffs_flat, degrees=SIGN_DEGREES):
    out, o = [], 0
    for d in degrees:
        out.append(np.asarray(coeffs_flat[o:o + d + 1], dtype=np.float64))
        o += d + 1
    return out


def relu_poly(x, stages, prescale: float, postscale: int) -> np.ndarray:
    """The encrypted ReLU on cleartext: postscale * (p x) * step(p x) with
    the composite polynomial for step (Chebyshev series on [-1, 1])."""
    y = np.asarray(x, dtype=np.float64) * prescale
    s = y
    for c in stages:
        s = _cheb.chebval(s, c)
    return postscale * y * s


class _ReLU:
    def __init__(self, absmax: float):
        a = absmax * MARGIN
        self.postscale = int(math.ceil(a)) if a > 1 else 1
        self.prescale = 1.0 / self.postscale
        self.boot = None        # _Boot when a bootstrap precedes the sign
        self.level_in = None    # the ReLU input level
        self.pre_pt = None


class _Boot:
    def __init__(self, lo: float, hi: float, elements: int, slots: int):
        center, half = (lo + hi) / 2, (hi - lo) / 2
        low, high = center - MARGIN * half, center + MARGIN * half
        self.postscale, self.prescale = 1, 1.0
        if high - low > 2:
            self.postscale = int(math.ceil((high - low) / 2))
            self.prescale = 1.0 / self.postscale
        self.constant = -(low + high) / 2
        self.elements = int(elements)
        self.n = 1 << max(0, math.ceil(math.log2(max(1, elements))))
        self.n = min(self.n, slots)
        self.level_in = None
        self.mask_pt = None


class HELRM:
    """The config-4 network on a B200Library scheme created with the
    bootstrapping primes reserved (CKKSConfig(boot=True)).

    vocab: the tables' vocabulary sizes (default: config 2's 26);
    base: the digit base of the compressed one-hot selectors;
    ratio / emb_ratio: BSGS ratios of the MLP layers / the embedding (None:
    32 baby steps, 64 above 512 diagonals);
    boot_chunk: ciphertexts per bootstrap batch (bounds the working set);
    build=False stops after the fit and the level plan."""

    def __init__(self, lib, *, vocab=None, base: int = 64, bottom=BOTTOM, top_hidden=TOP_HIDDEN, seed: int = 0,
                 fit_queries: int = 256, ratio: float | None = None, emb_ratio: float | None = None,
                 boot_chunk: int = 32,
                 build: bool = True):
        self.lib = lib
        info = lib.scheme_info()
        self.slots = info["slots"]
        self.scale = float(lib._default_scale)
        self.chain = [float(q) for q in lib.GetModuliChain()]
        self.top_level = len(self.chain) - 1
        if len(lib.GetAllModuliChain()) == len(self.chain):
            raise RuntimeError("HELRM: the scheme needs the reserved bootstrapping primes (CKKSConfig(boot=True))")
        self.vocab = np.asarray(W.cfg2_vocab() if vocab is None else vocab, dtype=np.int64)
        self.base = int(base)
        self.boot_chunk = int(boot_chunk)
        fields = len(self.vocab)
        self.bottom_w = random_mlp(list(bottom), seed)
        top = [EMB * (fields + 1)] + list(top_hidden) + [1]
        self.top_w = random_mlp(top, seed + 1)
        self.emb = W.block_diag_matrix(self.vocab, self.base, EMB, 0.05, seed=seed + 2)
        self.b2t = copy_into(EMB, top[0], 0)
        self.s2t = copy_into(EMB * fields, top[0], EMB)
        self.sel_width = self.emb.shape[1]
        if max(self.sel_width, top[0], max(bottom), max(top)) > self.slots:
            raise ValueError("HELRM: a layer is wider than the ciphertext's slots")
        self._fit(fit_queries, seed)
        self._plan()
        if build:  # without: the fit and the level plan only (no device objects)
            self._compile(ratio, emb_ratio)

    # ------------------------------------------------------------ cleartext
    def selectors(self, queries) -> np.ndarray:
        return np.stack([W.selector(q, self.vocab, self.base) for q in queries])

    def cleartext(self, dense, sel, poly: bool = True, trace=None) -> np.ndarray:
        """Logits of the network on cleartext inputs (fp64): with poly the
        encrypted ReLUs' composite polynomial, else max(x, 0).  trace, a
        list, collects every ReLU input (the fit)."""
        relus = iter(self.relus) if poly else None

        def act(x):
            if trace is not None:
                trace.append(x)
            if not poly:
                return np.maximum(x, 0)
            r = next(relus)
            return relu_poly(x, self.stages, r.prescale, r.postscale)

        x = np.asarray(dense, dtype=np.float64)
        for w, b in self.bottom_w:
            x = act(x @ w.T.astype(np.float64) + b)
        d = x @ self.b2t.T.astype(np.float64)
        s = (np.asarray(sel, dtype=np.float64) @ self.emb.T.astype(np.float64)) @ self.s2t.T.astype(np.float64)
        x = d + s
        for i, (w, b) in enumerate(self.top_w):
            x = x @ w.T.astype(np.float64) + b
            if i < len(self.top_w) - 1:
                x = act(x)
        return x[:, 0]

    def _fit(self, n: int, seed: int):
        dense = dense_inputs(n, seed + 100)
        sel = self.selectors(W.zipf_queries(self.vocab, n, seed=seed + 101))
        trace: list = []
        self.cleartext(dense, sel, poly=False, trace=trace)
        self.relus = [_ReLU(float(np.abs(t).max())) for t in trace]
        self._relu_in = [(float(t.min()), float(t.max()), t.shape[1]) for t in trace]
        self.stages = sign_stages(self.lib.GenerateMinimaxSignCoeffs(list(SIGN_DEGREES), 128, 6, 12, 0))

    # ------------------------------------------------------------ levels
    def _plan(self):
        """Levels of every layer from the top of the usable chain, with a
        bootstrap before a ReLU's sign whenever the sign and the product
        would leave fewer levels than the layers up to the next ReLU need
        (the next transform, its prescale and the bootstrap's mask)."""
        T = self.top_level
        nb = len(self.bottom_w)
        nt = len(self.top_w)
        self.boots = 0
        plan = []

        def relu(i, lvl, reserve):
            r = self.relus[i]
            r.level_in = lvl
            if r.prescale != 1.0:
                lvl -= 1
            lo, hi, width = self._relu_in[i]
            if lvl - SIGN_DEPTH - 1 < reserve:
                if lvl < 1:
                    raise RuntimeError("HELRM: no level left for the bootstrap's mask")
                r.boot = _Boot(lo * r.prescale, hi * r.prescale, width, self.slots)
                r.boot.level_in = lvl
                self.boots += 1
                lvl = T
            out = lvl - SIGN_DEPTH - 1
            if out < 0:
                raise RuntimeError("HELRM: the usable chain is too short for one ReLU")
            plan.append(("relu", i, r.level_in, out, r.boot is not None))
            return out

        lvl = T
        self.level_dense = T
        self.bottom_levels = []
        for i in range(nb):
            self.bottom_levels.append(lvl)
            lvl -= 1
            reserve = 3 if i < nb - 1 else 4
            lvl = relu(i, lvl, reserve)
        self.level_b2t = lvl
        lvl -= 1
        self.level_add = lvl
        self.level_sel = lvl + 2
        if self.level_sel > T:
            raise RuntimeError("HELRM: the selector would sit above the top of the chain")
        self.top_levels = []
        for i in range(nt):
            self.top_levels.append(lvl)
            lvl -= 1
            if i < nt - 1:
                reserve = 3 if i < nt - 2 else 1
                lvl = relu(nb + i, lvl, reserve)
        self.level_out = lvl
        self.plan = plan

    # ------------------------------------------------------------ compile
    def _compile(self, ratio: float, emb_ratio: float):
        lib = self.lib
        nb = len(self.bottom_w)
        self.bottom = [LinearLayer(lib, w, b, lvl, ratio=ratio, narrow=False)
                       for (w, b), lvl in zip(self.bottom_w, self.bottom_levels)]
        self.b2t_layer = LinearLayer(lib, self.b2t, None, self.level_b2t, ratio=ratio, narrow=False)
        self.emb_layer = LinearLayer(lib, self.emb, None, self.level_sel, ratio=emb_ratio, narrow=False)
        self.s2t_layer = LinearLayer(lib, self.s2t, None, self.level_sel - 1, ratio=ratio, narrow=False)
        nt = len(self.top_w)
        self.top = [LinearLayer(lib, w, b, lvl, last=(i == nt - 1), ratio=ratio, narrow=False)
                    for i, ((w, b), lvl) in enumerate(zip(self.top_w, self.top_levels))]
        self.polys = [lib.GenerateChebyshev(list(c)) for c in self.stages]
        if sum(lib.GetPolyDepth(p) for p in self.polys) != SIGN_DEPTH:
            raise RuntimeError("HELRM: the sign stages' depth differs from the level plan's")
        S = self.slots
        for r in self.relus:
            if r.prescale != 1.0:
                r.pre_pt = lib.Encode([r.prescale] * S, r.level_in, self.chain[r.level_in])
            if r.boot is not None:
                b = r.boot
                v = np.zeros(S)
                v[:b.elements] = b.prescale
                b.mask_pt = lib.Encode(list(v), b.level_in, self.chain[b.level_in])
                lib.NewBootstrapper(None, b.n)
        lib.Synchronize()

    def close(self):
        lib = self.lib
        for layer in self.bottom + self.top + [self.b2t_layer, self.emb_layer, self.s2t_layer]:
            layer.close()
        for r in self.relus:
            if r.pre_pt is not None:
                lib.DeletePlaintext(r.pre_pt)
            if r.boot is not None and r.boot.mask_pt is not None:
                lib.DeletePlaintext(r.boot.mask_pt)

    def info(self) -> dict:
        return {"levels": {"dense": self.level_dense, "selector": self.level_sel, "add": self.level_add,
                           "out": self.level_out},
                "bootstraps_per_query": self.boots,
                "boot_slots": [r.boot.n for r in self.relus if r.boot is not None],
                "relu_postscales": [r.postscale for r in self.relus],
                "plan": self.plan}

    # ------------------------------------------------------------ encrypted
    def encrypt(self, dense, sel):
        """Ciphertexts of the dense features (slots 0..12, top level) and of
        the selectors (slots 0..width-1, the embedding's level)."""
        lib = self.lib
        out = []
        for rows, level in ((dense, self.level_dense), (sel, self.level_sel)):
            pts = lib.EncodeBatch(np.asarray(rows, dtype=np.float64), level, self.scale)  # zero-padded on the device
            cts = [lib.Encrypt(p) for p in pts]
            for p in pts:
                lib.DeletePlaintext(p)
            out.append(cts)
        return out[0], out[1]

    def decrypt(self, cts) -> np.ndarray:
        lib = self.lib
        out = []
        for c in cts:
            pt = lib.Decrypt(c)
            out.append(lib.Decode(pt)[0])
            lib.DeletePlaintext(pt)
        return np.array(out)

    def _free(self, ids):
        for c in ids:
            self.lib.DeleteCiphertext(c)

    def _relu(self, xs, r: _ReLU) -> list[int]:
        lib = self.lib
        if r.pre_pt is not None:
            for x in xs:
                lib.MulPlaintext(x, r.pre_pt)
            lib.RescaleBatch(xs)
        if r.boot is not None:
            b = r.boot
            for x in xs:
                if b.constant != 0:
                    lib.AddScalar(x, b.constant)
                lib.MulPlaintext(x, b.mask_pt)
            lib.RescaleBatch(xs)
            booted = []
            for i in range(0, len(xs), self.boot_chunk):
                booted += lib.BootstrapBatch(xs[i:i + self.boot_chunk], b.n)
            self._free(xs)
            xs = booted
            for x in xs:
                if b.postscale != 1:
                    lib.MulScalarInt(x, b.postscale)
                if b.constant != 0:
                    lib.SubScalar(x, b.constant)
        cur = xs
        out_level = lib.GetCiphertextLevel(xs[0]) - SIGN_DEPTH
        for i, p in enumerate(self.polys):
            target = self.chain[out_level] if i == len(self.polys) - 1 else self.scale
            nxt = lib.EvaluatePolynomialBatch(cur, p, target)
            if cur is not xs:
                self._free(cur)
            cur = nxt
        res = lib.MulRelinCiphertextBatchNew(xs, cur)
        lib.RescaleBatch(res)
        self._free(cur)
        self._free(xs)
        if r.postscale != 1:
            for y in res:
                lib.MulScalarInt(y, r.postscale)
        return res

    def forward(self, dense_cts, sel_cts) -> list[int]:
        """The encrypted logits (slot 0) of a batch of queries; the inputs
        are left untouched."""
        if len(dense_cts) != len(sel_cts):
            raise ValueError("HELRM: one dense and one selector ciphertext per query")
        nb = len(self.bottom)
        x = list(dense_cts)
        for i, layer in enumerate(self.bottom):
            y = layer.forward(x)
            if i:
                self._free(x)
            x = self._relu(y, self.relus[i])
        d = self.b2t_layer.forward(x)
        self._free(x)
        e = self.emb_layer.forward(list(sel_cts))
        s = self.s2t_layer.forward(e)
        self._free(e)
        x = [self.lib.AddCiphertextNew(a, b) for a, b in zip(d, s)]
        self._free(d)
        self._free(s)
        for i, layer in enumerate(self.top):
            y = layer.forward(x)
            self._free(x)
            x = self._relu(y, self.relus[nb + i]) if i < len(self.top) - 1 else y
        return x
