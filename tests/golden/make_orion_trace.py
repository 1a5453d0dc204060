"""Record the backend calls the reference's Orion makes for ``backend: b200``.

    python tests/golden/make_orion_trace.py <reference checkout>

Runs the reference's own flow (orion/core/orion.py: init_scheme, fit,
compile, encode, encrypt, the encrypted forward, decrypt, decode) for small
networks (an ``on.Linear`` layer, an ``on.Embedding`` layer, ReLU MLPs with
and without placed bootstraps, and the reference's HELRM model of
examples/criteo/dlrm.py with its widths narrowed), with
``helrm_b200.orion_adapter.install()`` registering ``backend: b200``.  The
backend object handed to Orion here is a recording stand-in with the
B200Library's method names and its level, scale and slot rules (this
machine has no GPU); every call Orion makes on it is written, in order, to
``orion_trace.json`` with the array arguments in ``orion_trace.npz``,
together with the cleartext forward of each network.  The GPU test
``tests/test_gpu_orion_trace.py`` replays the calls on the real B200Library
and compares the decrypted result with the cleartext forward.

Test infrastructure only: the trace is a fixture, the reference is needed
only to regenerate it.
"""
from __future__ import annotations

import json
import math
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

CONFIG = {
    "ckks_params": {"LogN": 13, "LogQ": [40, 36, 36, 36, 36, 36], "LogP": [60, 60], "LogScale": 36, "H": 192,
                    "RingType": "Standard"},
    "orion": {"backend": "b200", "io_mode": "none", "debug": False, "embedding_method": "hybrid", "margin": 2},
}
# the ReLU network: 20 primes, enough levels for Linear -> ReLU (15 levels:
# prescale, the [15, 15, 27] sign stages, x * step(x)) -> Linear without
# bootstrapping
CONFIG_DEEP = {
    "ckks_params": {"LogN": 13, "LogQ": [40] + [36] * 19, "LogP": [60] * 4, "LogScale": 36, "H": 192,
                    "RingType": "Standard"},
    "orion": dict(CONFIG["orion"]),
}
# the network that needs bootstrapping: two ReLUs (15 levels each) over a
# usable chain of 17 levels, so Orion's placement inserts a bootstrap; the
# boot parameters make the backend reserve its bootstrapping primes
CONFIG_BOOT = {
    "ckks_params": {"LogN": 13, "LogQ": [50] + [36] * 17, "LogP": [60] * 6, "LogScale": 36, "H": 192,
                    "RingType": "Standard"},
    "boot_params": {"LogP": [60] * 6, "num_cts_levels": 1, "num_stc_levels": 1, "log_message_ratio": 14},
    "orion": dict(CONFIG["orion"]),
}


class Recorder:
    """Stand-in backend: hands out handles, tracks level / scale / slots with
    the B200Library's rules, and logs every call."""

    lt_output_prerescaled = False

    def __init__(self, primes):
        self.primes = list(primes)
        self.calls = []
        self.arrays = {}
        self.next_id = 1
        self.cts, self.pts, self.lts, self.polys = {}, {}, {}, {}

    # -- logging helpers -------------------------------------------------
    def _arr(self, values):
        key = f"a{len(self.arrays)}"
        self.arrays[key] = np.asarray(values, dtype=np.float64)
        return {"array": key}

    def _log(self, method, args, result):
        def plain(v):
            if isinstance(v, dict):
                return {k: plain(x) for k, x in v.items()}
            if isinstance(v, (list, tuple)):
                return [plain(x) for x in v]
            if isinstance(v, np.integer):
                return int(v)
            if isinstance(v, np.floating):
                return float(v)
            return v
        self.calls.append({"m": method, "a": plain(args), "r": plain(result)})
        return result

    def _new(self, reg, meta):
        i = self.next_id
        self.next_id += 1
        reg[i] = dict(meta)
        return i

    # -- lifecycle -------------------------------------------------------
    def setup_bindings(self, params):
        self._slots = 1 << (int(params.get_logn()) - 1)
        self._max_level = len(params.get_logq()) - 1
        self._default_scale = float(1 << int(params.get_logscale()))
        self.params = {"logn": int(params.get_logn()), "logq": [int(x) for x in params.get_logq()],
                       "logp": [int(x) for x in params.get_logp()], "logscale": int(params.get_logscale()),
                       "h": int(params.get_hamming_weight()),
                       "boot": params.get_boot_num_cts_levels() is not None}

    def __getattr__(self, name):
        # the setup and key calls Orion makes with nothing to return
        if (name.startswith("New") and name != "NewBootstrapper") or name in ("GenerateSecretKey", "GeneratePublicKey",
                                              "GenerateRelinearizationKey", "GenerateEvaluationKeys",
                                              "DeleteBootstrappers"):
            def noop(*a):
                return self._log(name, list(a), None)
            return noop
        raise AttributeError(f"Recorder: Orion called {name}, which the trace does not model")

    def DeleteScheme(self):
        self._log("DeleteScheme", [], None)

    def GetModuliChain(self):
        return self._log("GetModuliChain", [], [int(p) for p in self.primes])

    # -- encode / encrypt ------------------------------------------------
    def Encode(self, values, level, scale):
        i = self._new(self.pts, {"level": int(level), "scale": float(scale), "slots": self._slots})
        return self._log("Encode", [self._arr(values), int(level), float(scale)], {"pt": i})["pt"]

    def Encrypt(self, pt):
        m = self.pts[pt]
        i = self._new(self.cts, m)
        return self._log("Encrypt", [{"pt": pt}], {"ct": i})["ct"]

    def Decrypt(self, ct):
        i = self._new(self.pts, self.cts[ct])
        return self._log("Decrypt", [{"ct": ct}], {"pt": i})["pt"]

    def Decode(self, pt):
        self._log("Decode", [{"pt": pt}], "values")
        return [0.0] * self._slots

    # -- arithmetic ------------------------------------------------------
    def _ct_new(self, meta):
        return self._new(self.cts, meta)

    def Rescale(self, ct):
        m = self.cts[ct]
        m["scale"] /= self.primes[m["level"]]
        m["level"] -= 1
        return self._log("Rescale", [{"ct": ct}], {"ct": ct})["ct"]

    def RescaleNew(self, ct):
        m = dict(self.cts[ct])
        m["scale"] /= self.primes[m["level"]]
        m["level"] -= 1
        i = self._ct_new(m)
        return self._log("RescaleNew", [{"ct": ct}], {"ct": i})["ct"]

    def RotateNew(self, ct, k):
        i = self._ct_new(self.cts[ct])
        return self._log("RotateNew", [{"ct": ct}, int(k)], {"ct": i})["ct"]

    def Rotate(self, ct, k):
        return self._log("Rotate", [{"ct": ct}, int(k)], {"ct": ct})["ct"]

    def AddRotationKey(self, k):
        self._log("AddRotationKey", [int(k)], None)

    # -- scalars and ciphertext products (the B200Library's scale rules) ---
    def _scalar(self, name, ct, v, inplace, square):
        meta = dict(self.cts[ct])
        if square:
            meta["scale"] = meta["scale"] * meta["scale"]
        if inplace:
            self.cts[ct] = meta
            return self._log(name, [{"ct": ct}, v], {"ct": ct})["ct"]
        i = self._ct_new(meta)
        return self._log(name, [{"ct": ct}, v], {"ct": i})["ct"]

    def MulScalarIntNew(self, ct, v):
        return self._scalar("MulScalarIntNew", ct, int(v), False, False)

    def MulScalarInt(self, ct, v):
        return self._scalar("MulScalarInt", ct, int(v), True, False)

    def MulScalarFloatNew(self, ct, v):
        return self._scalar("MulScalarFloatNew", ct, float(v), False, True)

    def MulScalarFloat(self, ct, v):
        return self._scalar("MulScalarFloat", ct, float(v), True, True)

    def AddScalarNew(self, ct, v):
        return self._scalar("AddScalarNew", ct, float(v), False, False)

    def AddScalar(self, ct, v):
        return self._scalar("AddScalar", ct, float(v), True, False)

    def SubScalarNew(self, ct, v):
        return self._scalar("SubScalarNew", ct, float(v), False, False)

    def SubScalar(self, ct, v):
        return self._scalar("SubScalar", ct, float(v), True, False)

    # -- bootstrapping (the output at the top of the usable chain, the
    # input's scale; helrm_b200/bootstrap.py) ------------------------------
    def NewBootstrapper(self, logp, slots):
        self._log("NewBootstrapper", [None, int(slots)], None)

    def Bootstrap(self, ct, slots):
        meta = dict(self.cts[ct])
        meta["level"] = self._max_level
        i = self._ct_new(meta)
        return self._log("Bootstrap", [{"ct": ct}, int(slots)], {"ct": i})["ct"]

    def _relin(self, name, a, b, inplace):
        ma, mb = self.cts[a], self.cts[b]
        meta = {"level": min(ma["level"], mb["level"]), "scale": ma["scale"] * mb["scale"],
                "slots": max(ma["slots"], mb["slots"])}
        if inplace:
            self.cts[a] = meta
            return self._log(name, [{"ct": a}, {"ct": b}], {"ct": a})["ct"]
        i = self._ct_new(meta)
        return self._log(name, [{"ct": a}, {"ct": b}], {"ct": i})["ct"]

    def MulRelinCiphertextNew(self, a, b):
        return self._relin("MulRelinCiphertextNew", a, b, False)

    def MulRelinCiphertext(self, a, b):
        return self._relin("MulRelinCiphertext", a, b, True)

    # -- polynomials -------------------------------------------------------
    def GenerateMinimaxSignCoeffs(self, degrees, prec, logalpha, logerr, debug):
        sys.path.insert(0, ROOT)
        from helrm_b200.library import _composite_sign_coeffs
        out = _composite_sign_coeffs([int(d) for d in degrees], 2.0 ** (-float(logalpha)))
        return self._log("GenerateMinimaxSignCoeffs", [[int(d) for d in degrees], int(prec), int(logalpha),
                                                       int(logerr), int(debug)], out)

    def _poly(self, name, coeffs):
        c = [float(x) for x in coeffs]
        i = self._new(self.polys, {"n": len(c)})
        return self._log(name, [self._arr(c)], {"poly": i})["poly"]

    def GenerateChebyshev(self, coeffs):
        return self._poly("GenerateChebyshev", coeffs)

    def GenerateMonomial(self, coeffs):
        return self._poly("GenerateMonomial", coeffs)

    def EvaluatePolynomial(self, ct, poly, scale=None):
        n = self.polys[poly]["n"]
        depth = math.ceil(math.log2(n)) if n >= 3 else 1
        meta = dict(self.cts[ct])
        meta["level"] -= depth
        meta["scale"] = float(scale) if scale is not None else self._default_scale
        i = self._ct_new(meta)
        return self._log("EvaluatePolynomial", [{"ct": ct}, {"poly": poly},
                                                None if scale is None else float(scale)], {"ct": i})["ct"]

    def _binary(self, name, a, b, inplace, kind_b="ct"):
        ma = self.cts[a]
        mb = self.cts[b] if kind_b == "ct" else self.pts[b]
        meta = {"level": min(ma["level"], mb["level"]), "scale": ma["scale"], "slots": ma["slots"]}
        if name.startswith("MulPlaintext"):
            meta["scale"] = ma["scale"] * mb["scale"]
        if inplace:
            self.cts[a] = meta
            return self._log(name, [{"ct": a}, {kind_b: b}], {"ct": a})["ct"]
        i = self._ct_new(meta)
        return self._log(name, [{"ct": a}, {kind_b: b}], {"ct": i})["ct"]

    def AddCiphertextNew(self, a, b):
        return self._binary("AddCiphertextNew", a, b, False)

    def AddCiphertext(self, a, b):
        return self._binary("AddCiphertext", a, b, True)

    def SubCiphertextNew(self, a, b):
        return self._binary("SubCiphertextNew", a, b, False)

    def AddPlaintextNew(self, a, b):
        return self._binary("AddPlaintextNew", a, b, False, "pt")

    def AddPlaintext(self, a, b):
        return self._binary("AddPlaintext", a, b, True, "pt")

    def MulPlaintextNew(self, a, b):
        return self._binary("MulPlaintextNew", a, b, False, "pt")

    def MulPlaintext(self, a, b):
        return self._binary("MulPlaintext", a, b, True, "pt")

    # -- linear transforms -------------------------------------------------
    def GenerateLinearTransform(self, idxs, data, level, ratio, io_mode):
        i = self._new(self.lts, {"level": int(level), "ks": [int(k) for k in idxs], "ratio": ratio})
        return self._log("GenerateLinearTransform",
                         [[int(k) for k in idxs], self._arr(data), int(level),
                          ratio if isinstance(ratio, str) else float(ratio), io_mode], {"lt": i})["lt"]

    def GetLinearTransformRotationKeys(self, lt):
        sys.path.insert(0, ROOT)
        from helrm_b200 import workload as W
        t = self.lts[lt]
        r = t["ratio"]
        plan = W.bsgs_plan(t["ks"], "none" if (isinstance(r, str) or float(r) <= 0) else float(r), self._slots)
        return self._log("GetLinearTransformRotationKeys", [{"lt": lt}], list(plan["rotation_keys"]))

    def GenerateLinearTransformRotationKey(self, k):
        self._log("GenerateLinearTransformRotationKey", [int(k)], None)

    def EvaluateLinearTransform(self, lt, ct):
        m = dict(self.cts[ct])
        m["level"] = min(m["level"], self.lts[lt]["level"])
        m["scale"] *= float(self.primes[self.lts[lt]["level"]])  # diagonals at the level's prime
        i = self._ct_new(m)
        return self._log("EvaluateLinearTransform", [{"lt": lt}, {"ct": ct}], {"ct": i})["ct"]

    def DeleteLinearTransform(self, lt):
        # layers of a network recorded earlier in this process are garbage
        # collected while the next one runs, and their __del__
        # (orion/nn/linear.py:41-46) deletes their transforms through the
        # current backend: ids this recorder never handed out are not part
        # of the recorded flow
        if lt not in self.lts:
            return
        self.lts.pop(lt, None)
        self._log("DeleteLinearTransform", [{"lt": lt}], None)

    # -- metadata --------------------------------------------------------
    def DeleteCiphertext(self, ct):
        self.cts.pop(ct, None)
        self._log("DeleteCiphertext", [{"ct": ct}], None)

    def DeletePlaintext(self, pt):
        self.pts.pop(pt, None)
        self._log("DeletePlaintext", [{"pt": pt}], None)

    def GetCiphertextLevel(self, ct):
        return self._log("GetCiphertextLevel", [{"ct": ct}], self.cts[ct]["level"])

    def GetPlaintextLevel(self, pt):
        return self._log("GetPlaintextLevel", [{"pt": pt}], self.pts[pt]["level"])

    def GetCiphertextScale(self, ct):
        return self._log("GetCiphertextScale", [{"ct": ct}], self.cts[ct]["scale"])

    def GetPlaintextScale(self, pt):
        return self._log("GetPlaintextScale", [{"pt": pt}], self.pts[pt]["scale"])

    def SetCiphertextScale(self, ct, s):
        self.cts[ct]["scale"] = float(s)
        self._log("SetCiphertextScale", [{"ct": ct}, float(s)], None)

    def SetPlaintextScale(self, pt, s):
        self.pts[pt]["scale"] = float(s)
        self._log("SetPlaintextScale", [{"pt": pt}, float(s)], None)

    def GetCiphertextSlots(self, ct):
        return self._log("GetCiphertextSlots", [{"ct": ct}], self.cts[ct]["slots"])

    def GetPlaintextSlots(self, pt):
        return self._log("GetPlaintextSlots", [{"pt": pt}], self.pts[pt]["slots"])

    def SetCiphertextSlots(self, ct, s):
        self.cts[ct]["slots"] = int(s)
        self._log("SetCiphertextSlots", [{"ct": ct}, int(s)], None)

    def GetCiphertextDegree(self, ct):
        return self._log("GetCiphertextDegree", [{"ct": ct}], 2)

    def GetLiveCiphertexts(self):
        return self._log("GetLiveCiphertexts", [], len(self.cts))

    def GetLivePlaintexts(self):
        return self._log("GetLivePlaintexts", [], len(self.pts))


def _import_reference(ref_root):
    sys.path.insert(0, ref_root)
    for name in ["matplotlib", "matplotlib.pyplot", "h5py", "opt_einsum", "desilofhe"]:
        sys.modules.setdefault(name, types.ModuleType(name))
    import orion  # noqa: F401
    return orion


def record(net_kind: str, ref_root: str, config=None):
    import torch

    orion = _import_reference(ref_root)
    import orion.nn as on

    sys.path.insert(0, ROOT)
    from helrm_b200 import orion_adapter
    from oracle import oracle as om

    config = config or CONFIG
    main, _aux = om.scheme_primes(config["ckks_params"]["LogQ"], config["ckks_params"]["LogP"],
                                  config["ckks_params"]["LogN"])
    holder = {}

    def factory():
        holder["rec"] = Recorder(main)
        return holder["rec"]

    orion_adapter.install(factory=factory)
    torch.manual_seed(5)
    if net_kind == "linear":
        class Net(on.Module):
            def __init__(self):
                super().__init__()
                self.fc = on.Linear(32, 8)

            def forward(self, x):
                return self.fc(x)
        net = Net()
        inp = torch.randn(1, 32)
    elif net_kind == "mlp_boot":
        class Net(on.Module):
            def __init__(self):
                super().__init__()
                self.fc1 = on.Linear(16, 8)
                self.act1 = on.ReLU()
                self.fc2 = on.Linear(8, 8)
                self.act2 = on.ReLU()
                self.fc3 = on.Linear(8, 4)

            def forward(self, x):
                return self.fc3(self.act2(self.fc2(self.act1(self.fc1(x)))))
        net = Net()
        for seed in range(200):
            inp = torch.randn(1, 16, generator=torch.Generator().manual_seed(seed))
            h1 = net.fc1(inp).detach()
            h2 = net.fc2(torch.relu(h1)).detach()
            if (float(h1.abs().min()) >= 0.05 * float(h1.abs().max()) and
                    float(h2.abs().min()) >= 0.05 * float(h2.abs().max())):
                break
    elif net_kind == "mlp_relu":
        class Net(on.Module):
            def __init__(self):
                super().__init__()
                self.fc1 = on.Linear(16, 8)
                self.act = on.ReLU()
                self.fc2 = on.Linear(8, 4)

            def forward(self, x):
                return self.fc2(self.act(self.fc1(x)))
        net = Net()
        # an input whose hidden pre-activations stay clear of the sign's gap
        # (|h| >= 0.05 max|h|), where the composite step is within 1e-4
        for seed in range(100):
            inp = torch.randn(1, 16, generator=torch.Generator().manual_seed(seed))
            h = net.fc1(inp).detach().abs()
            if float(h.min()) >= 0.05 * float(h.max()):
                break
    elif net_kind == "helrm":
        # the reference's own encrypted model (examples/criteo/dlrm.py:181-229),
        # its module-level widths narrowed to fit LogN 13: two tables (50 and
        # 300 categories, radix-4 digits above 20), embedding dim 4, bottom
        # MLP 13-16-4, top MLP 12-8-1
        sys.path.insert(0, os.path.join(ref_root, "examples", "criteo"))
        import dlrm
        dlrm.sparse_fields, dlrm.embedding_features = 2, 4
        dlrm.bottom_widths = [dlrm.dense_features, 16, 4]
        dlrm.top_widths = [4 * 3, 8, 1]
        net = dlrm.HELRM([50, 300], compress_threshold=20, base=4)
        # dense features log1p(lognormal) and indices whose ReLU inputs stay
        # clear of the composite sign's gap (|h| >= 0.05 max|h| per layer)
        for seed in range(2000):
            g = torch.Generator().manual_seed(seed)
            dense = torch.log1p(torch.exp(torch.randn(1, 13, generator=g)))
            sparse = torch.tensor([int(torch.randint(0, 50, (1,), generator=g)),
                                   int(torch.randint(0, 300, (1,), generator=g))])
            d_in, s_in = net.fhe_input(dense, sparse)
            hs = []
            x = d_in
            for layer in net.bottom:
                x = layer(x)
                if isinstance(layer, on.Linear):
                    hs.append(x.detach())
            top_in = net.bottom_to_top(x) + net.sparse_to_top(net.sparse(s_in))
            x = top_in
            for layer in net.top:
                x = layer(x)
                if isinstance(layer, on.Linear):
                    hs.append(x.detach())
            if all(float(h.abs().min()) >= 0.05 * float(h.abs().max()) for h in hs[:-1]):
                break
        inp = [d_in, s_in]
    else:
        class Net(on.Module):
            def __init__(self):
                super().__init__()
                self.emb = on.Embedding(64, 16)

            def forward(self, x):
                return self.emb(x)
        net = Net()
        inp = torch.zeros(1, 64)
        inp[0, 37] = 1.0  # one-hot selector, the HE-LRM lookup's input
    scheme = orion.init_scheme(config)
    rec = holder["rec"]
    net.eval()
    inputs = inp if isinstance(inp, list) else [inp]
    out_clear = net(*inputs).detach().numpy().ravel()
    orion.fit(net, inp)
    level = orion.compile(net)
    ctxts = [orion.encrypt(orion.encode(x, level)) for x in inputs]
    net.he()
    out_ct = net(*ctxts)
    mark = len(rec.calls)
    out_pt = out_ct.decrypt()
    out_pt.decode()
    decodes = [i for i, c in enumerate(rec.calls) if c["m"] == "Decode" and i >= mark]
    del scheme
    return rec, out_clear, decodes, level


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HELRM_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_orion_trace.py <reference checkout>")
    traces, arrays = {}, {}
    configs = {"mlp_relu": CONFIG_DEEP, "mlp_boot": CONFIG_BOOT, "helrm": CONFIG_BOOT}
    for kind in ("linear", "embedding", "mlp_relu", "mlp_boot", "helrm"):
        rec, out_clear, decodes, level = record(kind, ref, configs.get(kind, CONFIG))
        traces[kind] = {"params": rec.params, "calls": rec.calls, "output_decode_calls": decodes,
                        "input_level": int(level), "cleartext_output": [float(v) for v in out_clear]}
        for k, v in rec.arrays.items():
            arrays[f"{kind}/{k}"] = v
        print(kind, len(rec.calls), "calls,", sorted({c["m"] for c in rec.calls}))
    with open(os.path.join(HERE, "orion_trace.json"), "w") as f:
        json.dump(traces, f)
    np.savez_compressed(os.path.join(HERE, "orion_trace.npz"), **arrays)
    print("trace written to", HERE)


if __name__ == "__main__":
    main()
