"""Helpers for the GPU parity tests: one library scheme plus the oracle
bound to the same primes, keys and encryption seeds."""
import numpy as np

from helrm_b200 import B200Library, CKKSConfig


class Pair:
    """A B200 scheme and the CPU oracle with identical parameters.

    The library derives every key and encryption from `seed` with the
    counter-based sampler; the oracle restates that sampler, so keys and
    ciphertexts can be regenerated on the CPU and compared bit for bit."""

    def __init__(self, cfg: CKKSConfig, dnum: int, seed: int, oracle_mod):
        self.cfg = cfg
        self.seed = seed
        self.lib = B200Library(dnum=dnum, seed=seed, device=0)
        self.lib.setup_bindings(cfg)
        self.lib.GenerateSecretKey()
        self.lib.GenerateRelinearizationKey()
        self.info = self.lib.scheme_info()
        self.o = oracle_mod.Oracle(cfg.logn, self.lib.GetAllModuliChain(), self.lib.GetAuxModuliChain(), dnum)
        assert self.o.alpha == self.info["alpha"] and self.o.dnum == self.info["dnum"]
        self.om = oracle_mod
        self.enc_count = 0
        self.sk = self.o.secret_ntt(self.o.sample_secret(seed, cfg.h))
        self.N = self.info["N"]
        self.slots = self.info["slots"]
        self.scale = float(1 << cfg.logscale)

    def close(self):
        self.lib.DeleteScheme()

    def encrypt(self, values, level=None, scale=None):
        level = self.info["max_level"] if level is None else level
        pt = self.lib.Encode(list(values), level, scale or self.scale)
        ct = self.lib.Encrypt(pt)
        self.enc_count += 1
        self.lib.DeletePlaintext(pt)
        return ct

    def next_ct_seed(self):
        """seed the library's next Encrypt call will use"""
        return int(self.om.lib().ora_rand64(self.seed, 1000, self.enc_count))

    def decrypt(self, ct):
        pt = self.lib.Decrypt(ct)
        vals = np.array(self.lib.Decode(pt))
        self.lib.DeletePlaintext(pt)
        return vals

    def ct_data(self, ct):
        return self.lib.GetCiphertextData(ct)

    def key(self, galois):
        return self.lib.GetKeyData(galois)
