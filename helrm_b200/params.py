"""Stand-alone CKKS parameter object with the getters Orion's
``NewParameters`` exposes (orion/backend/python/parameters.py:237-309), so
``B200Library.setup_bindings`` takes either Orion's object or this one."""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class CKKSConfig:
    logn: int
    logq: list = field(default_factory=list)
    logp: list = field(default_factory=list)
    logscale: int = 40
    h: int = 192
    ringtype: str = "standard"
    boot: bool = False   # reserve the bootstrapping primes above the chain

    @classmethod
    def from_dict(cls, cfg: dict) -> "CKKSConfig":
        """Accepts Orion's YAML layout ({"ckks_params": {...}}) or a flat dict."""
        p = cfg.get("ckks_params", cfg)
        norm = {k.lower(): v for k, v in p.items()}
        return cls(logn=int(norm["logn"]), logq=list(norm["logq"]), logp=list(norm["logp"]),
                   logscale=int(norm.get("logscale", 40)), h=int(norm.get("h", 192)),
                   ringtype=str(norm.get("ringtype", "standard")))

    def get_logn(self):
        return self.logn

    def get_logq(self):
        return self.logq

    def get_logp(self):
        return self.logp

    def get_logscale(self):
        return self.logscale

    def get_default_scale(self):
        return 1 << self.logscale

    def get_hamming_weight(self):
        return self.h

    def get_ringtype(self):
        return self.ringtype

    def get_max_level(self):
        return len(self.logq) - 1

    def get_slots(self):
        return 1 << (self.logn - 1)

    def get_ring_degree(self):
        return 1 << self.logn


# Parameter sets of the BASELINE configs and of the reference's oracle tests.
TEST_CONFIG = CKKSConfig(logn=13, logq=[29, 26, 26, 26], logp=[29], logscale=26, h=8192)  # tests/oracle/conftest.py:40-55
CFG1 = CKKSConfig(logn=13, logq=[40] * 5, logp=[60], logscale=40, h=192)
CFG2 = CKKSConfig(logn=16, logq=[36] * 24, logp=[60] * 4, logscale=36, h=192)
CFG2_DNUM = 4
# config 4 (the bootstrapped HE-LRM forward): config 2's 36-bit chain under
# a 50-bit q0 (message ratio 2^14 for bootstrapping: EvalMod without the
# arcsine, 11 reserved 60-bit primes above the chain), six 60-bit special
# primes; dnum 6 keeps every digit (at most six primes of up to 60 bits) at
# the special modulus' size
CFG4 = CKKSConfig(logn=16, logq=[50] + [36] * 23, logp=[60] * 6, logscale=36, h=192, boot=True)
CFG4_DNUM = 6
