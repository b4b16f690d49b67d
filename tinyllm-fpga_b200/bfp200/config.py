"""BfpConfig: the run configuration, with the reference's field names.

The reference reads MODEL, D, H_Q, H_KV, HD, FFN, NL, MAX_CTX, PROMPT, N_GEN,
PREFIX, OUT from the environment (rtl/vc707/host/gen_smollm_blockfp_full.py:53-64)
and NPROMPT_MAX from gen_smollm_blockfp_cfg.py:44.  ``BfpConfig.from_env()``
reads the same variables with the same defaults; ``to_c()`` gives the C
struct of include/bfp200.h.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, fields

from . import _lib


# variables the reference reads from the environment
ENV_FIELDS = ("D", "H_Q", "H_KV", "HD", "FFN", "NL", "MAX_CTX", "N_GEN", "PREFIX", "OUT", "NPROMPT_MAX")


@dataclass
class BfpConfig:
    D: int = 576
    H_Q: int = 9
    H_KV: int = 3
    HD: int = 64
    FFN: int = 1536
    NL: int = 30
    VOCAB: int = 49152
    MAX_CTX: int = 64          # the reference's default (:60)
    NPROMPT_MAX: int = 48      # gen_smollm_blockfp_cfg.py:44
    N_GEN: int = 15            # :62
    PREFIX: str = "lbfp_full_"
    OUT: str = "generated"
    max_seqs: int = 1
    rope_base: float = 10000.0  # rope_fp's default base (:250); SmolLM2's rope_theta is 1e5
    eps: float = 1e-5

    @classmethod
    def from_env(cls, environ=None, **overrides):
        """Reads the reference's environment variables (same names, same defaults)."""
        env = os.environ if environ is None else environ
        kw = {}
        for f in fields(cls):
            if f.name in ENV_FIELDS and f.name in env:
                kw[f.name] = int(env[f.name]) if f.type == "int" else env[f.name]
        kw.update(overrides)
        return cls(**kw)

    @property
    def NT_D(self):
        return self.D // 16

    @property
    def KVD(self):
        return self.H_KV * self.HD

    def to_c(self) -> _lib.Cfg:
        c = _lib.Cfg()
        for name in ("D", "H_Q", "H_KV", "HD", "FFN", "NL", "VOCAB", "MAX_CTX", "NPROMPT_MAX", "max_seqs"):
            setattr(c, name, int(getattr(self, name)))
        c.rope_base = float(self.rope_base)
        c.eps = float(self.eps)
        return c


SMOLLM2_135M = BfpConfig()
