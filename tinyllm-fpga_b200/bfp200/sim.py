"""Drop-in module for the reference's bit-exact BFP simulator
(jrrk2/tinyllm-fpga rtl/vc707/host/gen_smollm_blockfp_full.py): same names,
same signatures, same numpy arrays in and out -- computed on the GPU.

Module-level configuration is read from the same environment variables as
the reference (:53-64).  ``fwd_layer`` mutates ``kv`` in place like the
reference (:270-272).  There is no CPU path: without libbfp200 and a B200
every call raises ``bfp200.BfpError``.
"""
from __future__ import annotations

import numpy as np

from . import ops
from .config import BfpConfig
from .engine import Decoder
from .pack import build_image

_cfg = BfpConfig.from_env()
D, H_Q, H_KV, HD, FFN, NL, MAX_CTX = _cfg.D, _cfg.H_Q, _cfg.H_KV, _cfg.HD, _cfg.FFN, _cfg.NL, _cfg.MAX_CTX
N_GEN, PREFIX, OUT = _cfg.N_GEN, _cfg.PREFIX, _cfg.OUT
TILE = 16
LANES = 16
BFP_MANT_W = 16
BFP_EXP_W = 8
ALIGN_MAX = 47
NT_D = D // TILE
NT_FFN = FFN // TILE
NT_KV = (H_KV * HD) // TILE
H2 = HD // 2

tile_quantize = ops.tile_quantize          # :90-97
tile_decode = ops.tile_decode              # :100-102
fp_quantize_vec = ops.fp_quantize_vec      # :105-107
matvec_hw_golden = ops.matvec_hw_golden    # :217-233
rmsnorm_fp = ops.rmsnorm_fp                # :236-238
silu_fp = ops.silu_fp                      # :241-242
softmax_fp = ops.softmax_fp                # :245-247


def quantize_W(W):
    """:110-119."""
    from .pack import quantize_W as q
    return q(W)


def rope_fp(x, pos, base=10000.0):
    """:250-258."""
    return ops.rope_fp(x, pos, base)


# the single-layer decoder of the most recently used layer-weights dict
_keep = {}


class _LayerDecoder:
    """A 1-layer image built from a reference-style ``lw`` dict."""

    def __init__(self, lw, max_ctx):
        self.cfg = BfpConfig(D=D, H_Q=H_Q, H_KV=H_KV, HD=HD, FFN=FFN, NL=1, VOCAB=16, MAX_CTX=max_ctx,
                             max_seqs=1)
        layer = {k: (np.asarray(lw[k][0], np.int16), np.asarray(lw[k][1], np.int8))
                 for k in ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd")}
        g1 = ops.tile_quantize(np.asarray(lw["g1"], np.float64))
        g2 = ops.tile_quantize(np.asarray(lw["g2"], np.float64))
        zero_emb = (np.zeros((16, NT_D, TILE), np.int16), np.full((16, NT_D), -127, np.int8))
        ones = ops.tile_quantize(np.ones(D))
        img = build_image(self.cfg, [layer], [(g1[0].ravel(), g1[1])], [(g2[0].ravel(), g2[1])], zero_emb,
                          (ones[0].ravel(), ones[1]))
        self.dec = Decoder(self.cfg)
        self.dec.load_image(img)


def fwd_layer(h, lw, pos, kv, kv_pos):
    """gen_smollm_blockfp_full.py:261-293 on the GPU.  ``lw`` holds 'Wq'..'Wd'
    as (m, e) and 'g1', 'g2' as float vectors on the BFP grid; ``kv`` holds
    float64 'k' and 'v' caches of shape (max_ctx, H_KV, HD), updated at
    kv_pos."""
    max_ctx = kv["k"].shape[0]
    key = (id(lw), max_ctx)
    ld = _keep.get(key)
    if ld is None:
        ld = _LayerDecoder(lw, max_ctx)
        _keep.clear()            # one cached layer at a time
        _keep[key] = ld
    kc = np.ascontiguousarray(kv["k"], np.float64)[None].copy()
    vc = np.ascontiguousarray(kv["v"], np.float64)[None].copy()
    out = ld.dec.fwd_layer(0, h, pos, kc, vc, kv_pos=kv_pos)
    kv["k"][kv_pos] = kc[0, kv_pos]
    kv["v"][kv_pos] = vc[0, kv_pos]
    return out


def generate(image, prompt_ids, n_gen=N_GEN, feed_mode="sim", cfg: BfpConfig | None = None, device=0):
    """The golden driver loop (:425-449) over a packed image: returns
    prompt + n_gen ids (feed_mode='sim') like <PREFIX>GOLDEN_TOKENS.txt."""
    cfg = cfg or BfpConfig(MAX_CTX=max(MAX_CTX, len(prompt_ids) + n_gen))
    with Decoder(cfg, device) as dec:
        dec.load_image(image)
        return dec.generate([list(prompt_ids)], n_gen, feed_mode)[0]
