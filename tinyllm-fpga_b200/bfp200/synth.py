"""Seeded synthetic SmolLM2-135M weights and the benchmark prompts.

No checkpoint is available offline, so the benchmarks use a random-init model
of the SmolLM2-135M architecture:

* matrices W ~ N(0, 0.02), gammas g1, g2, norm_w = 1 + N(0, 0.05), from one
  ``np.random.default_rng(seed)`` stream drawn per layer in the order Wq, Wk,
  Wv, Wo, Wg, Wu, Wd, g1, g2, then the tied embedding, then norm_w (matrices
  in the HuggingFace (out, in) orientation gen_smollm_blockfp_full.py:312-319
  reads);
* every tensor replaced by decode(quantize(.)) applied twice (a BFP fixed
  point), so the packed image carries exactly the float values the
  simulator's head reads (:439);
* quantization runs on the GPU (bfp200.ops); the image is then packed
  byte-for-byte like gen_smollm_blockfp_ddr.py.
"""
from __future__ import annotations

import numpy as np

from . import ops
from .config import BfpConfig
from .pack import build_image

MATS = ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd")


def mat_shapes(cfg: BfpConfig):
    kvd = cfg.H_KV * cfg.HD
    return {"Wq": (cfg.D, cfg.D), "Wk": (kvd, cfg.D), "Wv": (kvd, cfg.D), "Wo": (cfg.D, cfg.D),
            "Wg": (cfg.FFN, cfg.D), "Wu": (cfg.FFN, cfg.D), "Wd": (cfg.D, cfg.FFN)}


def _fixed_point_me(x):
    """(m, e) of the BFP fixed point of x: quantize(decode(quantize(decode(quantize(x)))))."""
    flat = x.reshape(-1)
    y = ops.fp_quantize_vec(ops.fp_quantize_vec(flat))
    return ops.tile_quantize(y)


def synthetic_model(cfg: BfpConfig, seed: int = 0):
    """Returns (layers [{name: (m, e)}], g1 [(m, e)], g2, embed (m, e), norm_w (m, e))."""
    rng = np.random.default_rng(seed)
    shapes = mat_shapes(cfg)
    layers, g1, g2 = [], [], []
    for _ in range(cfg.NL):
        lw = {}
        for nm in MATS:
            w = 0.02 * rng.standard_normal(shapes[nm])
            m, e = _fixed_point_me(w)
            dout, din = shapes[nm]
            lw[nm] = (m.reshape(dout, din // 16, 16), e.reshape(dout, din // 16))
        for lst in (g1, g2):
            g = 1.0 + 0.05 * rng.standard_normal(cfg.D)
            m, e = _fixed_point_me(g)
            lst.append((m.reshape(-1), e))
        layers.append(lw)
    emb = 0.02 * rng.standard_normal((cfg.VOCAB, cfg.D))
    m, e = _fixed_point_me(emb)
    embed = (m.reshape(cfg.VOCAB, cfg.D // 16, 16), e.reshape(cfg.VOCAB, cfg.D // 16))
    del emb
    nw = 1.0 + 0.05 * rng.standard_normal(cfg.D)
    m, e = _fixed_point_me(nw)
    return layers, g1, g2, embed, (m.reshape(-1), e)


def synthetic_image(cfg: BfpConfig, seed: int = 0) -> bytes:
    """<PREFIX>DDR3.bin bytes of the seeded synthetic model."""
    layers, g1, g2, embed, nw = synthetic_model(cfg, seed)
    return build_image(cfg, layers, g1, g2, embed, nw)


def config_prompts(cfg_id: int, vocab: int = 49152):
    """Seeded prompts of the benchmark configurations (ids, n_gen):

    cfg1: 8 ids ~ U[0, vocab) from default_rng(1), 16 generated tokens;
    cfg2: 48 ids from default_rng(2), 256 generated tokens;
    cfg3: 256 sequences of U{8..48} ids from default_rng(3), 128 generated tokens.
    """
    if cfg_id == 1:
        return [np.random.default_rng(1).integers(0, vocab, size=8).tolist()], 16
    if cfg_id == 2:
        return [np.random.default_rng(2).integers(0, vocab, size=48).tolist()], 256
    if cfg_id == 3:
        rng = np.random.default_rng(3)
        lens = rng.integers(8, 49, size=256)
        return [rng.integers(0, vocab, size=int(n)).tolist() for n in lens], 128
    raise ValueError(f"unknown benchmark config {cfg_id}")
