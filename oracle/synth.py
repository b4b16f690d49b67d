"""Seeded synthetic SmolLM2-135M model for the oracle (TEST ONLY).

The model is random-init (no checkpoint is available offline):

* every matrix W ~ N(0, 0.02), every gamma (g1, g2, norm_w) = 1 + N(0, 0.05);
* one ``np.random.default_rng(seed)`` stream, drawn in this order: for each
  layer Wq, Wk, Wv, Wo, Wg, Wu, Wd, g1, g2; then the tied embedding; then
  norm_w.  Matrices are drawn in the HuggingFace (out, in) orientation that
  gen_smollm_blockfp_full.py:312-319 reads;
* each float tensor is replaced by decode(quantize(.)) applied twice, which
  makes it a fixed point (a tile that clips to -32768 converges on the second
  pass).  The packed image then carries exactly the simulator's float values,
  including the un-quantized embedding the head reads (:439).

The product has its own generator (bfp200.synth) that must produce the same
bytes; tests compare the two.
"""
from __future__ import annotations

import numpy as np

from . import bfp_oracle as O

MATS = ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd")


def mat_shapes(cfg: O.Cfg):
    kvd = cfg.H_KV * cfg.HD
    return {"Wq": (cfg.D, cfg.D), "Wk": (kvd, cfg.D), "Wv": (kvd, cfg.D), "Wo": (cfg.D, cfg.D),
            "Wg": (cfg.FFN, cfg.D), "Wu": (cfg.FFN, cfg.D), "Wd": (cfg.D, cfg.FFN)}


def snap(x):
    """decode(quantize(.)) twice -> a BFP fixed point (flat 16-tiling)."""
    shape = x.shape
    y = O.fp_quantize_vec(O.fp_quantize_vec(x.reshape(-1)))
    return y.reshape(shape)


class Model:
    """Float fixed-point weights plus their (m, e) form, as the simulator holds them."""

    def __init__(self, cfg: O.Cfg, layers_float, embed, norm_w):
        self.cfg = cfg
        self.layers_float = layers_float
        self.embed = embed
        self.norm_w = norm_w
        self.norm_w_q = O.fp_quantize_vec(norm_w)           # :413
        self.layers = []
        for lf in layers_float:
            lw = {}
            for nm in MATS:
                lw[nm] = O.quantize_W(lf[nm])                # :320
            lw["g1"] = O.fp_quantize_vec(lf["g1"])            # :322
            lw["g2"] = O.fp_quantize_vec(lf["g2"])            # :323
            self.layers.append(lw)

    def embed_q(self, tid):
        """:411-412 (per row, on demand)."""
        return O.fp_quantize_vec(self.embed[tid])

    def cache_float_weights(self):
        """Pre-expand mantissas for the BLAS tile-sum path (memory for speed)."""
        for lw in self.layers:
            for nm in MATS:
                m, _ = lw[nm]
                lw["Wf_" + nm] = np.ascontiguousarray(m.astype(np.float64).transpose(1, 0, 2))


def make_model(seed=0, cfg: O.Cfg = O.Cfg(), snap_weights=True) -> Model:
    rng = np.random.default_rng(seed)
    shapes = mat_shapes(cfg)
    layers = []
    for _ in range(cfg.NL):
        lf = {}
        for nm in MATS:
            lf[nm] = 0.02 * rng.standard_normal(shapes[nm])
        lf["g1"] = 1.0 + 0.05 * rng.standard_normal(cfg.D)
        lf["g2"] = 1.0 + 0.05 * rng.standard_normal(cfg.D)
        layers.append(lf)
    embed = 0.02 * rng.standard_normal((cfg.VOCAB, cfg.D))
    norm_w = 1.0 + 0.05 * rng.standard_normal(cfg.D)
    if snap_weights:
        for lf in layers:
            for k in lf:
                lf[k] = snap(lf[k])
        embed = snap(embed)
        norm_w = snap(norm_w)
    return Model(cfg, layers, embed, norm_w)


def config_prompts(cfg_id: int, vocab=49152):
    """Seeded prompts of the benchmark configurations.

    cfg1: 8 ids ~ U[0, vocab) from default_rng(1), n_gen 16.
    cfg2: 48 ids ~ U[0, vocab) from default_rng(2), n_gen 256.
    cfg3: 256 sequences, lengths ~ U{8..48}, ids ~ U[0, vocab), default_rng(3), n_gen 128.
    """
    if cfg_id == 1:
        return [np.random.default_rng(1).integers(0, vocab, size=8).tolist()], 16
    if cfg_id == 2:
        return [np.random.default_rng(2).integers(0, vocab, size=48).tolist()], 256
    if cfg_id == 3:
        rng = np.random.default_rng(3)
        lens = rng.integers(8, 49, size=256)
        return [rng.integers(0, vocab, size=int(n)).tolist() for n in lens], 128
    raise ValueError(cfg_id)
