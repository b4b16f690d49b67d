"""Seeded input generators shared by make_golden.py and the tests.

Everything here is deterministic (numpy default_rng with fixed seeds) so the
tests regenerate exactly the inputs the committed golden outputs were made
from.  Shapes and value distributions follow the benchmark configurations:

* weight-shape sweep (cfg4): shapes D_out x D_in in SWEEP_SHAPES, mantissas
  uniform int16, tile exponents uniform in [-20, 4], activations are the
  simulator's BFP form of N(0, 1), batch in SWEEP_BATCHES, seed 4;
* leaf ops / attention (cfg5): activations from N(0, 1) with 1% of the
  elements scaled x30, seed 5.
"""
from __future__ import annotations

import numpy as np

TILE = 16
SWEEP_SHAPES = [(576, 576), (192, 576), (1536, 576), (576, 1536), (49152, 576)]
SWEEP_BATCHES = [1, 8, 64, 256, 1024]
LAYER_KV_POS = [0, 1, 5, 63, 303, 2047]


def _q(v):
    """BFP quantization (restated here so the generators are self-contained;
    identical arithmetic to gen_smollm_blockfp_full.py:90-97)."""
    flat = np.asarray(v, dtype=np.float64).reshape(-1, TILE)
    max_abs = np.maximum(np.abs(flat).max(axis=1), 1e-300)
    e = (np.floor(np.log2(max_abs)).astype(np.int32) + 1).clip(-127, 127)
    m = np.clip(np.round(flat / np.power(2.0, e.astype(np.float64))[:, None] * 32768.0).astype(np.int64),
                -32768, 32767)
    return m.astype(np.int16), e.astype(np.int8)


def _fpq(v):
    m, e = _q(v)
    return ((m.astype(np.float64) / 32768.0) * np.power(2.0, e.astype(np.float64))[:, None]).reshape(-1)


def outlier_normal(rng, n):
    """N(0,1) with 1% of elements multiplied by 30 (cfg5 activations)."""
    x = rng.standard_normal(n)
    idx = rng.random(n) < 0.01
    x[idx] *= 30.0
    return x


def quant_cases():
    """Edge-case tiles for tile_quantize: returns a flat float64 vector."""
    rng = np.random.default_rng(11)
    tiles = []
    tiles += list(rng.standard_normal((64, TILE)))
    tiles += list(rng.standard_normal((64, TILE)) * np.exp2(rng.integers(-140, 130, size=(64, 1))))
    tiles += list(outlier_normal(rng, 64 * TILE).reshape(64, TILE))
    # exact powers of two and their neighbours (floor(log2) boundary)
    for j in list(range(-130, 131, 3)) + [-3, -2, -1, 0, 1, 2, 3, 4, 5, 8, 9, 17, 33, 65]:
        p = np.ldexp(1.0, j)
        below = [p]
        y = p
        for _ in range(TILE - 1):
            y = np.nextafter(y, 0.0)
            below.append(y)
        t = np.array(below)
        tiles.append(t)
        tiles.append(-t[::-1])
        for n in (1, 2, 5, 11, 22, 44, 45, 88, 89):
            y = p
            for _ in range(n):
                y = np.nextafter(y, 0.0)
            t2 = rng.standard_normal(TILE) * p * 0.1
            t2[rng.integers(TILE)] = y
            tiles.append(t2)
    # -32768 after rounding, +32768 clipped, ties to even, zeros, tiny, huge
    for e in (-5, 0, 3, 20):
        p = np.ldexp(1.0, e)
        t = rng.standard_normal(TILE) * p * 0.3
        t[0] = -p * (1 - 2.0 ** -17)        # rounds to -32768
        tiles.append(t)
        t = rng.standard_normal(TILE) * p * 0.3
        t[1] = p * (1 - 2.0 ** -17)         # rounds to 32768 -> clip 32767
        tiles.append(t)
        t = (rng.integers(-32768, 32767, size=TILE) + 0.5) * p / 32768.0 * 0.5
        t[2] = p * 0.99
        tiles.append(t)                     # exact .5 ties
    tiles.append(np.zeros(TILE))
    tiles.append(-np.zeros(TILE))
    tiles.append(np.full(TILE, 1e-310))     # subnormal, below the 1e-300 floor
    tiles.append(rng.standard_normal(TILE) * 1e-45)
    tiles.append(rng.standard_normal(TILE) * 2.0 ** 128)
    tiles.append(np.array([2.0 ** 127] + [1.0] * (TILE - 1)))
    return np.concatenate([np.asarray(t, dtype=np.float64) for t in tiles])


def sweep_weights(D_out, D_in):
    rng = np.random.default_rng([4, D_out, D_in])
    W_m = rng.integers(-32768, 32768, size=(D_out, D_in // TILE, TILE)).astype(np.int16)
    W_e = rng.integers(-20, 5, size=(D_out, D_in // TILE)).astype(np.int8)
    return W_m, W_e


def sweep_x(D_in, B, D_out):
    rng = np.random.default_rng([4, D_out, D_in, B, 1])
    m, e = _q(rng.standard_normal(B * D_in))
    return m.reshape(B, D_in // TILE, TILE), e.reshape(B, D_in // TILE)


def ref_batch_limit(D_out):
    """Largest batch the (slow) reference matvec is run on per shape; larger
    batches are pinned through the oracle."""
    return 8 if D_out > 4096 else 64


def matvec_edge_cases():
    rng = np.random.default_rng(12)
    cases = {}
    # 1. shift > 47 masks tiles; shift == 47 keeps them
    D_in, D_out = 576, 32
    NT = D_in // TILE
    W_m = rng.integers(-32768, 32768, size=(D_out, NT, TILE)).astype(np.int16)
    W_e = np.zeros((D_out, NT), dtype=np.int8)
    W_e[:, 0] = 60
    W_e[:, 1] = 13      # shift 47 against tile 0 (x_e equal)
    W_e[:, 2] = 12      # shift 48 -> masked
    W_e[:16, 3] = -67   # very large shift
    x_m, x_e = _q(rng.standard_normal(D_in))
    x_e = np.zeros_like(x_e)
    cases["shift_mask"] = (x_m.reshape(NT, TILE), x_e, W_m, W_e)
    # 2. saturation: 8200 tiles of (-32768)^2 * 16 = 2^34 each -> acc > 2^47
    NT2 = 8200
    W_m2 = np.full((16, NT2, TILE), -32768, dtype=np.int16)
    W_m2[8:] = 32767
    W_e2 = np.zeros((16, NT2), dtype=np.int8)
    x_m2 = np.full((NT2, TILE), -32768, dtype=np.int16)
    x_e2 = np.zeros(NT2, dtype=np.int8)
    cases["saturate"] = (x_m2, x_e2, W_m2, W_e2)
    # 3. mixed: zero x tiles, -32768 mantissas, extreme exponents
    W_m3 = rng.integers(-32768, 32768, size=(64, 36, TILE)).astype(np.int16)
    W_m3[:, :, 0] = -32768
    W_e3 = rng.integers(-127, 128, size=(64, 36)).astype(np.int8)
    x_m3, x_e3 = _q(outlier_normal(rng, 576))
    x_m3 = x_m3.copy()
    x_m3[5] = 0
    x_e3 = x_e3.copy()
    x_e3[5] = -127
    cases["mixed"] = (x_m3, x_e3, W_m3, W_e3)
    # 4. all-zero activation
    cases["zero_x"] = (np.zeros((36, TILE), np.int16), np.full(36, -127, np.int8),
                       W_m3, W_e3)
    return cases


def layer_case(kv_pos, max_ctx):
    """Hidden state + KV cache (positions < kv_pos filled) for a layer test."""
    rng = np.random.default_rng([5, kv_pos])
    h = _fpq(outlier_normal(rng, 576))
    K = np.zeros((max_ctx, 3, 64))
    V = np.zeros((max_ctx, 3, 64))
    if kv_pos:
        K[:kv_pos] = _fpq(rng.standard_normal(kv_pos * 192)).reshape(kv_pos, 3, 64)
        V[:kv_pos] = _fpq(rng.standard_normal(kv_pos * 192)).reshape(kv_pos, 3, 64)
    return h, K, V
