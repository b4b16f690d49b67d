"""Packer surface: BFP weight quantization and the byte-exact DDR3 image.

Mirrors rtl/vc707/host/gen_smollm_blockfp_ddr.py (jrrk2/tinyllm-fpga):
``quantize_W`` (:65-74) runs on the GPU through the C ABI; the two layout
functions (:88-119) are pure byte shuffles done with numpy reshapes; the
image assembly follows main() (:155-241).
"""
from __future__ import annotations

import numpy as np

from . import ops
from .config import BfpConfig
from .image import ALIGN, align4k, region_map

TILE = 16
LANES = 16


def quantize_W(W):
    """quantize_W (:65-74): per-row tile quantization on the GPU.
    W (D_out, D_in) -> m (D_out, D_in/16, 16) int16, e (D_out, D_in/16) int8."""
    W = np.asarray(W, dtype=np.float64)
    D_out, D_in = W.shape
    assert D_in % TILE == 0
    m, e = ops.tile_quantize(W.reshape(-1))
    return m.reshape(D_out, D_in // TILE, TILE), e.reshape(D_out, D_in // TILE)


def pack_layer_mantissas(m, e=None):
    """pack_layer_mantissas (:88-104): entry (chunk, col) = 16 LE int16
    mantissas of rows chunk*16 .. chunk*16+15 at column col."""
    m = np.asarray(m, dtype=np.int16)
    D_out, NT, _ = m.shape
    D_in = NT * TILE
    a = m.reshape(D_out // LANES, LANES, D_in).transpose(0, 2, 1)   # (chunk, col, lane)
    return np.ascontiguousarray(a).astype("<i2").tobytes()


def pack_layer_exponents(e):
    """pack_layer_exponents (:107-119): entry (chunk, tile) = 16 exponents."""
    e = np.asarray(e, dtype=np.int8)
    D_out, NT = e.shape
    a = e.reshape(D_out // LANES, LANES, NT).transpose(0, 2, 1)     # (chunk, tile, lane)
    return np.ascontiguousarray(a).tobytes()


def build_image(cfg: BfpConfig, layers, g1, g2, embed, norm_w) -> bytes:
    """Assembles <PREFIX>DDR3.bin (:155-241).

    layers: list of NL dicts {'Wq'..'Wd': (m, e)}; g1, g2: lists of (m, e);
    embed: (m (VOCAB, NT, 16), e (VOCAB, NT)); norm_w: (m, e)."""
    key = {"WQ": "Wq", "WK": "Wk", "WV": "Wv", "WO": "Wo", "WG": "Wg", "WU": "Wu", "WDN": "Wd"}
    rmap = {name: (off, size) for name, off, size in region_map(cfg)}
    img = bytearray(rmap["END"][0])

    def put(name, data):
        off, size = rmap[name]
        assert len(data) == size, (name, len(data), size)
        img[off:off + size] = data

    for tag, k in key.items():
        put(f"{tag}_m", b"".join(pack_layer_mantissas(layers[li][k][0]) for li in range(cfg.NL)))
        put(f"{tag}_e", b"".join(pack_layer_exponents(layers[li][k][1]) for li in range(cfg.NL)))
    put("G1_m", b"".join(np.asarray(m, "<i2").tobytes() for m, _ in g1))
    put("G1_e", b"".join(np.asarray(e, np.int8).tobytes() for _, e in g1))
    put("G2_m", b"".join(np.asarray(m, "<i2").tobytes() for m, _ in g2))
    put("G2_e", b"".join(np.asarray(e, np.int8).tobytes() for _, e in g2))
    em, ee = embed
    put("EMBED_m", pack_layer_mantissas(em))
    put("EMBED_e", pack_layer_exponents(ee))
    put("EMBED_LU_m", np.asarray(em, "<i2").tobytes())
    lu_e = np.zeros((ee.shape[0], 64), dtype=np.int8)       # rows padded to 64 B (:207-216)
    lu_e[:, :ee.shape[1]] = ee
    put("EMBED_LU_e", lu_e.tobytes())
    put("NORM_W_m", np.asarray(norm_w[0], "<i2").tobytes())
    put("NORM_W_e", np.asarray(norm_w[1], np.int8).tobytes())
    return bytes(img)


def unpack_image(cfg: BfpConfig, img):
    """Inverse of build_image for the host-side readers (ROMs, gammas):
    returns g1, g2 (lists of (m, e)) and norm_w (m, e)."""
    b = memoryview(img)
    rmap = {name: (off, size) for name, off, size in region_map(cfg)}

    def arr(name, dtype, shape):
        off, size = rmap[name]
        return np.frombuffer(b[off:off + size], dtype=dtype).reshape(shape)

    ntd = cfg.D // 16
    g1m, g1e = arr("G1_m", "<i2", (cfg.NL, cfg.D)), arr("G1_e", np.int8, (cfg.NL, ntd))
    g2m, g2e = arr("G2_m", "<i2", (cfg.NL, cfg.D)), arr("G2_e", np.int8, (cfg.NL, ntd))
    nwm, nwe = arr("NORM_W_m", "<i2", (cfg.D,)), arr("NORM_W_e", np.int8, (ntd,))
    return ([(g1m[i], g1e[i]) for i in range(cfg.NL)], [(g2m[i], g2e[i]) for i in range(cfg.NL)], (nwm, nwe))


__all__ = ["quantize_W", "pack_layer_mantissas", "pack_layer_exponents", "build_image", "unpack_image",
           "ALIGN", "align4k"]
