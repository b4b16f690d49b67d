"""The product's packer layout and image assembly against the reference
packer's bytes (gen_smollm_blockfp_ddr.py), CPU only (the mantissas and
exponents come from the oracle's quantizer; the GPU quantizer is checked in
test_gpu_model.py)."""
import hashlib
import struct

import numpy as np

from common import golden_path, manifest, oracle_model
from oracle import bfp_oracle as O
from bfp200 import pack, image
from bfp200.config import BfpConfig


def _ref_pack_mantissas(m):
    """Byte loop of gen_smollm_blockfp_ddr.py:88-104, restated for a small matrix."""
    D_out, NT, _ = m.shape
    D_in = NT * 16
    buf = bytearray((D_out // 16) * D_in * 32)
    for chunk in range(D_out // 16):
        for col in range(D_in):
            base = (chunk * D_in + col) * 32
            for lane in range(16):
                struct.pack_into("<H", buf, base + lane * 2, int(m[chunk * 16 + lane, col // 16, col % 16]) & 0xFFFF)
    return bytes(buf)


def _ref_pack_exponents(e):
    """:107-119."""
    D_out, NT = e.shape
    buf = bytearray((D_out // 16) * NT * 16)
    for chunk in range(D_out // 16):
        for t in range(NT):
            for lane in range(16):
                buf[(chunk * NT + t) * 16 + lane] = int(e[chunk * 16 + lane, t]) & 0xFF
    return bytes(buf)


def test_layout_matches_reference_loops():
    rng = np.random.default_rng(3)
    m = rng.integers(-32768, 32768, size=(48, 5, 16)).astype(np.int16)
    e = rng.integers(-127, 128, size=(48, 5)).astype(np.int8)
    assert pack.pack_layer_mantissas(m, e) == _ref_pack_mantissas(m)
    assert pack.pack_layer_exponents(e) == _ref_pack_exponents(e)


def test_region_map_matches_reference_image():
    cfg = BfpConfig()
    gold = manifest()["image"]
    rm = image.region_map(cfg)
    assert {n: o for n, o, _ in rm[:-1]} == gold["offsets"]
    assert rm[-1][1] == gold["len"] == image.image_size(cfg)


def test_full_image_bytes_match_reference_packer():
    model = oracle_model()
    cfg = BfpConfig()
    layers = [{k: lw[k] for k in ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd")} for lw in model.layers]
    g1 = [O.tile_quantize(lf["g1"]) for lf in model.layers_float]
    g2 = [O.tile_quantize(lf["g2"]) for lf in model.layers_float]
    g1 = [(m.reshape(-1), e) for m, e in g1]
    g2 = [(m.reshape(-1), e) for m, e in g2]
    embed = O.quantize_W(model.embed)
    nw = O.tile_quantize(model.norm_w)
    img = pack.build_image(cfg, layers, g1, g2, embed, (nw[0].reshape(-1), nw[1]))
    assert hashlib.sha256(img).hexdigest() == manifest()["image"]["sha256"]
    heads = np.load(golden_path("image_heads.npz"))
    for name, off, _ in image.region_map(cfg)[:-1]:
        assert bytes(img[off:off + 4096]) == heads[name].tobytes(), name
    g1b, g2b, nwb = pack.unpack_image(cfg, img)
    assert np.array_equal(g1b[4][0], g1[4][0]) and np.array_equal(nwb[1], nw[1])
