"""The C-ABI library and the host-side surface, CPU only: the in-tree
libbfp200.so loads and exports every symbol include/bfp200.h declares,
host-only functions match the reference, and compute calls fail loudly
without a GPU (no CPU fallback)."""
import math
import os
import re

import numpy as np
import pytest

from common import gpu_available
from bfp200 import BfpConfig, BfpError, _lib, image

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    with open(os.path.join(REPO, "include", "bfp200.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"^(?:int|void)\s+(bfp200_\w+)\(", text, re.M)))


def test_library_exports_every_header_symbol():
    L = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), s
    assert set(syms) - {"bfp200_default_cfg"} <= set(_lib.SIGNATURES)


def test_default_cfg_matches_reference():
    c = _lib.Cfg()
    _lib.lib().bfp200_default_cfg(c)
    ref = BfpConfig()
    for f in ("D", "H_Q", "H_KV", "HD", "FFN", "NL", "VOCAB", "MAX_CTX", "NPROMPT_MAX"):
        assert getattr(c, f) == getattr(ref, f), f
    assert c.rope_base == 10000.0 and c.eps == 1e-5


def test_rope_table_matches_python_math():
    """The (cos, sin) table the kernels use equals the reference's math.cos /
    math.sin of theta = 1/(base**(2j/HD)) * pos (gen_smollm_blockfp_full.py:253-254)."""
    from bfp200 import ops
    for base in (10000.0, 100000.0):
        t = ops.rope_table(2048, 64, base)
        for pos in list(range(0, 2048, 7)) + [2047]:
            for j in range(32):
                theta = 1.0 / (base ** (2 * j / 64)) * pos
                assert t[pos, j, 0] == math.cos(theta) and t[pos, j, 1] == math.sin(theta), (pos, j)


@pytest.mark.skipif(gpu_available(), reason="checks the no-GPU failure path")
def test_compute_fails_loudly_without_gpu():
    from bfp200 import Decoder, ops
    with pytest.raises(BfpError) as ei:
        Decoder(BfpConfig())
    assert ei.value.code == _lib.ENODEV
    with pytest.raises(BfpError):
        ops.tile_quantize(np.zeros(16))


def test_hex_roundtrip(tmp_path):
    vals = np.array([0, 1, 0x7FFF, 0x8000, 0xFFFF, 0x1234], np.uint16)
    p = tmp_path / "x.hex"
    image.write_hex(p, vals, 4)
    assert np.array_equal(image.parse_hex_file(p), vals)
    # comments and junk are skipped like bfp_client's parse_hex_file
    p.write_text("// header\n00ff # c\nzz 0010\n\n12345\n")
    assert image.parse_hex_file(p).tolist() == [0xFF, 0x10, 0x2345]


def test_rom_files_roundtrip(tmp_path):
    rng = np.random.default_rng(0)
    g = [(rng.integers(-32768, 32768, 64).astype(np.int16), rng.integers(-127, 128, 4).astype(np.int8))
         for _ in range(2)]
    image.write_roms(tmp_path, "p_", g, g, g[0], [1, 2, 3])
    roms = image.read_roms(tmp_path, "p_")
    assert roms[6].tolist() == [1, 2, 3]
    assert np.array_equal(roms[0].astype(np.int16), np.concatenate([m for m, _ in g]))
    assert np.array_equal((roms[1] & 0xFF).astype(np.uint8).view(np.int8), np.concatenate([e for _, e in g]))


def test_release_rom_fixture_format():
    """The reference's release ROM files (real SmolLM2 gammas): every tile is
    normalised (max |m| in [16384, 32767]) and the prompt is the 8-token
    'Once upon a time' encoding."""
    ref = os.environ.get("BFP200_REFERENCE", os.path.join(os.path.dirname(REPO), "reference"))
    rel = os.path.join(ref, "rtl", "vc707", "release")
    if not os.path.isdir(rel):
        pytest.skip("reference checkout not present (set BFP200_REFERENCE)")
    roms = image.read_roms(rel, "lbfp_full_")
    assert roms[6].tolist() == [34, 50, 14669, 5728, 34, 50, 1758, 9148]
    m = roms[0].astype(np.int16).astype(np.int64).reshape(-1, 16)
    assert (np.abs(m).max(axis=1) >= 16384).all() and len(roms[1]) == 30 * 36


def test_cfg_svh_roundtrip(tmp_path):
    cfg = BfpConfig(MAX_CTX=304)
    p = tmp_path / "cfg.svh"
    image.write_cfg_svh(p, cfg, n_prompt=8, n_gen=16)
    back = image.read_cfg_svh(p)
    assert (back.D, back.NL, back.MAX_CTX, back.VOCAB, back.N_GEN) == (576, 30, 304, 49152, 16)
    assert image.rtl_tokens_line([1, 2, 3]) == "RTL_TOKENS: 1 2 3"


def test_config_from_env():
    cfg = BfpConfig.from_env({"D": "64", "NL": "2", "PREFIX": "x_", "MAX_CTX": "128"})
    assert (cfg.D, cfg.NL, cfg.PREFIX, cfg.MAX_CTX, cfg.FFN) == (64, 2, "x_", 128, 1536)
