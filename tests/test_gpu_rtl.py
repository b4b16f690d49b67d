"""The fixed-point ("rtl-exact") leaf ops on the GPU against the reference
generators' golden vectors (tests/golden/rtl_ops.npz) and against the
integer restatement on seeded random inputs, including saturating and
degenerate cases."""
import os

import numpy as np
import pytest

from oracle import bfp_rtl_oracle as R

pytestmark = pytest.mark.gpu

Z = np.load(os.path.join(os.path.dirname(__file__), "golden", "rtl_ops.npz"))


def _tq(rng, shape, scale):
    v = rng.standard_normal(shape + (16,)) * scale
    e = (np.floor(np.log2(np.maximum(np.abs(v).max(axis=-1), 1e-300))).astype(np.int32) + 1).clip(-127, 127)
    m = np.clip(np.round(v / np.power(2.0, e)[..., None] * 32768.0), -32768, 32767).astype(np.int16)
    return m, e.astype(np.int8)


def test_roms_match_generators():
    from bfp200 import rtl
    import hashlib
    assert hashlib.sha256(rtl.exp_lut().tobytes()).digest() == Z["exp_lut_sha"].tobytes()
    assert hashlib.sha256(rtl.silu_lut().tobytes()).digest() == Z["silu_lut_sha"].tobytes()
    assert np.array_equal(rtl.rope_freq_turns(100000.0), Z["rope100000_freq"])


@pytest.mark.parametrize("D", [64, 576, 1536])
def test_matvec_golden(D):
    from bfp200 import rtl
    for i in range(Z[f"mv{D}_xm"].shape[0]):
        m, e = rtl.matvec(Z[f"mv{D}_xm"][i], Z[f"mv{D}_xe"][i], Z[f"mv{D}_wm"][i], Z[f"mv{D}_we"][i])
        assert np.array_equal(m, Z[f"mv{D}_ym"][i]) and np.array_equal(e, Z[f"mv{D}_ye"][i]), i


def test_matvec_batched_random():
    from bfp200 import rtl
    rng = np.random.default_rng(1)
    xm, xe = _tq(rng, (5, 36), 3.0)
    xe[2] -= 60                                     # exponent gaps beyond the 48-bit window
    wm, we = _tq(rng, (40, 36), 0.5)
    we[:, ::4] += 20
    wm[7] = 32767; wm[8] = -32768; we[7] = 127; we[8] = 127     # saturation
    m, e = rtl.matvec(xm, xe, wm, we)
    for b in range(5):
        om, oe = R.matvec(xm[b], xe[b], wm, we)
        assert np.array_equal(m[b], om) and np.array_equal(e[b], oe), b


@pytest.mark.parametrize("D", [64, 576])
def test_rmsnorm_golden(D):
    from bfp200 import rtl
    m, e = rtl.rmsnorm(Z[f"rms{D}_xm"], Z[f"rms{D}_xe"], Z[f"rms{D}_gm"], Z[f"rms{D}_ge"])
    n = Z[f"rms{D}_xm"].shape[0]
    assert np.array_equal(m.reshape(n, -1), Z[f"rms{D}_ym"]) and np.array_equal(e, Z[f"rms{D}_ye"])


def test_rmsnorm_random_and_zero():
    from bfp200 import rtl
    rng = np.random.default_rng(2)
    for D, scale in ((1536, 2.0), (576, 1e-30), (128, 1e30)):
        xm, xe = _tq(rng, (3, D // 16), scale)
        gm, ge = _tq(rng, (3, D // 16), 1.0)
        xm[1] = 0                                     # all-zero vector: epsilon only
        m, e = rtl.rmsnorm(xm, xe, gm, ge)
        for b in range(3):
            om, oe = R.rmsnorm(xm[b], xe[b], gm[b], ge[b])
            assert np.array_equal(m[b].reshape(-1), om) and np.array_equal(e[b], oe), (D, b)


@pytest.mark.parametrize("base", [10000, 100000])
def test_rope_golden(base):
    from bfp200 import rtl
    m, e = rtl.rope(Z[f"rope{base}_xm"], Z[f"rope{base}_xe"], Z[f"rope{base}_pos"], Z[f"rope{base}_freq"])
    assert np.array_equal(m, Z[f"rope{base}_ym"]) and np.array_equal(e, Z[f"rope{base}_ye"])


def test_rope_all_positions():
    from bfp200 import rtl
    rng = np.random.default_rng(3)
    turns = rtl.rope_freq_turns(100000.0)
    pos = np.arange(0, 2048, 7)
    xm, xe = _tq(rng, (pos.size, 4), 1.0)
    xe[::5, 1] -= 20                               # pairs whose halves are 16+ bits apart
    m, e = rtl.rope(xm, xe, pos, turns)
    for i, p in enumerate(pos):
        om, oe = R.rope(xm[i], xe[i], int(p), turns)
        assert np.array_equal(m[i], om) and np.array_equal(e[i], oe), p


@pytest.mark.parametrize("N", [1, 8, 37, 64])
def test_softmax_golden(N):
    from bfp200 import rtl
    m, e = rtl.softmax(Z[f"sm{N}_xm"], Z[f"sm{N}_xe"])
    assert np.array_equal(m, Z[f"sm{N}_ym"]) and np.array_equal(e, Z[f"sm{N}_ye"])


def test_softmax_long_and_extreme_exponents():
    from bfp200 import rtl
    rng = np.random.default_rng(4)
    lut = R.exp_lut()
    for n, e0 in ((2048, -3), (300, 40), (100, -70), (5, 127)):
        xm = rng.integers(-32768, 32768, size=(2, n)).astype(np.int16)
        m, e = rtl.softmax(xm, np.array([e0, e0 + 1]))
        for b in range(2):
            om, oe = R.softmax(xm[b], e0 + b, lut)
            assert np.array_equal(m[b], om) and e[b] == oe, (n, e0, b)


@pytest.mark.parametrize("D", [64, 1536])
def test_swiglu_golden(D):
    from bfp200 import rtl
    m, e = rtl.swiglu(Z[f"sw{D}_gm"], Z[f"sw{D}_ge"], Z[f"sw{D}_um"], Z[f"sw{D}_ue"])
    n = Z[f"sw{D}_gm"].shape[0]
    assert np.array_equal(m.reshape(n, -1), Z[f"sw{D}_ym"]) and np.array_equal(e, Z[f"sw{D}_ye"])


def test_swiglu_extreme_gate_exponents():
    from bfp200 import rtl
    rng = np.random.default_rng(5)
    gm, ge = _tq(rng, (40,), 1.0)
    um, ue = _tq(rng, (40,), 1.0)
    ge[:] = np.arange(-100, 120, 220 / 40).astype(np.int8)[:40]
    m, e = rtl.swiglu(gm, ge, um, ue)
    om, oe = R.swiglu(gm, ge, um, ue, R.silu_lut())
    assert np.array_equal(m.reshape(-1), om) and np.array_equal(e, oe)


@pytest.mark.parametrize("D", [64, 576])
def test_residual_golden(D):
    from bfp200 import rtl
    m, e = rtl.residual(Z[f"res{D}_am"], Z[f"res{D}_ae"], Z[f"res{D}_bm"], Z[f"res{D}_be"])
    n = Z[f"res{D}_am"].shape[0]
    assert np.array_equal(m.reshape(n, -1), Z[f"res{D}_ym"]) and np.array_equal(e, Z[f"res{D}_ye"])
