"""The fixed-point ("rtl-exact") leaf-op restatement against the golden
vectors made by the reference's own per-op generators (tests/golden/
make_rtl_golden.py -> rtl_ops.npz)."""
import hashlib
import os

import numpy as np
import pytest

from oracle import bfp_rtl_oracle as R

Z = np.load(os.path.join(os.path.dirname(__file__), "golden", "rtl_ops.npz"))


def test_roms():
    e = R.exp_lut()
    s = R.silu_lut()
    assert hashlib.sha256(e.tobytes()).digest() == Z["exp_lut_sha"].tobytes()
    assert hashlib.sha256(s.tobytes()).digest() == Z["silu_lut_sha"].tobytes()
    assert np.array_equal(e[[0, 1, 511, 767, 895, 1022, 1023]], Z["exp_lut_head"])
    for base in (10000, 100000):
        assert np.array_equal(R.rope_freq_turns(float(base)), Z[f"rope{base}_freq"])


@pytest.mark.parametrize("D", [64, 576, 1536])
def test_matvec(D):
    for i in range(Z[f"mv{D}_xm"].shape[0]):
        m, e = R.matvec(Z[f"mv{D}_xm"][i], Z[f"mv{D}_xe"][i], Z[f"mv{D}_wm"][i], Z[f"mv{D}_we"][i])
        assert np.array_equal(m, Z[f"mv{D}_ym"][i]) and np.array_equal(e, Z[f"mv{D}_ye"][i]), i


@pytest.mark.parametrize("D", [64, 576])
def test_rmsnorm(D):
    for i in range(Z[f"rms{D}_xm"].shape[0]):
        m, e = R.rmsnorm(Z[f"rms{D}_xm"][i], Z[f"rms{D}_xe"][i], Z[f"rms{D}_gm"][i], Z[f"rms{D}_ge"][i])
        assert np.array_equal(m, Z[f"rms{D}_ym"][i]) and np.array_equal(e, Z[f"rms{D}_ye"][i]), i


@pytest.mark.parametrize("base", [10000, 100000])
def test_rope(base):
    turns = Z[f"rope{base}_freq"]
    for i, pos in enumerate(Z[f"rope{base}_pos"]):
        m, e = R.rope(Z[f"rope{base}_xm"][i], Z[f"rope{base}_xe"][i], int(pos), turns)
        assert np.array_equal(m, Z[f"rope{base}_ym"][i]) and np.array_equal(e, Z[f"rope{base}_ye"][i]), pos


@pytest.mark.parametrize("N", [1, 8, 37, 64])
def test_softmax(N):
    lut = R.exp_lut()
    for i in range(Z[f"sm{N}_xm"].shape[0]):
        m, e = R.softmax(Z[f"sm{N}_xm"][i], int(Z[f"sm{N}_xe"][i]), lut)
        assert np.array_equal(m, Z[f"sm{N}_ym"][i]) and e == int(Z[f"sm{N}_ye"][i]), i


@pytest.mark.parametrize("D", [64, 1536])
def test_swiglu(D):
    lut = R.silu_lut()
    for i in range(Z[f"sw{D}_gm"].shape[0]):
        m, e = R.swiglu(Z[f"sw{D}_gm"][i], Z[f"sw{D}_ge"][i], Z[f"sw{D}_um"][i], Z[f"sw{D}_ue"][i], lut)
        assert np.array_equal(m, Z[f"sw{D}_ym"][i]) and np.array_equal(e, Z[f"sw{D}_ye"][i]), i


@pytest.mark.parametrize("D", [64, 576])
def test_residual(D):
    for i in range(Z[f"res{D}_am"].shape[0]):
        m, e = R.residual(Z[f"res{D}_am"][i], Z[f"res{D}_ae"][i], Z[f"res{D}_bm"][i], Z[f"res{D}_be"][i])
        assert np.array_equal(m, Z[f"res{D}_ym"][i]) and np.array_equal(e, Z[f"res{D}_ye"][i]), i
