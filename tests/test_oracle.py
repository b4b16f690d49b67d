"""The oracle (numpy restatement of the reference simulator) against the
golden vectors produced by running the reference's own functions
(tests/golden/make_golden.py).  CPU only."""
import math

import numpy as np
import pytest

import inputs
from common import golden_path, load_sampled, load_tokens, manifest, oracle_model, sha
from oracle import bfp_oracle as O
from oracle import synth


def test_tile_quantize_golden():
    z = np.load(golden_path("quant.npz"))
    m, e = O.tile_quantize(z["v"])
    assert np.array_equal(m, z["m"]) and np.array_equal(e, z["e"])
    assert np.array_equal(O.tile_decode(m, e), z["d"])
    # the generators the GPU tests use reproduce the fixture's input
    assert np.array_equal(inputs.quant_cases(), z["v"])


def _roundup_count(j):
    """Closed form the device code uses for numpy's floor(log2(.)) (see
    bfp_device.cuh log2_roundup_count)."""
    if j == 0:
        return 0
    a = abs(j).bit_length() - 1
    b = a - 1 if (j > 0 and (j & (j - 1)) == 0) else a
    return 0 if b < 1 else int(math.floor(math.log(2) * 2 ** b))


def test_log2_threshold_model():
    """numpy's log2 on THIS host rounds up to j exactly for the doubles the
    closed form predicts, and agrees with the golden host."""
    here = O.floor_log2_threshold_counts(-130, 130)
    gold = {int(k): v for k, v in manifest()["log2_round_up_counts"].items()}
    assert here == gold
    assert all(here[j] == _roundup_count(j) for j in here)


def _pairwise(a, lo, n):
    """numpy's pairwise summation, the algorithm np_pw_leaf / np_pw_combine
    (bfp_device.cuh) implement."""
    if n < 8:
        r = 0.0
        for i in range(n):
            r += a[lo + i]
        return r
    if n <= 128:
        r = [a[lo + j] for j in range(8)]
        i = 8
        while i < n - (n % 8):
            for j in range(8):
                r[j] += a[lo + i + j]
            i += 8
        res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]))
        while i < n:
            res += a[lo + i]
            i += 1
        return res
    n2 = n // 2
    n2 -= n2 % 8
    return _pairwise(a, lo, n2) + _pairwise(a, lo + n2, n - n2)


def test_numpy_pairwise_sum_model():
    rng = np.random.default_rng(0)
    for n in list(range(1, 260)) + [576, 1536, 2047, 2048, 3000]:
        a = rng.standard_normal(n) * np.exp(rng.standard_normal(n) * 4)
        assert 0.0 + _pairwise(a, 0, n) == np.add.reduce(a), n


def _sweep_sha(Y):
    ym, ye = O.tile_quantize(Y.reshape(-1))
    return sha(ym, ye)


@pytest.mark.parametrize("shape", inputs.SWEEP_SHAPES[:4])
def test_matvec_sweep_golden(shape):
    D_out, D_in = shape
    W_m, W_e = inputs.sweep_weights(D_out, D_in)
    gold = manifest()["matvec_sha"]
    for B in (1, 8, 64):
        X_m, X_e = inputs.sweep_x(D_in, B, D_out)
        Y = O.matvec_cols(X_m, X_e, W_m, W_e)
        assert _sweep_sha(Y) == gold[f"{D_out}x{D_in}_b{B}"], (shape, B)


def test_matvec_head_shape_golden():
    W_m, W_e = inputs.sweep_weights(49152, 576)
    X_m, X_e = inputs.sweep_x(576, 8, 49152)
    Y = O.matvec_cols(X_m, X_e, W_m, W_e)
    assert _sweep_sha(Y) == manifest()["matvec_sha"]["49152x576_b8"]


@pytest.mark.parametrize("name", ["shift_mask", "saturate", "mixed", "zero_x"])
def test_matvec_edge_golden(name):
    z = np.load(golden_path(f"matvec_edge_{name}.npz"))
    y = O.matvec_hw_golden(z["x_m"], z["x_e"], z["W_m"], z["W_e"])
    assert np.array_equal(y, z["y"])


def test_fwd_layer_golden():
    model = oracle_model()
    z = np.load(golden_path("layer.npz"))
    cfg = O.Cfg()
    for kv_pos in inputs.LAYER_KV_POS:
        h, K, V = inputs.layer_case(kv_pos, max_ctx=kv_pos + 1)
        kv = {"k": K.copy(), "v": V.copy()}
        out = O.fwd_layer(h, model.layers[0], kv_pos, kv, kv_pos, cfg)
        assert np.array_equal(out, z[f"out_{kv_pos}"]), kv_pos
        assert np.array_equal(kv["k"][kv_pos], z[f"k_{kv_pos}"])
        assert np.array_equal(kv["v"][kv_pos], z[f"v_{kv_pos}"])
    assert O.STATS["score_dots_wide_spread"] == 0


def test_synthetic_weights_are_fixed_points():
    model = oracle_model()
    lf = model.layers_float[3]
    for k in ("Wq", "Wd", "g1"):
        assert np.array_equal(O.fp_quantize_vec(lf[k].reshape(-1)), lf[k].reshape(-1))
    rows = model.embed[::997]
    assert np.array_equal(O.fp_quantize_vec(rows.reshape(-1)), rows.reshape(-1))


def test_tokens_cfg1_golden():
    model = oracle_model()
    prompts, n_gen = synth.config_prompts(1)
    assert O.generate(model, prompts[0], n_gen) == load_tokens(1)[0]


def test_tokens_cfg2_prefix_golden():
    """cfg2 (48-token prompt): the first 12 generated tokens (the full 256 are
    checked on the GPU against the same fixture)."""
    model = oracle_model()
    prompts, _ = synth.config_prompts(2)
    gold = load_tokens(2)[0]
    got = O.generate(model, prompts[0], 12, max_ctx=48 + 256)
    assert got == gold[:48 + 12]


def test_config_prompts_match_product():
    """The product's benchmark prompt generator equals the oracle's."""
    from bfp200 import synth as PS
    for cfg_id in (1, 2, 3):
        assert PS.config_prompts(cfg_id) == synth.config_prompts(cfg_id)


def test_sampled_streams_golden():
    """The oracle's sampling loop (generate_sampled) reproduces the streams the
    reference emulator's own fwd_hw and sampling loop (sim_rtl_fp_hw.py:
    196-216, np.random.seed(SEED)) produced, for every (T, TOPK, SEED) case."""
    model = oracle_model()
    from oracle import synth
    prompt = synth.config_prompts(1)[0][0]
    for case in load_sampled()[1:3]:        # top-k 50 and 5 (the GPU tests run every case)
        got = O.generate_sampled(model, prompt, case["n_gen"], case["temperature"], case["top_k"], case["seed"])
        assert got == case["tokens"], case
