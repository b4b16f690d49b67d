"""GPU op-level parity: the kernels behind bfp200's C ABI against the golden
fixtures and the oracle.  Bit-exact for integer and IEEE-exact stages;
stages that call exp (silu_fp, softmax_fp) use CUDA's exp where the
reference uses numpy's, so they are held to a stated tolerance."""
import math

import numpy as np
import pytest

import inputs
from common import golden_path, manifest, sha
from oracle import bfp_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from bfp200 import ops as _ops
    return _ops


def test_tile_quantize_golden(ops):
    z = np.load(golden_path("quant.npz"))
    m, e = ops.tile_quantize(z["v"])
    assert np.array_equal(m, z["m"]) and np.array_equal(e, z["e"])
    assert np.array_equal(ops.tile_decode(m, e), z["d"])


def test_tile_quantize_random_and_thresholds(ops):
    rng = np.random.default_rng(21)
    v = np.concatenate([inputs.outlier_normal(rng, 16 * 4096),
                        rng.standard_normal(16 * 4096) * np.exp2(rng.integers(-200, 200, size=16 * 4096))])
    # doubles within 100 ulps below every power of two in the exponent range
    p = np.ldexp(1.0, np.repeat(np.arange(-140, 140), 16))
    k = np.tile(np.arange(16), 280) * 7
    near = p * (1.0 - k * 2.0 ** -53)
    # tiles mixing a near-power-of-two element with others: the near element
    # is the maximum (log2 round-up path), shares the maximum's binade without
    # being the maximum, or sits in a lower binade (exponent from the others)
    j = np.arange(-120, 120)
    nr = np.ldexp(1.0 - 3 * 2.0 ** -53, j)                  # binade j-1, top fraction bits all ones
    mixed = []
    for lead, rest in ((nr, 0.3 * nr), (0.75 * nr, nr), (0.5 * nr, 0.75 * nr), (nr * 0.999, nr)):
        t = np.repeat(rest[:, None], 16, axis=1) * rng.uniform(0.1, 1.0, size=(len(j), 16))
        t[:, rng.integers(0, 16, size=len(j))] = 0.0
        t[np.arange(len(j)), rng.integers(0, 16, size=len(j))] = lead
        mixed.append(t.reshape(-1))
    specials = np.array([0.0] * 16 + [np.inf] + [1.0] * 15 + [np.nan] + [2.0] * 15 + [-np.inf] + [0.0] * 15
                        + [1e-310] * 16 + [5e-301, 1e-300] + [2e-300] * 14)
    v = np.concatenate([v, near, -near] + mixed + [specials])
    m, e = ops.tile_quantize(v)
    mo, eo = O.tile_quantize(v)
    assert np.array_equal(m, mo) and np.array_equal(e, eo)


def _sweep_sha(Y):
    ym, ye = O.tile_quantize(Y.reshape(-1))
    return sha(ym, ye)


@pytest.mark.parametrize("shape", inputs.SWEEP_SHAPES)
def test_matvec_sweep(ops, shape):
    """cfg4: every weight shape at batch 1..1024, bit-exact: against the
    reference's own outputs (hash) where it was run, the oracle otherwise."""
    D_out, D_in = shape
    W_m, W_e = inputs.sweep_weights(D_out, D_in)
    gold = manifest()["matvec_sha"]
    for B in inputs.SWEEP_BATCHES:
        X_m, X_e = inputs.sweep_x(D_in, B, D_out)
        om, oe = ops.matvec(X_m, X_e, W_m, W_e)
        Y = ops.tile_decode(om.reshape(-1), oe.reshape(-1)).reshape(B, D_out)
        key = f"{D_out}x{D_in}_b{B}"
        if key in gold:
            assert _sweep_sha(Y) == gold[key], key
        cols = np.arange(B) if D_out * B <= 64 * 1536 else np.linspace(0, B - 1, 6).astype(int)
        ref = O.matvec_cols(X_m[cols], X_e[cols], W_m, W_e)
        assert np.array_equal(Y[cols], ref), key


@pytest.mark.parametrize("shape", [(576, 576), (576, 1536)])
def test_matvec_batched_shift_paths(ops, shape):
    """Batched (tensor-core) matvec with model-like exponent spreads, where
    every per-tile shift is small, and with outlier tiles that push some
    shifts past 16: both shift paths of the epilogue against the oracle."""
    D_out, D_in = shape
    rng = np.random.default_rng([9, D_out, D_in])
    NT = D_in // 16
    W_m = rng.integers(-32768, 32768, size=(D_out, NT, 16)).astype(np.int16)
    W_e = rng.integers(-3, 1, size=(D_out, NT)).astype(np.int8)
    B = 256
    X_m, X_e = inputs.sweep_x(D_in, B, D_out)
    cols = np.linspace(0, B - 1, 12).astype(int)
    om, oe = ops.matvec(X_m, X_e, W_m, W_e)
    Y = ops.tile_decode(om.reshape(-1), oe.reshape(-1)).reshape(B, D_out)
    assert np.array_equal(Y[cols], O.matvec_cols(X_m[cols], X_e[cols], W_m, W_e))
    X_e2 = X_e.copy()
    X_e2[::3, NT // 2] += 20                    # outlier tiles: shifts of 17..30 elsewhere
    om, oe = ops.matvec(X_m, X_e2, W_m, W_e)
    Y = ops.tile_decode(om.reshape(-1), oe.reshape(-1)).reshape(B, D_out)
    assert np.array_equal(Y[cols], O.matvec_cols(X_m[cols], X_e2[cols], W_m, W_e))


@pytest.mark.parametrize("name", ["shift_mask", "saturate", "mixed", "zero_x"])
def test_matvec_edges(ops, name):
    z = np.load(golden_path(f"matvec_edge_{name}.npz"))
    assert np.array_equal(ops.matvec_hw_golden(z["x_m"], z["x_e"], z["W_m"], z["W_e"]), z["y"])


def test_rmsnorm_fp_exact(ops):
    """cfg5-style activations (N(0,1), 1% x30): bit-exact (IEEE ops + numpy
    pairwise mean reproduced)."""
    rng = np.random.default_rng(5)
    x = O.fp_quantize_vec(inputs.outlier_normal(rng, 64 * 576)).reshape(64, 576)
    g = O.fp_quantize_vec(1.0 + 0.05 * rng.standard_normal(576))
    got = ops.rmsnorm_fp(x, g)
    want = np.stack([O.rmsnorm_fp(x[i], g) for i in range(64)])
    assert np.array_equal(got, want)


def test_rope_fp_exact(ops):
    """RoPE at positions 0..2047 on 64-dim heads: bit-exact."""
    rng = np.random.default_rng(6)
    x = O.fp_quantize_vec(inputs.outlier_normal(rng, 2048 * 64)).reshape(2048, 64)
    pos = np.arange(2048)
    got = ops.rope_fp(x, pos)
    want = np.stack([O.rope_fp(x[i], int(pos[i])) for i in range(2048)])
    assert np.array_equal(got, want)


def test_silu_fp_tolerance(ops):
    """silu_fp = fpq(x / (1 + exp(-x))): CUDA exp vs numpy exp may differ in
    the last ulp, which can move a BFP mantissa only when the quotient sits
    on a rounding boundary.  Tolerance: at most 1 mantissa LSB, on at most
    1e-5 of the elements."""
    rng = np.random.default_rng(7)
    x = O.fp_quantize_vec(inputs.outlier_normal(rng, 64 * 1536))
    got = ops.silu_fp(x)
    want = O.silu_fp(x)
    diff = got != want
    assert diff.mean() <= 1e-5
    if diff.any():
        _, e = O.tile_quantize(want)
        lsb = np.repeat(np.power(2.0, e.astype(np.float64) - 15), 16)
        assert (np.abs(got - want)[diff] <= lsb[diff]).all()


def test_pairwise_sum_exact(ops):
    """The device reduction reproduces numpy's pairwise summation bit for bit
    (every tree shape up to the largest KV length)."""
    rng = np.random.default_rng(10)
    for n in list(range(1, 300)) + [576, 1000, 1536, 2047, 2048, 3072]:
        x = rng.standard_normal((4, n)) * np.exp(rng.standard_normal((4, n)) * 4)
        assert np.array_equal(ops.pairwise_sum(x), np.add.reduce(x, axis=1)), n


def test_softmax_fp_tolerance(ops):
    """softmax_fp over T=2048 scores.  CUDA's exp and numpy's exp (its AVX-512
    kernel is correctly rounded on ~95% of inputs) differ by <= 1 ulp, so the
    stated tolerance is max |rel err| <= 4 ulp; the max, the pairwise sum
    and the division are reproduced exactly."""
    rng = np.random.default_rng(8)
    x = inputs.outlier_normal(rng, 64 * 2048).reshape(64, 2048)
    got = ops.softmax_fp(x)
    want = np.stack([O.softmax_fp(x[i]) for i in range(64)])
    rel = np.abs(got - want) / np.maximum(np.abs(want), np.finfo(float).tiny)
    assert rel.max() <= 4 * 2.0 ** -52
    assert (got == want).mean() > 0.85


@pytest.mark.parametrize("shape", [(576, 576), (192, 576), (576, 1536)])
def test_matvec_tensor_core_few_columns(ops, shape):
    """16..63 columns run on the tensor cores too (a ragged last 16- or
    32-column tile): every column against the oracle."""
    D_out, D_in = shape
    W_m, W_e = inputs.sweep_weights(D_out, D_in)
    for B in (16, 17, 33, 48, 63):
        X_m, X_e = inputs.sweep_x(D_in, B, D_out)
        om, oe = ops.matvec(X_m, X_e, W_m, W_e)
        Y = ops.tile_decode(om.reshape(-1), oe.reshape(-1)).reshape(B, D_out)
        assert np.array_equal(Y, O.matvec_cols(X_m, X_e, W_m, W_e)), (shape, B)
