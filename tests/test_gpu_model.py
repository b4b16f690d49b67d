"""GPU model-level parity: the full SmolLM2-135M synthetic image built on the
GPU (byte-identical to the reference packer), one layer against the
reference's fwd_layer outputs, and greedy token streams against the
reference simulator's golden tokens (cfg1, cfg2, cfg3 prefix)."""
import hashlib

import numpy as np
import pytest

import inputs
from common import golden_path, load_tokens, manifest, oracle_model
from oracle import bfp_oracle as O

pytestmark = pytest.mark.gpu

_IMG = {}


def full_image():
    if "img" not in _IMG:
        from bfp200 import BfpConfig, synth
        _IMG["img"] = synth.synthetic_image(BfpConfig(), seed=0)
    return _IMG["img"]


def test_gpu_packed_image_matches_reference_packer():
    """Quantization on the GPU + the product's packer = the reference
    packer's bytes for the whole 337 MB image."""
    assert hashlib.sha256(full_image()).hexdigest() == manifest()["image"]["sha256"]


@pytest.fixture(scope="module")
def layer_decoder():
    from bfp200 import BfpConfig, Decoder
    dec = Decoder(BfpConfig(MAX_CTX=2048, max_seqs=4))
    dec.load_image(full_image())
    yield dec
    dec.close()


def test_fwd_layer_golden(layer_decoder):
    """fwd_layer (:261-293) at KV lengths 1..2048 vs the reference's outputs."""
    z = np.load(golden_path("layer.npz"))
    for kv_pos in inputs.LAYER_KV_POS:
        h, K, V = inputs.layer_case(kv_pos, max_ctx=2048)
        kc, vc = K[None].copy(), V[None].copy()
        out = layer_decoder.fwd_layer(0, h, kv_pos, kc, vc)
        assert np.array_equal(out, z[f"out_{kv_pos}"]), kv_pos
        assert np.array_equal(kc[0, kv_pos], z[f"k_{kv_pos}"]), kv_pos
        assert np.array_equal(vc[0, kv_pos], z[f"v_{kv_pos}"]), kv_pos


def test_fwd_layer_stages_and_batch(layer_decoder):
    """Per-stage tensors (the N1..D dumps) vs the oracle, 4 columns at once
    on layer 17 with different positions."""
    model = oracle_model()
    cfg = O.Cfg()
    rng = np.random.default_rng(9)
    pos = [0, 3, 40, 300]
    H, KC, VC = [], [], []
    for p in pos:
        H.append(O.fp_quantize_vec(inputs.outlier_normal(rng, 576)))
        K = np.zeros((2048, 3, 64)); V = np.zeros((2048, 3, 64))
        if p:
            K[:p] = O.fp_quantize_vec(rng.standard_normal(p * 192)).reshape(p, 3, 64)
            V[:p] = O.fp_quantize_vec(rng.standard_normal(p * 192)).reshape(p, 3, 64)
        KC.append(K); VC.append(V)
    kc, vc = np.stack(KC), np.stack(VC)
    out, stages = layer_decoder.fwd_layer(17, np.stack(H), pos, kc, vc, stages=True)
    for c, p in enumerate(pos):
        kv = {"k": KC[c].copy(), "v": VC[c].copy()}
        st = {}
        want = O.fwd_layer(H[c], model.layers[17], p, kv, p, cfg, stages=st)
        assert np.array_equal(out[c], want)
        g = stages[c]
        assert np.array_equal(g["n1"], O.tile_decode(*O.tile_quantize(st["n1"])))
        assert np.array_equal(g["q"], st["q"]) and np.array_equal(g["k"], st["k"])
        assert np.array_equal(g["v"], st["v"])
        assert np.array_equal(g["attn"], O.tile_decode(*O.tile_quantize(st["attn"])))
        for nm in ("o", "h1", "g", "u", "d"):
            assert np.array_equal(g[nm], st[nm]), nm
        assert np.array_equal(g["mlp"], O.tile_decode(*O.tile_quantize(st["mlp"])))


def test_fwd_layer_batched_group_attention():
    """A layer at 112 columns, where attention runs one CTA per (column, KV
    head) for the three query heads sharing it, with positions on both sides
    of the batched kernel's 80-row K/V staging chunk (and of 128); every
    column against the oracle."""
    from bfp200 import BfpConfig, Decoder
    model = oracle_model()
    cfg = O.Cfg()
    rng = np.random.default_rng(11)
    ncols, ctx = 112, 320
    pos = rng.integers(0, 300, ncols)
    pos[:9] = [0, 1, 79, 80, 81, 127, 128, 160, 299]
    H = np.stack([O.fp_quantize_vec(inputs.outlier_normal(rng, 576)) for _ in range(ncols)])
    kc = O.fp_quantize_vec(rng.standard_normal(ncols * ctx * 192)).reshape(ncols, ctx, 3, 64)
    vc = O.fp_quantize_vec(rng.standard_normal(ncols * ctx * 192)).reshape(ncols, ctx, 3, 64)
    for c in range(ncols):
        kc[c, pos[c]:] = 0.0
        vc[c, pos[c]:] = 0.0
    with Decoder(BfpConfig(MAX_CTX=ctx, max_seqs=ncols)) as dec:
        dec.load_image(full_image())
        out = dec.fwd_layer(5, H, pos, kc.copy(), vc.copy())
    for c in range(ncols):
        kv = {"k": kc[c].copy(), "v": vc[c].copy()}
        want = O.fwd_layer(H[c], model.layers[5], int(pos[c]), kv, int(pos[c]), cfg)
        assert np.array_equal(out[c], want), c


def test_fwd_layer_long_arena_attention():
    """A layer at 20 columns in a 2048-position arena, where attention
    streams each (column, KV head)'s K / V rows through a ring of 64-row
    chunks: positions on both sides of the chunk boundaries and up to the
    last position; every column against the oracle."""
    from bfp200 import BfpConfig, Decoder
    model = oracle_model()
    cfg = O.Cfg()
    rng = np.random.default_rng(12)
    ncols, ctx = 20, 2048
    pos = np.array([0, 1, 62, 63, 64, 65, 127, 128, 319, 320, 383, 384, 385, 1000, 1023, 1024, 1535, 2046, 2047, 700])
    H = np.stack([O.fp_quantize_vec(inputs.outlier_normal(rng, 576)) for _ in range(ncols)])
    kc = np.zeros((ncols, ctx, 3, 64))
    vc = np.zeros((ncols, ctx, 3, 64))
    for c in range(ncols):
        p = int(pos[c])
        if p:
            kc[c, :p] = O.fp_quantize_vec(rng.standard_normal(p * 192)).reshape(p, 3, 64)
            vc[c, :p] = O.fp_quantize_vec(rng.standard_normal(p * 192)).reshape(p, 3, 64)
    with Decoder(BfpConfig(MAX_CTX=ctx, max_seqs=ncols)) as dec:
        dec.load_image(full_image())
        out = dec.fwd_layer(9, H, pos, kc.copy(), vc.copy())
    for c in range(ncols):
        kv = {"k": kc[c].copy(), "v": vc[c].copy()}
        want = O.fwd_layer(H[c], model.layers[9], int(pos[c]), kv, int(pos[c]), cfg)
        assert np.array_equal(out[c], want), (c, int(pos[c]))


@pytest.fixture(scope="module")
def decoder():
    from bfp200 import BfpConfig, Decoder
    dec = Decoder(BfpConfig(MAX_CTX=48 + 256, max_seqs=256))
    dec.load_image(full_image())
    yield dec
    dec.close()


def test_tokens_cfg1(decoder):
    from bfp200 import synth
    prompts, n_gen = synth.config_prompts(1)
    assert decoder.generate(prompts, n_gen) == [load_tokens(1)[0]]
    assert decoder.uncertified_steps() == 0


def test_tokens_cfg1_rtl_feed(decoder):
    """feed_mode='rtl' (autoregress_bfp_top.sv:358-384) vs the oracle."""
    from bfp200 import synth
    prompts, n_gen = synth.config_prompts(1)
    got = decoder.generate(prompts, 6, feed_mode="rtl")[0]
    want = O.generate(oracle_model(), prompts[0], 6, feed_mode="rtl")
    assert got == want


def test_tokens_cfg2(decoder):
    from bfp200 import synth
    prompts, n_gen = synth.config_prompts(2)
    assert decoder.generate(prompts, n_gen) == [load_tokens(2)[0]]
    assert decoder.uncertified_steps() == 0


def test_tokens_cfg3_batched(decoder):
    """All 256 ragged sequences in one batch, each against the reference
    simulator's own golden stream (tests/golden/tokens_cfg3.json)."""
    from bfp200 import synth
    prompts, n_gen = synth.config_prompts(3)
    out = decoder.generate(prompts, n_gen)
    gold = load_tokens(3)
    assert len(gold) == 256
    for i, toks in gold.items():
        assert out[i] == toks, i
    assert decoder.uncertified_steps() == 0
    # batching does not change a sequence's stream
    assert decoder.generate(prompts[:3], n_gen) == out[:3]


def test_tokens_cfg3_rank_share(decoder):
    """The first 33 cfg3 sequences in one batch -- one GPU's share of the
    8-way sequence split: the tuned tensor-core matmuls at 33 columns (K
    split across a cluster) and the per-head batched attention, each stream
    against the reference simulator's golden tokens."""
    from bfp200 import synth
    prompts, n_gen = synth.config_prompts(3)
    out = decoder.generate(prompts[:33], n_gen)
    gold = load_tokens(3)
    for i in range(33):
        assert out[i] == gold[i], i
    assert decoder.uncertified_steps() == 0


@pytest.mark.parametrize("ncols", [1, 2, 4])
def test_decode_kernels_stages(layer_decoder, ncols):
    """Every intermediate tensor of the kernels a decode step runs for 1..4
    columns (the fused attention block + gate/up + down at one column, the
    five small-batch kernels at 2..4) against the oracle's stages of
    fwd_layer (:261-293), at positions on both sides of the warp and
    staging boundaries."""
    model = oracle_model()
    cfg = O.Cfg()
    rng = np.random.default_rng(40 + ncols)
    pos = [0, 1, 31, 33, 48, 177, 303, 1000]
    for p0 in range(0, len(pos), ncols):
        ps = pos[p0:p0 + ncols]
        ps = ps + [5] * (ncols - len(ps))
        H, KC, VC = [], [], []
        for p in ps:
            H.append(O.fp_quantize_vec(inputs.outlier_normal(rng, 576)))
            K = np.zeros((2048, 3, 64)); V = np.zeros((2048, 3, 64))
            if p:
                K[:p] = O.fp_quantize_vec(rng.standard_normal(p * 192)).reshape(p, 3, 64)
                V[:p] = O.fp_quantize_vec(rng.standard_normal(p * 192)).reshape(p, 3, 64)
            KC.append(K); VC.append(V)
        kc, vc = np.stack(KC), np.stack(VC)
        layer = 7 + p0
        out, stages = layer_decoder.fwd_layer(layer, np.stack(H), ps, kc, vc, stages=True, decode_kernels=True)
        for c, p in enumerate(ps):
            kv = {"k": KC[c].copy(), "v": VC[c].copy()}
            st = {}
            want = O.fwd_layer(H[c], model.layers[layer], p, kv, p, cfg, stages=st)
            g = stages[c]
            ctx = (ncols, c, p)
            assert np.array_equal(g["n1"], O.tile_decode(*O.tile_quantize(st["n1"]))), ctx
            for nm in ("q", "k", "v"):
                assert np.array_equal(g[nm], st[nm]), (nm,) + ctx
            assert np.array_equal(g["attn"], O.tile_decode(*O.tile_quantize(st["attn"]))), ctx
            for nm in ("o", "h1"):
                assert np.array_equal(g[nm], st[nm]), (nm,) + ctx
            assert np.array_equal(g["n2"], O.tile_decode(*O.tile_quantize(st["n2"]))), ctx
            for nm in ("g", "u"):
                assert np.array_equal(g[nm], st[nm]), (nm,) + ctx
            assert np.array_equal(g["mlp"], O.tile_decode(*O.tile_quantize(st["mlp"]))), ctx
            assert np.array_equal(g["d"], st["d"]), ctx
            assert np.array_equal(out[c], want), ctx
            assert np.array_equal(kc[c, p], kv["k"][p]) and np.array_equal(vc[c, p], kv["v"][p]), ctx


def test_fwd_layer_33_columns():
    """A layer at 33 columns (cfg3's share per GPU at 8 GPUs): the tensor-core
    matmuls with the store, residual and SwiGLU epilogues on a ragged column
    tile, against the oracle for every column."""
    from bfp200 import BfpConfig, Decoder
    model = oracle_model()
    cfg = O.Cfg()
    rng = np.random.default_rng(33)
    ncols, ctx = 33, 200
    pos = rng.integers(0, 190, ncols)
    H = np.stack([O.fp_quantize_vec(inputs.outlier_normal(rng, 576)) for _ in range(ncols)])
    kc = O.fp_quantize_vec(rng.standard_normal(ncols * ctx * 192)).reshape(ncols, ctx, 3, 64)
    vc = O.fp_quantize_vec(rng.standard_normal(ncols * ctx * 192)).reshape(ncols, ctx, 3, 64)
    for c in range(ncols):
        kc[c, pos[c]:] = 0.0
        vc[c, pos[c]:] = 0.0
    with Decoder(BfpConfig(MAX_CTX=ctx, max_seqs=ncols)) as dec:
        dec.load_image(full_image())
        out = dec.fwd_layer(11, H, pos, kc.copy(), vc.copy())
    for c in range(ncols):
        kv = {"k": kc[c].copy(), "v": vc[c].copy()}
        want = O.fwd_layer(H[c], model.layers[11], int(pos[c]), kv, int(pos[c]), cfg)
        assert np.array_equal(out[c], want), c
