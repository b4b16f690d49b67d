"""GPU parity on small random models (fast, many shapes): token streams of
the C-ABI decoder against the oracle for several seeds, ragged batches, both
feed modes and KV lengths up to MAX_CTX; error paths of the ABI."""
import numpy as np
import pytest

from oracle import bfp_oracle as O
from oracle import synth as OS

pytestmark = pytest.mark.gpu

SMALL = dict(D=128, H_Q=2, H_KV=1, HD=64, FFN=256, NL=3, VOCAB=512)


def _pair(seed, max_ctx, max_seqs, **kw):
    from bfp200 import BfpConfig, Decoder, synth
    dims = dict(SMALL, **kw)
    cfg = BfpConfig(MAX_CTX=max_ctx, max_seqs=max_seqs, **dims)
    dec = Decoder(cfg)
    dec.load_image(synth.synthetic_image(cfg, seed))
    ocfg = O.Cfg(**dims)
    return dec, OS.make_model(seed, ocfg), ocfg


@pytest.mark.parametrize("seed", [1, 2])
def test_small_model_ragged_batch(seed):
    dec, model, ocfg = _pair(seed, 40, 5)
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, 512, size=int(n)).tolist() for n in (1, 2, 7, 16, 30)]
    got = dec.generate(prompts, 10)
    for p, g in zip(prompts, got):
        assert g == O.generate(model, p, 10, max_ctx=40, cfg=ocfg)
    got_rtl = dec.generate(prompts[:2], 5, feed_mode="rtl")
    for p, g in zip(prompts[:2], got_rtl):
        assert g == O.generate(model, p, 5, max_ctx=40, cfg=ocfg, feed_mode="rtl")
    dec.close()


def test_small_model_full_context():
    """prompt + n_gen == MAX_CTX exactly; GQA with 3 query heads per KV head."""
    dec, model, ocfg = _pair(3, 64, 2, H_Q=3, D=192, FFN=384)
    prompts = [[5, 6, 7, 8], list(range(20, 44))]
    got = dec.generate(prompts, 40)
    assert got[0] == O.generate(model, prompts[0], 40, max_ctx=64, cfg=ocfg)
    got1 = dec.generate(prompts[1:], 40)[0]
    assert got1 == O.generate(model, prompts[1], 40, max_ctx=64, cfg=ocfg)
    dec.close()


def test_small_model_long_arena_decode():
    """A KV arena of 1024 positions and more than four sequences: batched
    attention streams K / V in 64-row chunks; 90 decode steps from prompts
    of 30-48 tokens cross the chunk boundaries 64 and 128 (the chunks below
    the last one stream before the dependency wait).  3 query heads per KV
    head, as in the full model."""
    dec, model, ocfg = _pair(4, 1024, 6, H_Q=3, D=192, FFN=384)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 512, size=n).tolist() for n in (30, 40, 47, 48, 45, 33)]
    got = dec.generate(prompts, 90)
    for p, g in zip(prompts, got):
        assert g == O.generate(model, p, 90, max_ctx=1024, cfg=ocfg)
    dec.close()


def test_error_paths():
    from bfp200 import BfpConfig, BfpError, Decoder, _lib, synth
    cfg = BfpConfig(MAX_CTX=16, max_seqs=2, **SMALL)
    dec = Decoder(cfg)
    with pytest.raises(BfpError) as e:
        dec.generate([[1, 2]], 4)
    assert e.value.code == _lib.ESTATE
    with pytest.raises(BfpError) as e:
        dec.load_image(b"\0" * 1000)
    assert e.value.code == _lib.EIMAGE
    dec.load_image(synth.synthetic_image(cfg, 1))
    with pytest.raises(BfpError) as e:
        dec.generate([[1, 2]], 15)                 # 2 + 15 > MAX_CTX
    assert e.value.code == _lib.EINVAL
    with pytest.raises(BfpError):
        dec.generate([[600]], 2)                   # token outside the vocabulary
    with pytest.raises(BfpError):
        dec.generate([[1]] * 3, 2)                 # more sequences than max_seqs
    with pytest.raises(BfpError):
        dec.generate([list(range(49))], 1)         # longer than NPROMPT_MAX
    with pytest.raises(BfpError):
        dec.load_rom(6, [])                        # empty prompt ROM
    with pytest.raises(BfpError):
        dec.load_rom(0, [0] * 10)                  # wrong gamma ROM length
    assert dec.generate([[1, 2]], 3)[0][:2] == [1, 2]
    dec.close()


def test_rom_prompt_and_gamma_roms():
    """load-roms path: prompt from the PROMPT ROM; gammas re-loaded from ROM
    entries give the same stream as the image's gammas."""
    from bfp200 import BfpConfig, Decoder, pack, synth
    cfg = BfpConfig(MAX_CTX=32, max_seqs=1, **SMALL)
    img = synth.synthetic_image(cfg, 4)
    g1, g2, nw = pack.unpack_image(cfg, img)
    dec = Decoder(cfg)
    dec.load_image(img)
    dec.load_rom(6, [9, 8, 7])
    a = dec.generate(None, 5)
    dec.load_rom(0, np.concatenate([m for m, _ in g1]).view(np.uint16))
    dec.load_rom(1, np.concatenate([e for _, e in g1]).astype(np.uint8).astype(np.uint16))
    b = dec.generate(None, 5)
    assert a == b and a[0][:3] == [9, 8, 7]
    dec.close()


@pytest.mark.parametrize("nseq", [1, 2, 3, 4])
def test_small_batch_kernels_match_general_kernels(nseq, monkeypatch):
    """1..4 columns: the graph-replayed decode kernels (the one-column
    attention block and the small-batch GEMVs, the default), the same with
    the attention block turned off (BFP200_NO_BLOCK), the general matmul path
    (BFP200_NO_SMALL) and the oracle agree."""
    from bfp200 import BfpConfig, Decoder, synth
    cfg = BfpConfig(MAX_CTX=48, max_seqs=4, **SMALL)
    img = synth.synthetic_image(cfg, 5)
    rng = np.random.default_rng(50 + nseq)
    prompts = [rng.integers(0, 512, size=int(n)).tolist() for n in (3, 11, 1, 20)[:nseq]]
    results = []
    for env in ({}, {"BFP200_NO_BLOCK": "1"}, {"BFP200_NO_SMALL": "1"}):
        for k in ("BFP200_NO_BLOCK", "BFP200_NO_SMALL"):
            monkeypatch.delenv(k, raising=False)
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        dec = Decoder(cfg)
        dec.load_image(img)
        results.append((dec.generate(prompts, 12), dec.generate(prompts, 5, feed_mode="rtl")))
        dec.close()
    assert results[0] == results[1] == results[2]
    ocfg = O.Cfg(**SMALL)
    model = OS.make_model(5, ocfg)
    for p, g in zip(prompts, results[0][0]):
        assert g == O.generate(model, p, 12, max_ctx=48, cfg=ocfg)


def test_single_stream_long_context():
    """One sequence decoded past 256 positions (positions 0..299) through the
    one-column attention block, against the oracle."""
    from bfp200 import BfpConfig, Decoder, synth
    cfg = BfpConfig(MAX_CTX=300, max_seqs=2, **SMALL)
    img = synth.synthetic_image(cfg, 7)
    prompt = [7, 9]
    with Decoder(cfg) as dec:
        dec.load_image(img)
        got = dec.generate([prompt], 298)[0]
    ocfg = O.Cfg(**SMALL)
    model = OS.make_model(7, ocfg)
    assert got == O.generate(model, prompt, 298, max_ctx=300, cfg=ocfg)


def test_bounded_wait_times_out_and_handle_recovers():
    """A device-side wait on a flag nothing sets gives up after its limit,
    records the timeout in the library's error flag (the path every bounded
    TMA-barrier / tensor-memory wait takes), the call returns BFP200_ETIMEOUT
    and the handle keeps decoding with the same results."""
    from bfp200 import BfpConfig, Decoder, synth, _lib
    cfg = BfpConfig(MAX_CTX=48, max_seqs=2, **SMALL)
    with Decoder(cfg) as dec:
        dec.load_image(synth.synthetic_image(cfg, 5))
        before = dec.generate([[1, 2, 3]], 4)
        rc = _lib.lib().bfp200_wait_probe(dec.handle, 50)
        assert rc == _lib.ETIMEOUT and "timed out" in _lib.last_error()
        assert dec.generate([[1, 2, 3]], 4) == before
        assert _lib.lib().bfp200_wait_probe(dec.handle, 50) == _lib.ETIMEOUT
