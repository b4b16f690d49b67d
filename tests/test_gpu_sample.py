"""Temperature / top-k sampling (sim_rtl_fp_hw.py:204-216): against the
streams the reference emulator itself produced (tests/golden/sampled.json)
and against the oracle's restatement with numpy's legacy generator: same
seeds, same token streams; draws the fp64 head cannot certify are counted
(none expected)."""
import numpy as np
import pytest

from oracle import bfp_oracle as O
from oracle import synth as OS

pytestmark = pytest.mark.gpu

SMALL = dict(D=128, H_Q=2, H_KV=1, HD=64, FFN=256, NL=3, VOCAB=512)


@pytest.fixture(scope="module")
def small():
    from bfp200 import BfpConfig, Decoder, synth
    cfg = BfpConfig(MAX_CTX=48, max_seqs=8, **SMALL)
    dec = Decoder(cfg)
    dec.load_image(synth.synthetic_image(cfg, 6))
    yield dec, OS.make_model(6, O.Cfg(**SMALL)), O.Cfg(**SMALL)
    dec.close()


@pytest.mark.parametrize("T,topk", [(1.0, 0), (0.7, 0), (0.8, 5), (1.3, 40), (2.0, 1)])
def test_sampled_tokens_match_oracle(small, T, topk):
    dec, model, ocfg = small
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 512, size=int(n)).tolist() for n in (4, 9, 1)]
    got = dec.generate_sampled(prompts, 14, T, topk, seed=3)
    for s, (p, g) in enumerate(zip(prompts, got)):
        assert g == O.generate_sampled(model, p, 14, T, topk, seed=3 + s, max_ctx=48, cfg=ocfg), (s, T, topk)
    assert dec.uncertified_steps() == 0


def test_zero_temperature_is_greedy(small):
    dec, model, ocfg = small
    p = [[5, 6, 7]]
    assert dec.generate_sampled(p, 8, 0.0) == dec.generate(p, 8)


def test_full_model_sampled_prefix():
    """Full SmolLM2-135M synthetic image, cfg1 prompt, a few sampled steps."""
    from bfp200 import BfpConfig, Decoder, synth
    from common import oracle_model
    dec = Decoder(BfpConfig(MAX_CTX=32, max_seqs=2))
    dec.load_image(synth.synthetic_image(BfpConfig(), seed=0))
    prompts, _ = synth.config_prompts(1)
    got = dec.generate_sampled(prompts, 4, 0.9, 50, seed=1)[0]
    assert got == O.generate_sampled(oracle_model(), prompts[0], 4, 0.9, 50, seed=1)
    assert dec.uncertified_steps() == 0
    dec.close()


def test_full_model_sampled_reference_streams():
    """Full SmolLM2-135M synthetic image, cfg1 prompt: every sampled stream the
    reference emulator produced (several temperatures, top-k and seeds)."""
    from bfp200 import BfpConfig, Decoder, synth
    from common import load_sampled
    prompts, _ = synth.config_prompts(1)
    with Decoder(BfpConfig(MAX_CTX=32, max_seqs=2)) as dec:
        dec.load_image(synth.synthetic_image(BfpConfig(), seed=0))
        for case in load_sampled():
            got = dec.generate_sampled(prompts, case["n_gen"], case["temperature"], case["top_k"],
                                       seed=case["seed"])[0]
            assert got == case["tokens"], case
        assert dec.uncertified_steps() == 0
