"""Vocabulary-sharded head (single-stream latency over several GPUs): every
rank runs the layers, scans its share of the embedding rows and the ranks
exchange (max logit, lowest index, runner-up, ||hn||) records with an NCCL
all-gather inside the decode graph.  The token streams must equal the
unsharded ones and the reference simulator's (np.argmax semantics,
gen_smollm_blockfp_full.py:439-440).  One-rank groups run on one GPU; the
2-GPU cases run when two devices are visible."""
import os

import numpy as np
import pytest

from common import load_tokens
from oracle import bfp_oracle as O
from oracle import synth as OS

pytestmark = pytest.mark.gpu

SMALL = dict(D=128, H_Q=2, H_KV=1, HD=64, FFN=256, NL=3, VOCAB=512)


def _n_gpus():
    import torch
    return torch.cuda.device_count()


def _small(seed, device=0):
    from bfp200 import BfpConfig, Decoder, synth
    cfg = BfpConfig(MAX_CTX=40, max_seqs=6, **SMALL)
    dec = Decoder(cfg, device=device)
    dec.load_image(synth.synthetic_image(cfg, seed))
    return dec, OS.make_model(seed, O.Cfg(**SMALL)), O.Cfg(**SMALL)


def test_one_rank_group_matches_oracle():
    """The sharded path (partial head -> NCCL all-gather -> combine) with one
    rank, for the single-launch head (1 column) and the batched head (6)."""
    from bfp200 import nccl_unique_id
    dec, model, ocfg = _small(4)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 512, size=int(n)).tolist() for n in (3, 9, 1, 20, 5, 12)]
    plain1 = dec.generate(prompts[:1], 12)
    plain6 = dec.generate(prompts, 12)
    dec.shard_head(nccl_unique_id(), 1, 0)
    assert dec.generate(prompts[:1], 12) == plain1
    got = dec.generate(prompts, 12)
    assert got == plain6
    for p, g in zip(prompts, got):
        assert g == O.generate(model, p, 12, max_ctx=40, cfg=ocfg)
    rtl = dec.generate(prompts[:2], 4, feed_mode="rtl")
    for p, g in zip(prompts[:2], rtl):
        assert g == O.generate(model, p, 4, max_ctx=40, cfg=ocfg, feed_mode="rtl")
    assert dec.last_launches() > 0
    dec.shard_head(None, 1, 0)                   # leave: the unsharded head again
    assert dec.generate(prompts, 12) == plain6
    dec.close()


def test_profile_refused_on_sharded_handle():
    from bfp200 import BfpError, nccl_unique_id
    dec, _, _ = _small(5)
    dec.shard_head(nccl_unique_id(), 1, 0)
    with pytest.raises(BfpError):
        dec.profile_forward(1, 3)
    dec.close()


def _full_pair(devices):
    from bfp200 import BfpConfig, Decoder, synth
    img = synth.synthetic_image(BfpConfig(), seed=0)
    decs = []
    for d in devices:
        dec = Decoder(BfpConfig(MAX_CTX=48 + 256, max_seqs=8), device=d)
        dec.load_image(img)
        decs.append(dec)
    return decs


@pytest.mark.skipif("_n_gpus() < 2")
def test_two_gpu_group_golden_tokens():
    """2 GPUs in one process: rows [0, 24576) and [24576, 49152); cfg1 and
    cfg2 streams equal the reference simulator's golden tokens, a ragged
    batch equals the golden cfg3 sequences."""
    from bfp200 import generate_sharded, shard_group, synth
    decs = _full_pair([0, 1])
    shard_group(decs)
    p1, n1 = synth.config_prompts(1)
    assert generate_sharded(decs, p1, n1) == [load_tokens(1)[0]]
    p2, n2 = synth.config_prompts(2)
    assert generate_sharded(decs, p2, n2) == [load_tokens(2)[0]]
    p3, n3 = synth.config_prompts(3)
    gold = load_tokens(3)
    idx = sorted(gold)[:6]
    out = generate_sharded(decs, [p3[i] for i in idx], n3)
    for i, toks in zip(idx, out):
        assert toks == gold[i], i
    assert all(d.uncertified_steps() == 0 for d in decs)
    for d in decs:
        d.close()


def _rank_job(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bfp200 import BfpConfig, Decoder, synth
        from bfp200.dist import shard_head_distributed
        dec = Decoder(BfpConfig(MAX_CTX=48 + 256, max_seqs=8), device=rank)
        dec.load_image(synth.synthetic_image(BfpConfig(), seed=0))
        shard_head_distributed(dec)
        p1, n1 = synth.config_prompts(1)
        q.put((rank, dec.generate(p1, n1)))
        dec.shard_head(None, 1, 0)
        dec.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif("_n_gpus() < 2")
def test_two_process_sharded_head():
    """One process per GPU (the torchrun layout): the NCCL id travels over the
    process group, each rank's library joins its own communicator."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_job, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert out[0] == out[1] == [load_tokens(1)[0]]
