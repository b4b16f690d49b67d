"""Multi-process host logic of the sequence-parallel decode and the sharded
head's argmax exchange, as world_size-2 gloo process groups on CPU (the
decoder is replaced by a deterministic stand-in; GPU decoding is covered by
the -m gpu tests and bench.py under torchrun)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from bfp200 import dist as bd


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class FakeDecoder:
    """Token stream = prompt + (sum(prompt) + 7 k) % 1000 for k < n_gen."""

    def __init__(self):
        self.calls = []

    def generate(self, prompts, n_gen, feed_mode="sim"):
        self.calls.append(len(prompts))
        return [list(p) + [(sum(p) + 7 * k) % 1000 for k in range(n_gen)] for p in prompts]


def _expected(prompts, n_gen):
    return FakeDecoder().generate(prompts, n_gen)


def _worker(rank, world, port, fn, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, fn(rank, world)))
    finally:
        dist.destroy_process_group()


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def _prompts():
    rng = np.random.default_rng(3)
    return [rng.integers(0, 49152, size=int(n)).tolist() for n in rng.integers(8, 49, size=37)]


def _gen_job(rank, world):
    dec = FakeDecoder()
    toks = bd.generate_distributed(dec, _prompts(), 5)
    return toks, dec.calls


def _argmax_job(rank, world):
    # rank r owns vocabulary rows [lo, hi) of a fixed logit vector with ties
    rng = np.random.default_rng(11)
    logits = np.round(rng.standard_normal(1000) * 4) / 4          # many exact ties
    lo, hi = bd.shard_rows(len(logits), world, rank)
    part = logits[lo:hi]
    i = int(np.argmax(part))
    second = float(np.max(np.delete(part, i)))
    v, idx, sec = bd.combine_argmax(float(part[i]), lo + i, second)
    return v, idx, sec, float(np.max(logits)), int(np.argmax(logits))


def test_partition_balances_steps_and_covers():
    lens = [8, 48, 8, 48, 20, 30, 33, 9] * 4
    for world in (1, 2, 4, 8):
        blocks = bd.partition_sequences(lens, 128, world)
        assert blocks[0][0] == 0 and blocks[-1][1] == len(lens)
        assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
        steps = [sum(L + 128 for L in lens[lo:hi]) for lo, hi in blocks]
        assert max(steps) - min(steps) <= max(lens) + 128


def test_partition_more_ranks_than_sequences():
    blocks = bd.partition_sequences([10, 12], 4, 4)
    assert [hi - lo for lo, hi in blocks] and sum(hi - lo for lo, hi in blocks) == 2


def test_generate_distributed_gloo_world2():
    out = _run(_gen_job)
    want = _expected(_prompts(), 5)
    for rank in (0, 1):
        toks, calls = out[rank]
        assert toks == want                       # every rank holds all streams, in input order
        assert len(calls) == 1                    # one generate call per rank: its own block
    assert sum(out[r][1][0] for r in (0, 1)) == len(_prompts())


def test_sharded_argmax_gloo_world2():
    out = _run(_argmax_job)
    for rank in (0, 1):
        v, idx, sec, vmax, imax = out[rank]
        assert v == vmax and idx == imax           # lowest index among the maxima
        assert sec <= v


@pytest.mark.parametrize("parts,want", [
    ([(1.0, 5, 0.5), (1.0, 3, 0.9)], (1.0, 3, 1.0)),
    ([(2.0, 7, 1.0), (1.5, 2, 1.4)], (2.0, 7, 1.5)),
    ([(-np.inf, 2**62, -np.inf), (0.0, 9, -1.0)], (0.0, 9, -1.0)),
])
def test_reduce_argmax(parts, want):
    assert bd.reduce_argmax(parts) == want


def _leave_between_steps(rank, world):
    """Rank 1 takes step 0, then leaves the job before step 1; rank 0 must
    notice at its step-1 check, on the host, within the time limit."""
    import time
    bd.check_peers(0, timeout_s=30)
    if rank == 1:
        return "left"
    t0 = time.monotonic()
    try:
        bd.check_peers(1, timeout_s=2)
    except bd.PeerLost as e:
        return ("lost", str(e), time.monotonic() - t0)
    return ("not noticed",)


def test_rank_leaving_between_steps_is_noticed_on_the_host():
    out = _run(_leave_between_steps)
    assert out[1] == "left"
    assert out[0][0] == "lost", out
    assert "rank(s) 1" in out[0][1] and out[0][2] < 20
