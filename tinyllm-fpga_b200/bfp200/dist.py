"""Multi-process (one process per GPU) decode over torch.distributed.

Independent sequences shard naturally: every rank holds a full replica of
the image and decodes a contiguous block of the sequences, with no
collective on the data path.  Blocks are balanced by total steps (prompt
length + n_gen), the rule bfp200_generate_multi uses inside one process.
The ranks meet only to gather the token streams at the end.

For single-stream latency the head can be split by vocabulary rows across
ranks; each rank reduces its rows to (max logit, lowest index, runner-up)
and the ranks combine those with one all-gather of 24 bytes per rank
(`combine_argmax`).  The combination keeps the lowest index on ties, so the
result is the argmax of the whole vocabulary (np.argmax semantics,
gen_smollm_blockfp_full.py:439-440).
"""
from __future__ import annotations

import bisect

import numpy as np


def partition_sequences(prompt_lens, n_gen, world):
    """Contiguous blocks [lo, hi) of the sequences for `world` ranks,
    balanced by total steps (prompt length + n_gen)."""
    n = len(prompt_lens)
    cum = [0]
    for L in prompt_lens:
        cum.append(cum[-1] + int(L) + int(n_gen))
    bounds = [0]
    for d in range(1, world):
        target = cum[n] * d // world
        b = bisect.bisect_left(cum, target)
        bounds.append(max(b, bounds[-1]))
    bounds.append(n)
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def _gather_objects(obj, world, group=None):
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj, group=group)
    return out


def generate_distributed(decoder, prompts, n_gen, feed_mode="sim", group=None):
    """Decodes this rank's block of `prompts` on its decoder and returns the
    token streams of all sequences (on every rank), in input order.

    `decoder` is anything with generate(prompts, n_gen, feed_mode) -> list
    of token lists (a bfp200.Decoder on the rank's GPU)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    blocks = partition_sequences([len(p) for p in prompts], n_gen, world)
    lo, hi = blocks[rank]
    mine = decoder.generate(prompts[lo:hi], n_gen, feed_mode=feed_mode) if hi > lo else []
    parts = _gather_objects((lo, hi, mine), world, group)
    out = [None] * len(prompts)
    for lo_r, hi_r, toks in parts:
        out[lo_r:hi_r] = toks
    return out


def _better(v, i, bv, bi):
    """(v, i) beats (bv, bi): larger logit, or equal logit with a lower index."""
    return v > bv or (v == bv and i < bi)


def reduce_argmax(parts):
    """Combines (best value, best index, runner-up value) triples of disjoint
    vocabulary shards into the global triple (lowest index on ties)."""
    best, bidx, sec = -np.inf, np.iinfo(np.int64).max, -np.inf
    for v, i, s in parts:
        v, i, s = float(v), int(i), float(s)
        if _better(v, i, best, bidx):
            sec = max(sec, best)
            best, bidx = v, i
        else:
            sec = max(sec, v)
        sec = max(sec, s)
    return best, bidx, sec


def combine_argmax(value, index, second, group=None):
    """All-gathers every rank's shard triple (24 bytes) and returns the
    global (value, index, runner-up) on every rank.  Works on the nccl
    backend (CUDA tensors) and on gloo (CPU)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    dev = torch.device("cuda", torch.cuda.current_device()) \
        if dist.get_backend(group) == "nccl" else torch.device("cpu")
    mine = torch.tensor([float(value), float(index), float(second)], dtype=torch.float64, device=dev)
    allv = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(allv, mine, group=group)
    parts = [(t[0].item(), int(t[1].item()), t[2].item()) for t in allv]
    return reduce_argmax(parts)


def shard_rows(vocab, world, rank):
    """Contiguous vocabulary rows [lo, hi) of `rank` for the sharded head
    (the split libbfp200's sharded head uses)."""
    return rank * vocab // world, (rank + 1) * vocab // world


def shard_head_distributed(decoder, group=None):
    """Joins this rank's decoder to a vocabulary-sharded head over the
    process group: rank 0 makes the NCCL id, the group broadcasts it, every
    rank joins the library's own communicator.  Afterwards every rank calls
    decoder.generate() with the same prompts and gets the same tokens; the
    argmax exchange runs inside the library's decode graph (one all-gather
    of 32 bytes per sequence and rank per step)."""
    import torch.distributed as dist
    from .engine import nccl_unique_id
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    box = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    decoder.shard_head(box[0], world, rank)


class PeerLost(RuntimeError):
    """A rank of the group did not reach the same step within the time limit."""


def _group_store(group=None):
    import torch.distributed as dist
    if group is None:
        from torch.distributed import distributed_c10d as c10d
        return c10d._get_default_store()
    raise ValueError("check_peers: pass store= for a non-default group")


def check_peers(step, timeout_s=10.0, group=None, store=None, prefix="bfp200/alive"):
    """Host-side liveness check between decode calls of a sharded head.

    Every rank posts `<prefix>/<step>/<rank>` to the process group's store and
    waits, at most `timeout_s`, for the keys of every other rank at the same
    step.  A rank that has left the job (exited, crashed, or stopped decoding)
    is noticed here, on the host and before this rank launches work that
    holds a collective, instead of by an exchange on the GPU that would wait
    for it.  Raises PeerLost naming the missing ranks."""
    import datetime
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    st = store if store is not None else _group_store(group)
    st.set(f"{prefix}/{step}/{rank}", "1")
    others = [f"{prefix}/{step}/{r}" for r in range(world) if r != rank]
    if not others:
        return
    try:
        st.wait(others, datetime.timedelta(seconds=timeout_s))
    except Exception as e:        # the store raises on its time limit
        missing = [k.rsplit("/", 1)[1] for k in others if not st.check([k])]
        raise PeerLost(f"step {step}: rank(s) {', '.join(missing) or '?'} did not arrive within {timeout_s} s") from e


__all__ = ["partition_sequences", "generate_distributed", "reduce_argmax", "combine_argmax", "shard_rows",
           "shard_head_distributed", "check_peers", "PeerLost"]
