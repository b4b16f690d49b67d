"""Shared helpers for the tests (fixtures, cached models)."""
from __future__ import annotations

import functools
import hashlib
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_path(name):
    return os.path.join(GOLDEN, name)


@functools.lru_cache(maxsize=None)
def manifest():
    with open(golden_path("manifest.json")) as f:
        return json.load(f)


def load_tokens(cfg_id):
    """Golden token lists of a config: {seq index: tokens} (reference simulator)."""
    out = {}
    for fn in sorted(os.listdir(GOLDEN)):
        if fn.startswith(f"tokens_cfg{cfg_id}") and fn.endswith(".json"):
            with open(golden_path(fn)) as f:
                for k, v in json.load(f).items():
                    out[int(k)] = v["tokens"]
    return out


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@functools.lru_cache(maxsize=None)
def oracle_model(seed=0):
    from oracle import synth
    m = synth.make_model(seed)
    m.cache_float_weights()
    return m


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def load_sampled():
    """Sampled streams of the reference emulator (tests/golden/sampled.json):
    [{temperature, top_k, seed, n_gen, tokens}] on the cfg1 prompt."""
    with open(golden_path("sampled.json")) as f:
        return json.load(f)
