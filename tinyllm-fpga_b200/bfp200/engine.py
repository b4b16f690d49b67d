"""Decoder: one libbfp200 handle on one GPU (the drop-in for the reference's
golden driver loop, rtl/vc707/host/gen_smollm_blockfp_full.py:406-449, fed by
the packed image and ROM files of the packers)."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from ._lib import arr, check, ptr
from .config import BfpConfig
from .image import ROM_KINDS, read_roms

FEED_MODES = {"sim": 0, "rtl": 1}


class Decoder:
    def __init__(self, cfg: BfpConfig | None = None, device: int = 0):
        self.cfg = cfg or BfpConfig()
        self.device = device
        self._h = C.c_void_p()
        self._rom_prompt_len = 0
        check(_lib.lib().bfp200_open(C.byref(self.cfg.to_c()), int(device), C.byref(self._h)))

    # -- lifecycle ------------------------------------------------------------
    def close(self):
        if self._h:
            _lib.lib().bfp200_close(self._h)
            self._h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    # -- loading ----------------------------------------------------------------
    def load_image(self, image):
        """<PREFIX>DDR3.bin contents (bytes) or a path to it."""
        if isinstance(image, (str, os.PathLike)):
            with open(image, "rb") as f:
                image = f.read()
        buf = np.frombuffer(image, dtype=np.uint8)
        check(_lib.lib().bfp200_load_image(self._h, buf.ctypes.data, buf.size))

    def load_rom(self, kind: int, entries):
        e = arr(entries, np.uint16)
        check(_lib.lib().bfp200_load_rom(self._h, int(kind), ptr(e), e.size))
        if int(kind) == 6:
            self._rom_prompt_len = int(e.size)

    def load_roms(self, directory, prefix="lbfp_full_"):
        """The client's load-roms (bfp_client.cpp:1381-1437) from a release dir."""
        for kind, entries in read_roms(directory, prefix).items():
            self.load_rom(kind, entries)

    # -- decode -----------------------------------------------------------------
    def generate(self, prompts=None, n_gen=None, feed_mode="sim"):
        """prompts: list of token-id lists (None: the loaded PROMPT ROM).
        Returns one list per sequence: prompt + n_gen ids (sim) or one argmax
        per step (rtl)."""
        n_gen = self.cfg.N_GEN if n_gen is None else int(n_gen)
        mode = FEED_MODES[feed_mode]
        if prompts is None:
            if not self._rom_prompt_len:
                raise ValueError("no prompt given and no PROMPT ROM loaded")
            out = np.empty(self._rom_prompt_len + n_gen, np.int32)
            check(_lib.lib().bfp200_generate(self._h, None, None, 1, n_gen, mode, ptr(out)))
            return [out.tolist()]
        lens = arr([len(p) for p in prompts], np.int32)
        ids = arr(np.concatenate([np.asarray(p, dtype=np.int64) for p in prompts]), np.int32)
        out = np.empty(int(lens.sum()) + len(prompts) * n_gen, np.int32)
        check(_lib.lib().bfp200_generate(self._h, ptr(ids), ptr(lens), len(prompts), n_gen, mode, ptr(out)))
        res, o = [], 0
        for L in lens:
            res.append(out[o:o + L + n_gen].tolist())
            o += L + n_gen
        return res

    def generate_sampled(self, prompts, n_gen, temperature, top_k=0, seed=1):
        """Temperature / top-k sampling like the reference emulator
        (sim_rtl_fp_hw.py:204-216, env TEMP / TOPK / SEED): sequence s uses
        np.random.seed(seed + s)'s stream.  temperature <= 0 is greedy.
        Returns prompt + n_gen ids per sequence."""
        lens = arr([len(p) for p in prompts], np.int32)
        ids = arr(np.concatenate([np.asarray(p, dtype=np.int64) for p in prompts]), np.int32)
        out = np.empty(int(lens.sum()) + len(prompts) * n_gen, np.int32)
        check(_lib.lib().bfp200_generate_sampled(self._h, ptr(ids), ptr(lens), len(prompts), int(n_gen),
                                                 float(temperature), int(top_k), int(seed) & 0xFFFFFFFF, ptr(out)))
        res, o = [], 0
        for L in lens:
            res.append(out[o:o + L + n_gen].tolist())
            o += L + n_gen
        return res

    def uncertified_steps(self) -> int:
        n = C.c_longlong()
        check(_lib.lib().bfp200_uncertified_steps(self._h, C.byref(n)))
        return n.value

    def last_timing(self):
        a, b = C.c_double(), C.c_double()
        check(_lib.lib().bfp200_last_timing(self._h, C.byref(a), C.byref(b)))
        return {"prefill_ms": a.value, "decode_ms": b.value}

    def last_launches(self):
        """Kernel launches of the last generate call (counted by the library)."""
        n = C.c_longlong()
        check(_lib.lib().bfp200_last_launches(self._h, C.byref(n)))
        return n.value

    PROFILE_KINDS = ("embed", "rmsnorm", "mm_qkv", "rope_kv", "attention", "mm_o", "mm_gu", "mm_d", "head_prep",
                     "head_logits", "head_reduce")

    def profile_forward(self, ncols, pos):
        """Per-kernel-kind device time (ms) and launch counts of one forward
        pass of ncols columns at position pos (serialised launches)."""
        ms = np.zeros(len(self.PROFILE_KINDS), np.float64)
        n = np.zeros(len(self.PROFILE_KINDS), np.int32)
        check(_lib.lib().bfp200_profile_forward(self._h, int(ncols), int(pos), ptr(ms), ptr(n)))
        return {k: (round(float(a), 4), int(b)) for k, a, b in zip(self.PROFILE_KINDS, ms, n)}

    def shard_head(self, uid, nranks, rank):
        """Joins rank `rank` of an `nranks`-way vocabulary-sharded head
        (every rank passes the same `uid` from nccl_unique_id(); blocks until
        all ranks joined).  uid=None leaves sharding; a one-rank group runs
        the sharded head path over the whole vocabulary.  Afterwards
        generate() must be called on every rank with the same arguments."""
        if uid is None:
            check(_lib.lib().bfp200_head_shard(self._h, None, 1, 0))
            return
        buf = np.frombuffer(bytes(uid), np.uint8).copy()
        assert buf.size == _lib.NCCL_ID_BYTES, "NCCL unique id must be 128 bytes"
        check(_lib.lib().bfp200_head_shard(self._h, ptr(buf), int(nranks), int(rank)))

    def time_matmuls(self, ncols, reps=20):
        """Device time (ms) of one decode step's matvecs (4 per layer, all
        layers) at ncols columns, replayed from a CUDA graph `reps` times
        between events; returns (ms per step, launches per step)."""
        ms, n = C.c_double(), C.c_int()
        check(_lib.lib().bfp200_time_matmuls(self._h, int(ncols), int(reps), C.byref(ms), C.byref(n)))
        return ms.value, n.value

    # -- one layer (fwd_layer, :261-293) ----------------------------------------
    def stage_dims(self):
        d = np.empty(_lib.NSTAGES, np.int32)
        check(_lib.lib().bfp200_stage_dims(self._h, ptr(d)))
        return d

    def fwd_layer(self, layer, h, pos, k_cache, v_cache, kv_pos=None, stages=False, decode_kernels=False):
        """h (ncols, D) grid doubles; k_cache/v_cache (ncols, max_ctx, H_KV, HD)
        float64, updated in place at kv_pos.  Returns h_out (and a list of
        per-stage dicts if stages).  decode_kernels: run the kernels a decode
        step uses for 1..4 columns (bfp200_fwd_layer_decode) instead of the
        general batched path."""
        h = arr(h, np.float64)
        one = h.ndim == 1
        h2 = h.reshape(1, -1) if one else h
        ncols = h2.shape[0]
        pos_a = arr(np.broadcast_to(np.asarray(pos), (ncols,)), np.int32)
        kvp = pos_a if kv_pos is None else arr(np.broadcast_to(np.asarray(kv_pos), (ncols,)), np.int32)
        kc = k_cache if k_cache.ndim == 4 else k_cache[None]
        vc = v_cache if v_cache.ndim == 4 else v_cache[None]
        if not (kc.flags["C_CONTIGUOUS"] and kc.dtype == np.float64 and vc.flags["C_CONTIGUOUS"]
                and vc.dtype == np.float64):
            raise ValueError("k_cache / v_cache must be C-contiguous float64")
        out = np.empty_like(h2)
        st = None
        if stages:
            dims = self.stage_dims()
            st = np.empty(ncols * int(dims.sum()), np.float64)
        fn = _lib.lib().bfp200_fwd_layer_decode if decode_kernels else _lib.lib().bfp200_fwd_layer
        check(fn(self._h, int(layer), ptr(h2), ptr(pos_a), ptr(kvp), ncols, ptr(kc), ptr(vc), kc.shape[1], ptr(out),
                 ptr(st)))
        res = out[0] if one else out
        if not stages:
            return res
        names = ["n1", "q", "k", "v", "attn", "o", "h1", "n2", "g", "u", "mlp", "d"]
        per = []
        o = 0
        for _ in range(ncols):
            dct = {}
            for nm, dd in zip(names, dims):
                dct[nm] = st[o:o + dd].copy()
                o += dd
            per.append(dct)
        return res, per


def _handles(decoders):
    return (C.c_void_p * len(decoders))(*[d.handle.value for d in decoders])


def _run_many(fn, decoders, prompts, n_gen, feed_mode):
    lens = arr([len(p) for p in prompts], np.int32)
    ids = arr(np.concatenate([np.asarray(p, dtype=np.int64) for p in prompts]), np.int32)
    out = np.empty(int(lens.sum()) + len(prompts) * n_gen, np.int32)
    check(fn(C.cast(_handles(decoders), C.c_void_p), len(decoders), ptr(ids), ptr(lens), len(prompts), int(n_gen),
             FEED_MODES[feed_mode], ptr(out)))
    res, o = [], 0
    for L in lens:
        res.append(out[o:o + L + n_gen].tolist())
        o += L + n_gen
    return res


def generate_multi(decoders, prompts, n_gen, feed_mode="sim"):
    """Sequences split into contiguous blocks over the decoders (one per GPU),
    run concurrently, no collectives (bfp200_generate_multi)."""
    return _run_many(_lib.lib().bfp200_generate_multi, decoders, prompts, n_gen, feed_mode)


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id for Decoder.shard_head (made by one rank)."""
    buf = np.zeros(_lib.NCCL_ID_BYTES, np.uint8)
    check(_lib.lib().bfp200_nccl_unique_id(ptr(buf)))
    return buf.tobytes()


def shard_group(decoders):
    """Shards the head's vocabulary over decoders on distinct GPUs of this
    process (rank = position in the list; one NCCL communicator)."""
    check(_lib.lib().bfp200_head_shard_group(C.cast(_handles(decoders), C.c_void_p), len(decoders)))


def generate_sharded(decoders, prompts, n_gen, feed_mode="sim"):
    """Every decoder of a sharded group decodes all `prompts` (single-stream
    latency: the layers run redundantly, the head is split by vocabulary
    rows and the argmax exchanged by NCCL); returns the common tokens."""
    return _run_many(_lib.lib().bfp200_generate_sharded, decoders, prompts, n_gen, feed_mode)


__all__ = ["Decoder", "generate_multi", "generate_sharded", "shard_group", "nccl_unique_id", "ROM_KINDS"]
