#!/usr/bin/env python3
"""Benchmark of the BFP SmolLM2-135M greedy decode path on B200.

Metric: BFP decode tok/s at bs1 and bs256, with the fraction
of the HBM roofline.  One JSON line on rank 0.

Workload (config.workload): configs[1] = "cfg2": synthetic SmolLM2-135M
(seeded random weights, BFP fixed points, packed like the reference), a
48-token prompt, 256 greedy tokens, KV up to 304 positions, batch 1.  A step
is one full generate call (prefill + 256 decode steps).  ``value`` =
generated tokens/s over all ranks (each rank decodes its own replica: bs1
does not shard, so N GPUs run N independent streams -- weak scaling).
The same line carries ``bs256``: configs[2] = "cfg3", 256 ragged sequences
x 128 tokens, sequences split over the ranks with no collectives (strong
scaling), and at N > 1 ``bs256_weak``: every rank serves the whole cfg3
batch (256 sequences per GPU, 256 N in all -- weak scaling).

Further keys of the final line: ``roofline`` (the bs1 decode's dominant
kernel, the per-layer attention block, against the measured HBM copy
bandwidth, with the gate/up and down GEMV figures in ``roofline.gemv``),
``path_roofline_frac`` (weight + KV bytes
per token over the decode time), ``bs256`` (tok/s, ms per step, and the
batched tensor-core matvecs' roofline), ``cpu_baseline`` (the oracle port on
all usable host cores, rank 0 at N = 1) and, at N > 1, ``sharded_head``
(single-stream decode with the vocabulary-sharded head; ``--no-sharded-head``
skips it).  The bulky sections -- ``cfg5`` (per-kernel times at batch 64 / KV
2047), ``cfg4`` (the isolated matvec over the model's weight shapes x batch
1 .. 1024) and ``kernel_profile_ms`` -- go on a preceding line
``{"detail": ...}``, so the last line stays short.

``--impl reference`` times the reference algorithm on the host cores (the
numpy restatement under oracle/, since the reference is Python that cannot
be installed on the GPU box) with the same metric and unit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "tinyllm-fpga_b200"))

import numpy as np  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---------------------------------------------------------------------------
# algorithmic bytes (packed BFP: 2 B mantissa + 1/16 B exponent per element)
# ---------------------------------------------------------------------------
def weight_bytes_per_token(cfg):
    kvd = cfg.H_KV * cfg.HD
    per_layer = 0
    for dout, din in ((cfg.D, cfg.D), (kvd, cfg.D), (kvd, cfg.D), (cfg.D, cfg.D), (cfg.FFN, cfg.D),
                      (cfg.FFN, cfg.D), (cfg.D, cfg.FFN)):
        per_layer += dout * din * 2 + dout * din // 16
    head = cfg.VOCAB * cfg.D * 2 + cfg.VOCAB * cfg.D // 16
    return cfg.NL * per_layer, head


def kv_bytes_per_position(cfg):
    return cfg.NL * 2 * cfg.H_KV * cfg.HD * 2 + cfg.NL * 2 * cfg.H_KV * cfg.HD // 16   # 23,760 B


def attn_block_bytes(cfg, pos):
    """Algorithmic bytes of one bfp_attn_block_kernel launch (one layer, one
    column, KV position pos): Q/K/V and O weights (int16 mantissas + int8
    exponents per 16), the f64 gamma, h in and h1 out (BFP), the cached K/V
    rows 0..pos-1 read and row pos written."""
    kvd = cfg.H_KV * cfg.HD
    w = (cfg.D + 2 * kvd) * cfg.D + cfg.D * cfg.D
    act = 2 * (cfg.D * 2 + cfg.D // 16)
    kv_row = kv_bytes_per_position(cfg) // cfg.NL               # 792 B per layer and position
    return w * 2 + w // 16 + cfg.D * 8 + act + kv_row * (pos + 1)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for i, nm in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


# ---------------------------------------------------------------------------
def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ["BFP200_DEVICE"] = str(local)       # the op-level helpers' device (bfp200.ops)
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------
def run_ours(args, world, rank, local):
    from bfp200 import BfpConfig, Decoder, synth, _lib

    pk, pk_kind = peaks()
    # the CPU baseline runs first, before this process touches the GPU, so its
    # worker pool can fork (rank 0 at N = 1 only)
    cpu = cpu_baselines(args) if (rank == 0 and world == 1 and not args.no_cpu) else None
    cfg2 = BfpConfig(MAX_CTX=48 + 256, max_seqs=256)
    t0 = time.time()
    img = synth.synthetic_image(BfpConfig(), seed=0)
    build_s = time.time() - t0
    dec = Decoder(cfg2, device=local)
    dec.load_image(img)
    prompts2, ngen2 = synth.config_prompts(2)
    ngen2 = args.n_gen
    prompts3, ngen3 = synth.config_prompts(3)
    # contiguous blocks balanced by total steps (bfp200.dist), one per rank
    from bfp200 import dist as bd
    lo, hi = bd.partition_sequences([len(p) for p in prompts3], ngen3, world)[rank]
    part3 = prompts3[lo:hi]

    # ---- cfg2 (bs1): device time of each generate (events on the library's stream)
    for _ in range(args.warmup):
        dec.generate(prompts2, ngen2)
    barrier(world)
    with ClockSampler(local) as clk:
        dev_ms = []
        launches = 0
        for _ in range(args.steps):
            dec.generate(prompts2, ngen2)
            t = dec.last_timing()
            dev_ms.append(t["prefill_ms"] + t["decode_ms"])
            launches += dec.last_launches()
        # e2e through the public API: host prompt ids in, host tokens out,
        # H2D/D2H inside the timed region (synchronous call, host clock)
        e2e_s = []
        for _ in range(max(1, args.steps // 2)):
            ts = time.perf_counter()
            out = dec.generate(prompts2, ngen2)
            e2e_s.append(time.perf_counter() - ts)
    barrier(world)
    uncert = dec.uncertified_steps()
    step_ms = max_over_ranks(statistics.mean(dev_ms), world)
    e2e_step_s = max_over_ranks(statistics.mean(e2e_s), world)
    tokens_per_step = ngen2 * world
    value = tokens_per_step / (step_ms / 1e3)
    e2e = tokens_per_step / e2e_step_s
    last = dec.last_timing()
    decode_tok_ms = last["decode_ms"] / ngen2

    # ---- roofline of the dominant kernel of the bs1 decode: the attention
    # block (RMSNorm, Q/K/V, RoPE, KV write, attention, O, residual; one
    # launch per layer, ~57% of a token's kernel time).  Its launch duration
    # is measured with CUDA events around each launch of one serialised
    # forward at KV position 176 (the cfg2 stream's mean); the other kernels
    # of that forward give the gate/up and down GEMV figures.
    wbytes, hbytes = weight_bytes_per_token(cfg2)
    peak = pk["hbm_gbs"]
    prof1 = dec.profile_forward(1, 176)
    a_ms, a_n = prof1["attention"]
    a_us = a_ms * 1e3 / max(1, a_n)
    a_bytes = attn_block_bytes(cfg2, 176)
    a_gbs = a_bytes / (a_us * 1e-6) / 1e9
    kvd = cfg2.H_KV * cfg2.HD
    gemv = {}
    for kind, rows, din in (("mm_gu", 2 * cfg2.FFN, cfg2.D), ("mm_d", cfg2.D, cfg2.FFN)):
        ms_k, n_k = prof1[kind]
        if n_k:
            us_k = ms_k * 1e3 / n_k
            b_k = rows * din * 2 + rows * din // 16
            gemv[kind] = {"us_per_launch": round(us_k, 3), "achieved_gbs": round(b_k / (us_k * 1e-6) / 1e9, 1),
                          "frac": round(b_k / (us_k * 1e-6) / 1e9 / peak, 4)}
    # the matvec engine alone: one token's 120 matvecs (Q/K/V, O, gate/up,
    # down) on the GEMV kernel, replayed from a graph between events
    mm_ms, mm_n = dec.time_matmuls(1, args.mm_reps)
    gemv["engine_120_matvecs"] = {"ms_per_token": round(mm_ms, 4), "achieved_gbs": round(wbytes / (mm_ms / 1e3) / 1e9, 1),
                                  "frac": round(wbytes / (mm_ms / 1e3) / 1e9 / peak, 4)}
    roof = {"kernel": "bfp_attn_block_kernel (RMSNorm + Q/K/V + RoPE + KV + attention + O + residual, bs1)",
            "bound": "hbm", "achieved": round(a_gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(a_gbs / peak, 4),
            "traffic": ATTN_BLOCK_TRAFFIC_POS176,
            "traffic_unit": "bytes per launch at KV position 176 (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
            "algorithmic_bytes": a_bytes, "peak_kind": pk_kind, "launches_per_token": a_n,
            "us_per_launch": round(a_us, 3), "timing": "CUDA events around each launch of a serialised forward, KV 176",
            "gemv": gemv}
    # whole-path roofline: weights + KV per token over the decode time
    mean_pos = 48 + ngen2 / 2
    path_bytes = wbytes + hbytes + kv_bytes_per_position(cfg2) * (mean_pos + 1)
    path_frac = path_bytes / (decode_tok_ms / 1e3) / 1e9 / peak

    # ---- bs256 (cfg3), sequences split over ranks
    bs256 = None
    for _ in range(0 if args.no_bs256 else max(1, args.warmup // 3)):
        dec.generate(part3, ngen3)
    if not args.no_bs256:
        barrier(world)
        b_ms = []
        for _ in range(max(1, args.steps // 4)):
            dec.generate(part3, ngen3)
            t = dec.last_timing()
            b_ms.append(t["prefill_ms"] + t["decode_ms"])
        barrier(world)
        b_step = max_over_ranks(statistics.mean(b_ms), world)
        bs256 = {"metric": "BFP decode tok/s (bs256, cfg3)",
                 "value": round(len(prompts3) * ngen3 / (b_step / 1e3), 1), "unit": "tok/s",
                 "ms_per_step": round(b_step, 3), "sequences": len(prompts3), "n_gen": ngen3,
                 "scaling": "strong", "uncertified_steps": dec.uncertified_steps()}
        if part3:
            bs256["roofline"] = batched_roofline(dec, len(part3), max(1, args.mm_reps // 5), pk, pk_kind)

    # ---- bs256, weak scaling: every rank serves all 256 cfg3 sequences
    bs256_weak = None
    if world > 1 and not args.no_bs256:
        dec.generate(prompts3, ngen3)                   # warm-up (graphs at 256 columns)
        barrier(world)
        w_ms = []
        for _ in range(max(1, args.steps // 4)):
            dec.generate(prompts3, ngen3)
            t = dec.last_timing()
            w_ms.append(t["prefill_ms"] + t["decode_ms"])
        barrier(world)
        w_step = max_over_ranks(statistics.mean(w_ms), world)
        bs256_weak = {"value": round(world * len(prompts3) * ngen3 / (w_step / 1e3), 1), "unit": "tok/s",
                      "ms_per_step": round(w_step, 3), "sequences_per_gpu": len(prompts3), "scaling": "weak"}

    profile = {"bs1_pos176": prof1}
    if not args.no_bs256 and part3:
        profile["bs256_pos100"] = dec.profile_forward(len(part3), 100)
    sharded = None
    if world > 1 and not args.no_sharded_head:
        sharded = sharded_head_run(dec, prompts2, ngen2, args, world, decode_tok_ms)
    dec.close()
    cfg5 = None
    if not args.no_cfg5 and rank == 0:                  # per-GPU kernel profile: rank 0
        # cfg5: leaf ops and attention at batch 64, KV length 2048 (serialised
        # per-kernel times of one forward pass at position 2047)
        d5 = Decoder(BfpConfig(MAX_CTX=2048, max_seqs=64), device=local)
        d5.load_image(img)
        cfg5 = {"batch": 64, "pos": 2047, "kernel_ms": d5.profile_forward(64, 2047)}
        d5.close()
        # attention's HBM rate: the K / V rows 0..2047 of every sequence and
        # layer (mantissas + tile exponents) per 30 launches, against the
        # measured copy bandwidth
        att_ms, att_n = cfg5["kernel_ms"]["attention"]
        att_bytes = 64 * 2048 * kv_bytes_per_position(BfpConfig())
        if att_ms > 0:
            gbs = att_bytes / (att_ms / 1e3) / 1e9
            cfg5["attention_hbm"] = {"kernel": "attention_long_kernel", "bytes_per_forward": att_bytes,
                                     "achieved_gbs": round(gbs, 1), "frac": round(gbs / pk["hbm_gbs"], 4),
                                     "peak_kind": pk_kind}
    del img
    cfg4 = None if (args.no_cfg4 or rank != 0) else cfg4_sweep(args.cfg4_batches, pk)   # per-GPU: rank 0
    res = {
        "metric": "BFP decode tok/s (bs1, cfg2)", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int16-BFP/int64/f64", "data": "synthetic",
        "config": {"workload": "cfg2: 48-token prompt + 256 greedy tokens, bs1, KV<=304",
                   "model": "SmolLM2-135M arch, seeded random BFP weights", "global_batch": world,
                   "seq_len": 48 + 256, "parallelism": f"replicas{world}",
                   "l2": "inputs larger than L2 (277 MB of weights streamed per token)"},
        "decode_us_per_token": round(decode_tok_ms * 1e3, 2),
        "prefill_ms": round(last["prefill_ms"], 3),
        "path_roofline_frac": round(path_frac, 4),
        "roofline": roof,
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 48 * 4 + 4,
                "d2h_bytes_per_step": (48 + ngen2) * 4 + 8},
        "gpu_launches": int(sum_over_ranks(launches, world)),
        "bs256": bs256,
        "bs256_weak": bs256_weak,
        "sharded_head": sharded,
        "uncertified_steps": uncert,
        "image_build_s": round(build_s, 1),
        "clocks": clk.summary(),
    }
    if cpu is not None:
        res["cpu_baseline"] = cpu["cfg2"]
        if bs256 is not None:
            bs256["cpu_baseline"] = cpu["cfg3"]
    detail = {"kernel_profile_ms": profile, "cfg5": cfg5, "cfg4": cfg4}
    return res, detail


CFG4_SHAPES = ((576, 576), (192, 576), (1536, 576), (576, 1536), (49152, 576))


def cfg4_sweep(batches, pk):
    """configs[3] (cfg4): the isolated BFP matvec over the model's weight
    shapes (D_out x D_in), mantissas uniform int16, tile exponents uniform in
    [-20, 4], inputs tile_quantize(N(0,1)), seed 4; device time per call
    (bfp200_matvec_timed, weights and inputs resident, 10 repetitions) of the
    kernel a decode step uses at that column count (small-batch GEMV at 1..4,
    dp2a matmul at 5..15, tensor cores from 16), with its roofline fraction:
    HBM (weight + activation bytes over the measured copy bandwidth) up to 8
    columns, tensor (int16 MACs as 4 int8 limb MACs over twice the measured
    bf16 rate) from 64."""
    from bfp200 import ops
    rng = np.random.default_rng(4)
    out = {}
    for dout, din in CFG4_SHAPES:
        nt = din // 16
        W_m = rng.integers(-32768, 32768, size=(dout, nt, 16), dtype=np.int64).astype(np.int16)
        W_e = rng.integers(-20, 5, size=(dout, nt)).astype(np.int8)
        row = {}
        for b in batches:
            xm, xe = ops.tile_quantize(rng.standard_normal(b * din))
            _, _, ms = ops.matvec_timed(xm.reshape(b, nt, 16), xe.reshape(b, nt), W_m, W_e, reps=10)
            s = ms / 1e3
            kern = ("bfp_gemv_small_kernel" if b <= 4 else "bfp_matmul_kernel (dp2a)" if b < 16
                    else "tc_matmul_kernel (tcgen05)")
            byts = dout * din * 2.0625 + b * din * 2.0625 + b * dout * 2.0625
            ent = {"kernel": kern, "us": round(ms * 1e3, 2), "weight_gbs": round(dout * din * 2.0625 / s / 1e9, 1),
                   "tmacs": round(dout * din * b / s / 1e12, 3)}
            if b <= 8:
                ent["hbm_frac"] = round(byts / s / 1e9 / pk["hbm_gbs"], 4)
            if b >= 64:
                ent["tensor_frac"] = round(dout * din * b * 4 * 2 / s / 1e12 / (2 * pk["bf16_tflops"]), 5)
            row[str(b)] = ent
        out[f"{dout}x{din}"] = row
    return out


def sharded_head_run(dec, prompts, n_gen, args, world, replica_tok_ms):
    """cfg5's single-stream mode: the cfg2 stream decoded by all ranks with
    the head split by vocabulary rows and the argmax exchanged by NCCL inside
    the library's decode graph.  Device time per generated token, max over
    ranks, next to the unsharded (replica) time."""
    from bfp200.dist import check_peers, shard_head_distributed
    err = None
    ms = []
    try:
        shard_head_distributed(dec)
        nw, nt = max(1, args.warmup // 2), max(1, args.steps // 2)
        for i in range(nw + nt):
            check_peers(f"sharded{i}", timeout_s=60)    # a rank that left is noticed here, before the exchange
            dec.generate(prompts, n_gen)
            if i >= nw:
                ms.append(dec.last_timing()["decode_ms"] / n_gen)
    except Exception as e:            # the library's bounded waits end a stalled exchange with an error
        err = f"{type(e).__name__}: {e}"[:200]
    try:
        dec.shard_head(None, 1, 0)
    except Exception as e:
        err = err or f"{type(e).__name__}: {e}"[:200]
    # every rank takes the same collective steps, failed or not
    tok_ms = max_over_ranks(statistics.mean(ms) if ms and err is None else float("inf"), world)
    if err is not None or tok_ms == float("inf"):
        return {"ranks": world, "error": err or "another rank failed"}
    return {"ranks": world, "decode_us_per_token": round(tok_ms * 1e3, 2),
            "replica_decode_us_per_token": round(replica_tok_ms * 1e3, 2),
            "vocab_rows_per_rank": 49152 // world, "exchange": "NCCL all-gather of 32 B per rank per step"}


# DRAM bytes (read + write) of one bfp_attn_block_kernel launch at KV position
# 176, the mean of three launches of an ncu capture of a serialised forward
# (dram__bytes_read.sum + dram__bytes_write.sum, writes 0); algorithmic bytes
# at that position: 1,971,936 (the excess is about the kernel's code).
ATTN_BLOCK_TRAFFIC_POS176 = 2_064_896
# DRAM bytes of one layer's four batched matvecs at 256 columns (Q/K/V, O,
# gate/up, down; reads only, the outputs stay in L2) from one ncu capture,
# times 30 layers
TC_STEP_TRAFFIC_256 = 30 * (1_780_480 + 1_568_768 + 4_615_424 + 3_517_440)

LAYER_MACS = 106_168_320      # int16 MACs of one token's 4 x 30 layer matvecs (head excluded)


def batched_roofline(dec, ncols, reps, pk, pk_kind):
    """The batched matvecs of one decode step at this rank's column count:
    tcgen05 kind::i8 (>= 16 columns) or the dp2a kernel.  Algorithmic work =
    the int16 MACs, counted as 4 int8 limb MACs each (2 ops per MAC), against
    the int8 dense peak taken as twice the measured bf16 GEMM rate (the
    nominal int8 : bf16 ratio of B200).  ``traffic``: DRAM bytes of the
    step's 120 launches from one ncu capture at 256 columns (cold cache:
    weight records + input columns), reported at that column count only."""
    ms, n = dec.time_matmuls(ncols, reps)
    tops = LAYER_MACS * ncols * 4 * 2 / (ms / 1e3) / 1e12
    peak = 2 * pk["bf16_tflops"]
    out = {"kernel": "tc_matmul_kernel (tcgen05 kind::i8 limbs)" if ncols >= 16 else "bfp_matmul_kernel (dp2a)",
           "bound": "tensor", "achieved": round(tops, 2), "peak": round(peak, 1), "unit": "TOPS (int8)",
           "frac": round(tops / peak, 5), "traffic": None, "peak_kind": f"2 x bf16 ({pk_kind})",
           "ncols": ncols, "ms_per_step": round(ms, 4), "launches_per_step": n,
           "int16_macs_per_s": round(LAYER_MACS * ncols / (ms / 1e3) / 1e12, 3)}
    if ncols == 256 and n == 120:
        out["traffic"] = TC_STEP_TRAFFIC_256
        out["traffic_unit"] = "bytes per step, 120 launches (ncu dram__bytes_read.sum + dram__bytes_write.sum, 256 columns)"
    return out


# ---------------------------------------------------------------------------
# CPU side: the oracle port (numpy restatement of the reference simulator),
# one decode stream per host process.  The model is built once in the parent
# and the workers fork from it (copy-on-write), which is why the GPU arm runs
# these samples before it touches the GPU.
_CPU_MODEL = None


def _cpu_model():
    global _CPU_MODEL
    if _CPU_MODEL is None:
        sys.path.insert(0, REPO)
        from oracle import synth as OS
        _CPU_MODEL = OS.make_model(0)
        _CPU_MODEL.cache_float_weights()
    return _CPU_MODEL


def _cpu_stream(job):
    """Worker: decode n_steps x per_step tokens of one stream from KV length
    kv_len (cache filled with quantized N(0,1) values: the values do not
    change the cost); returns the wall seconds of each step."""
    kv_len, n_steps, per_step, seed = job
    from threadpoolctl import threadpool_limits
    from oracle import bfp_oracle as O
    threadpool_limits(1)
    model = _cpu_model()
    cfg = O.Cfg()
    kv = O.new_kv(cfg, kv_len + n_steps * per_step)
    rng = np.random.default_rng(seed)
    for li in range(cfg.NL):
        for k in ("k", "v"):
            kv[li][k][:kv_len] = O.fp_quantize_vec(rng.standard_normal(kv_len * 192)).reshape(kv_len, 3, 64)
    tok, pos = 123 + seed, kv_len
    times = []
    for _ in range(n_steps):
        t = time.perf_counter()
        for _ in range(per_step):
            h = model.embed_q(tok)
            cs = O.rope_cos_sin(pos)
            for li in range(cfg.NL):
                h = O.fwd_layer(h, model.layers[li], pos, kv[li], pos, cfg, cs=cs)
            tok = int(np.argmax(O.head_logits(h, model.norm_w_q, model.embed)))
            pos += 1
        times.append(time.perf_counter() - t)
    return times


def _host_info(procs):
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "usable": len(os.sched_getaffinity(0)), "cpu_model": model, "processes": procs}


def _cpu_procs(args):
    usable = len(os.sched_getaffinity(0))
    return max(1, args.cpu_procs or min(32, usable))


def _run_streams(jobs, procs):
    """Runs the jobs on `procs` forked workers; returns their per-step times."""
    import multiprocessing as mp
    _cpu_model()
    torch_mod = sys.modules.get("torch")
    if torch_mod is not None and torch_mod.cuda.is_initialized():
        raise RuntimeError("CPU baseline must run before the process initialises CUDA (workers fork)")
    with mp.get_context("fork").Pool(procs) as pool:
        return pool.map(_cpu_stream, jobs, chunksize=1)


def cpu_baselines(args):
    """The oracle port on the host cores (one stream per process).
    cfg2: one stream per process decoding at KV length 176 (the cfg2 mean),
    aggregate tok/s.  cfg3: the first 32 cfg3 sequences, each decoding 2
    tokens at its mid-generation KV length (prompt + 64), aggregate tok/s."""
    procs = _cpu_procs(args)
    info = _host_info(procs)
    steps2 = 3
    t = time.perf_counter()
    res2 = _run_streams([(176, steps2, 1, 10 + i) for i in range(procs)], procs)
    wall2 = time.perf_counter() - t
    v2 = procs * steps2 / max(sum(r) for r in res2)
    sys.path.insert(0, REPO)
    from oracle import synth as OS
    prompts3, _ = OS.config_prompts(3)
    jobs3 = [(len(p) + 64, 1, 2, 100 + i) for i, p in enumerate(prompts3[:32])]
    t = time.perf_counter()
    _run_streams(jobs3, procs)
    wall3 = time.perf_counter() - t
    v3 = 2 * len(jobs3) / wall3
    return {
        "cfg2": dict(value=round(v2, 3), unit="tok/s", cores=procs, kind="port",
                     sample=f"{procs} processes x {steps2} decode steps of a cfg2-shaped stream at KV length 176 "
                            f"(numpy oracle, 1 BLAS thread each; {wall2:.1f} s wall)", **info),
        "cfg3": dict(value=round(v3, 3), unit="tok/s", cores=procs, kind="port",
                     sample=f"first 32 cfg3 sequences x 2 decode steps at KV length prompt+64, {procs} processes "
                            f"(numpy oracle, 1 BLAS thread each; {wall3:.1f} s wall)", **info),
    }


def run_reference(args, world, rank):
    """--impl reference: the reference algorithm (the numpy restatement of the
    simulator under oracle/) on the host cores, rank 0 only: one cfg2 stream
    per process, every process decoding `per_step` tokens per step from KV
    length 48 (the end of the cfg2 prompt); a step's time is the slowest
    process's, value = processes x per_step / mean step time."""
    if rank != 0:
        return None
    procs = _cpu_procs(args)
    per_step = 2
    n = args.warmup + args.steps
    res = _run_streams([(48, n, per_step, 20 + i) for i in range(procs)], procs)
    step_s = [max(r[i] for r in res) for i in range(args.warmup, n)]
    mean_s = statistics.mean(step_s)
    v = procs * per_step / mean_s
    info = _host_info(procs)
    return {"impl": "reference", "metric": "BFP decode tok/s (bs1, cfg2)", "value": round(v, 4), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(mean_s * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64/f64",
            "data": "synthetic",
            "config": {"workload": "cfg2: 48-token prompt + greedy decode, bs1 per stream, KV<=304",
                       "model": "SmolLM2-135M arch, seeded random BFP weights", "global_batch": procs,
                       "seq_len": 304, "parallelism": f"host processes x{procs}"},
            "cpu_baseline": dict(value=round(v, 4), unit="tok/s", cores=procs, kind="port",
                                 sample=f"{procs} processes, each {per_step} decode steps per timed step of a "
                                        f"cfg2-shaped stream from KV length 48 (numpy restatement of the "
                                        f"reference simulator, 1 BLAS thread each)", **info),
            "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n-gen", type=int, default=256, help="generated tokens of the bs1 workload (profiling runs)")
    ap.add_argument("--no-bs256", action="store_true", help="skip the bs256 measurement (profiling runs)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--mm-reps", type=int, default=50, help="graph replays for the matmul roofline timing")
    ap.add_argument("--no-cfg5", action="store_true", help="skip the batch-64 / KV-2048 kernel profile")
    ap.add_argument("--no-cfg4", action="store_true", help="skip the matvec shape x batch sweep")
    ap.add_argument("--no-sharded-head", action="store_true",
                    help="with N > 1 GPUs, skip the single-stream decode with the vocabulary-sharded head")
    ap.add_argument("--cpu-procs", type=int, default=0,
                    help="host processes of the CPU baselines (default: usable cores, at most 32)")
    ap.add_argument("--cfg4-batches", type=lambda s: [int(x) for x in s.split(",")], default=[1, 8, 64, 256, 1024],
                    help="batch sizes of the matvec sweep")
    args = ap.parse_args()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        res = run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    world, rank, local = dist_init()
    res, detail = run_ours(args, world, rank, local)
    if rank == 0:
        print(json.dumps({"detail": detail}), flush=True)
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
