#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's
own simulator functions (jrrk2/tinyllm-fpga rtl/vc707/host/
gen_smollm_blockfp_full.py and gen_smollm_blockfp_ddr.py).

This script needs a checkout of the reference (environment variable
REF_ROOT) plus torch and transformers, which the reference imports at
module level.  It is run once, in a container that has the reference, and its
outputs are committed; the tests never need the reference itself.

Usage:  python tests/golden/make_golden.py <part> [<part> ...]
parts:  quant matvec layer tokens1 tokens2 tokens3:<i0>:<i1> merge3 image log2 sampled
        (tokens3:<i0>:<i1> writes tokens_cfg3_<i0>_<i1>.json for sequences
        i0..i1-1, so slices can run as parallel processes; merge3 joins every
        slice into tokens_cfg3.json and removes the slices)
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

from oracle import synth  # noqa: E402  (input data: the seeded synthetic model)
import inputs  # noqa: E402  (seeded input generators shared with the tests)

REF_ROOT = os.environ["REF_ROOT"]          # the reference checkout


_OUT_DIR = None


def load_ref(name, max_ctx=64):
    # the reference module writes its packer outputs under $OUT at import:
    # point it at a private temporary directory
    global _OUT_DIR
    if _OUT_DIR is None:
        _OUT_DIR = tempfile.mkdtemp(prefix="bfp200_ref_out_")
    os.environ["OUT"] = _OUT_DIR
    os.environ["MAX_CTX"] = str(max_ctx)
    path = os.path.join(REF_ROOT, "rtl/vc707/host", name)
    spec = importlib.util.spec_from_file_location(name[:-3], path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def save_manifest(key, value):
    path = os.path.join(HERE, "manifest.json")
    data = json.load(open(path)) if os.path.exists(path) else {}
    data[key] = value
    with open(path, "w") as f:
        json.dump(data, f, indent=1, sort_keys=True)


# ---------------------------------------------------------------------------
def part_quant(R):
    """tile_quantize on edge-case vectors (:90-97)."""
    v = inputs.quant_cases()
    m, e = R.tile_quantize(v)
    d = R.tile_decode(m, e)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), v=v, m=m, e=e, d=d)


def part_matvec(R):
    """matvec_hw_golden (:217-233) over the weight-shape sweep and edge cases."""
    out = {}
    for (D_out, D_in) in inputs.SWEEP_SHAPES:
        W_m, W_e = inputs.sweep_weights(D_out, D_in)
        for B in inputs.SWEEP_BATCHES:
            if B > inputs.ref_batch_limit(D_out):
                continue
            X_m, X_e = inputs.sweep_x(D_in, B, D_out)
            t = time.time()
            cols = [R.matvec_hw_golden(X_m[b], X_e[b], W_m, W_e) for b in range(B)]
            Y = np.stack(cols)
            ym, ye = R.tile_quantize(Y.reshape(-1))
            key = f"{D_out}x{D_in}_b{B}"
            out[key] = sha(ym, ye)
            print(key, f"{time.time() - t:.1f}s", file=sys.stderr)
            if D_out * B <= 8192:
                np.savez_compressed(os.path.join(HERE, f"matvec_{key}.npz"), y=Y)
    for name, (x_m, x_e, W_m, W_e) in inputs.matvec_edge_cases().items():
        y = R.matvec_hw_golden(x_m, x_e, W_m, W_e)
        np.savez_compressed(os.path.join(HERE, f"matvec_edge_{name}.npz"), x_m=x_m, x_e=x_e,
                            W_m=W_m, W_e=W_e, y=y)
    save_manifest("matvec_sha", out)


def part_layer(R):
    """fwd_layer (:261-293) at several KV lengths, layer 0 of the synthetic model,
    over a KV cache pre-filled with quantized N(0,1) values."""
    model = synth.make_model(0)
    lw = {k: model.layers[0][k] for k in ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd", "g1", "g2")}
    res = {}
    for kv_pos in inputs.LAYER_KV_POS:
        h, K, V = inputs.layer_case(kv_pos, max_ctx=kv_pos + 1)
        kv = {"k": K.copy(), "v": V.copy()}
        t = time.time()
        out = R.fwd_layer(h, lw, kv_pos, kv, kv_pos)
        print("layer kv_pos", kv_pos, f"{time.time() - t:.2f}s", file=sys.stderr)
        res[f"out_{kv_pos}"] = out
        res[f"k_{kv_pos}"] = kv["k"][kv_pos]
        res[f"v_{kv_pos}"] = kv["v"][kv_pos]
    np.savez_compressed(os.path.join(HERE, "layer.npz"), **res)


def ref_generate(R, model, ids, n_gen, max_ctx):
    """The reference's driver loop, gen_smollm_blockfp_full.py:425-443,
    restated around its own fwd_layer / fp_quantize_vec (main() needs the HF
    hub, so only this loop is re-driven)."""
    NL = model.cfg.NL
    layers_fwd = [{k: model.layers[li][k] for k in ("Wq", "Wk", "Wv", "Wo", "Wg", "Wu", "Wd", "g1", "g2")}
                  for li in range(NL)]
    embed = model.embed
    norm_w_q = R.fp_quantize_vec(model.norm_w)
    kv = [{'k': np.zeros((max_ctx, 3, 64)), 'v': np.zeros((max_ctx, 3, 64))} for _ in range(NL)]
    generated = list(ids)
    margins = []
    for step in range(len(ids) + n_gen):
        tid = ids[step] if step < len(ids) else generated[-1]
        h = R.fp_quantize_vec(embed[tid].astype(np.float64))
        for li in range(NL):
            h = R.fwd_layer(h, layers_fwd[li], pos=step, kv=kv[li], kv_pos=step)
        if step >= len(ids) - 1:
            h_normed = (h / np.sqrt(np.mean(h * h) + 1e-5)) * norm_w_q
            logits = h_normed @ embed.T
            nid = int(np.argmax(logits))
            top2 = np.sort(logits)[-2:]
            margins.append(float(top2[1] - top2[0]))
            if step >= len(ids):
                generated.append(nid)
    return generated, margins


def part_tokens(R, cfg_id, i0=None, i1=None):
    model = synth.make_model(0)
    prompts, n_gen = synth.config_prompts(cfg_id)
    if i0 is not None:
        prompts = prompts[i0:i1]
    out = {}
    for i, ids in enumerate(prompts):
        t = time.time()
        toks, margins = ref_generate(R, model, ids, n_gen, len(ids) + n_gen)
        idx = i + (i0 or 0)
        out[str(idx)] = {"tokens": toks, "min_margin": min(margins)}
        print(f"cfg{cfg_id} seq {idx}: {time.time() - t:.0f}s min_margin {min(margins):.3e}",
              file=sys.stderr)
    suffix = "" if i0 is None else f"_{i0}_{i1}"
    with open(os.path.join(HERE, f"tokens_cfg{cfg_id}{suffix}.json"), "w") as f:
        json.dump(out, f)


# (temperature, top-k, seed) of the sampled-decode fixtures
SAMPLED_CASES = [(0.8, 0, 1), (1.0, 50, 7), (0.6, 5, 3), (1.3, 1000, 11), (2.0, 1, 5)]
SAMPLED_N_GEN = 12


def load_ref_hw():
    """rtl/vc707/host/sim_rtl_fp_hw.py, the hardware emulator whose main()
    holds the temperature / top-k sampling loop (:196-216).  It imports
    sim_blockfp from its own directory and seeds numpy at import."""
    host = os.path.join(REF_ROOT, "rtl/vc707/host")
    if host not in sys.path:
        sys.path.insert(0, host)
    spec = importlib.util.spec_from_file_location("sim_rtl_fp_hw", os.path.join(host, "sim_rtl_fp_hw.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def part_sampled(H):
    """Sampled streams of the reference emulator: its own fwd_hw per layer
    (sim_rtl_fp_hw.py:111-145) on the synthetic model, and its sampling loop
    (:196-216, main() needs the HF checkpoint, so the loop is restated here
    around the module's functions) with the global numpy generator seeded by
    np.random.seed(SEED), the cfg1 prompt and SAMPLED_N_GEN tokens."""
    model = synth.make_model(0)
    c = model.cfg
    prompt = [int(t) for t in synth.config_prompts(1)[0][0]]
    n_steps = len(prompt) + SAMPLED_N_GEN
    cfg = dict(D=c.D, H_Q=c.H_Q, H_KV=c.H_KV, HD=c.HD, FFN=c.FFN, NL=c.NL, MAX_CTX=n_steps)
    layers = []
    for li in range(c.NL):
        d = {nm + "_me": model.layers[li][nm] for nm in synth.MATS}
        d["g1"] = model.layers[li]["g1"]
        d["g2"] = model.layers[li]["g2"]
        layers.append(d)
    embed, norm_w = model.embed, model.norm_w
    out = []
    for T, TOPK, SEED in SAMPLED_CASES:
        t0 = time.time()
        kv = [{"k": np.zeros((n_steps, c.H_KV, c.HD)), "v": np.zeros((n_steps, c.H_KV, c.HD))} for _ in range(c.NL)]
        np.random.seed(SEED)
        generated = list(prompt)
        for step in range(n_steps):
            tid = prompt[step] if step < len(prompt) else generated[-1]
            h = H.fp_quantize(embed[tid].astype(np.float64))
            for li in range(c.NL):
                h = H.fwd_hw(h, layers[li], pos=step, kv=kv[li], kv_pos=step, cfg=cfg)
            if step >= len(prompt) - 1:
                h_normed = (h / np.sqrt(np.mean(h * h) + 1e-5)) * norm_w
                logits = h_normed @ embed.T
                scaled = logits / T
                if TOPK > 0:
                    idx = np.argsort(scaled)[-TOPK:]
                    mask = np.full_like(scaled, -np.inf)
                    mask[idx] = scaled[idx]
                    scaled = mask
                scaled -= scaled.max()
                p = np.exp(scaled)
                p = p / p.sum()
                nid = int(np.random.choice(len(p), p=p))
                if step >= len(prompt):
                    generated.append(nid)
        out.append({"temperature": T, "top_k": TOPK, "seed": SEED, "n_gen": SAMPLED_N_GEN, "tokens": generated})
        print(f"sampled T={T} topk={TOPK} seed={SEED}: {time.time() - t0:.0f}s {generated[len(prompt):]}",
              file=sys.stderr)
    with open(os.path.join(HERE, "sampled.json"), "w") as f:
        json.dump(out, f)


def part_merge3():
    import glob
    allt = {}
    slices = sorted(glob.glob(os.path.join(HERE, "tokens_cfg3_*.json")))
    for fn in slices:
        with open(fn) as f:
            for k, v in json.load(f).items():
                allt[int(k)] = v
    with open(os.path.join(HERE, "tokens_cfg3.json"), "w") as f:
        json.dump({str(k): allt[k] for k in sorted(allt)}, f)
    for fn in slices:
        os.remove(fn)
    print("cfg3 sequences:", len(allt), file=sys.stderr)


def part_image(D):
    """Byte image through the reference packer's own functions
    (gen_smollm_blockfp_ddr.py:65-119), assembled in the region order of its
    main() (:155-221)."""
    model = synth.make_model(0)
    NL = model.cfg.NL
    regions = []

    def add_region(name, data):
        size_aligned = D.align4k(len(data))
        regions.append((name, data + b"\x00" * (size_aligned - len(data))))

    layers_q = []
    for li in range(NL):
        lf = model.layers_float[li]
        row = {nm: D.quantize_W(lf[nm]) for nm in synth.MATS}
        row["g1"] = D.tile_quantize(lf["g1"])
        row["g2"] = D.tile_quantize(lf["g2"])
        layers_q.append(row)
    for tag, key in [("WQ", "Wq"), ("WK", "Wk"), ("WV", "Wv"), ("WO", "Wo"),
                     ("WG", "Wg"), ("WU", "Wu"), ("WDN", "Wd")]:
        t = time.time()
        m_buf = b"".join(D.pack_layer_mantissas(*layers_q[li][key]) for li in range(NL))
        e_buf = b"".join(D.pack_layer_exponents(layers_q[li][key][1]) for li in range(NL))
        add_region(f"{tag}_m", m_buf)
        add_region(f"{tag}_e", e_buf)
        print(tag, f"{time.time() - t:.0f}s", file=sys.stderr)
    for g in ("g1", "g2"):
        add_region(g.upper() + "_m", b"".join(layers_q[li][g][0].tobytes() for li in range(NL)))
        add_region(g.upper() + "_e", b"".join(layers_q[li][g][1].tobytes() for li in range(NL)))
    emb_m, emb_e = D.quantize_W(model.embed)
    add_region("EMBED_m", D.pack_layer_mantissas(emb_m, emb_e))
    add_region("EMBED_e", D.pack_layer_exponents(emb_e))
    lu_m = b""
    lu_e = []
    for r in range(model.embed.shape[0]):
        m, e = D.tile_quantize(model.embed[r])
        lu_e.append(e.tobytes() + b"\x00" * (64 - len(e.tobytes())))
    lu_m = emb_m.reshape(model.embed.shape[0], -1).tobytes()   # row-major m, same bytes as :211
    add_region("EMBED_LU_m", lu_m)
    add_region("EMBED_LU_e", b"".join(lu_e))
    nw_m, nw_e = D.tile_quantize(model.norm_w)
    add_region("NORM_W_m", nw_m.tobytes())
    add_region("NORM_W_e", nw_e.tobytes())
    img = bytearray()
    offsets = {}
    for name, data in regions:
        offsets[name] = len(img)
        img.extend(data)
    h = hashlib.sha256(img).hexdigest()
    save_manifest("image", {"sha256": h, "len": len(img), "offsets": offsets})
    # first 64 KiB of every region, to localise a mismatch
    heads = {name: np.frombuffer(bytes(img[off:off + 4096]), dtype=np.uint8) for name, off in offsets.items()}
    np.savez_compressed(os.path.join(HERE, "image_heads.npz"), **heads)
    print("image", len(img), h, file=sys.stderr)


def part_log2():
    from oracle import bfp_oracle as O
    save_manifest("log2_round_up_counts", {str(k): v for k, v in O.floor_log2_threshold_counts(-130, 130).items()})


def main(argv):
    for part in argv:
        t = time.time()
        if part == "image":
            part_image(load_ref("gen_smollm_blockfp_ddr.py"))
        elif part == "log2":
            part_log2()
        elif part == "merge3":
            part_merge3()
        elif part == "sampled":
            part_sampled(load_ref_hw())
        elif part.startswith("tokens"):
            cfg_id = int(part[6])
            if ":" in part:
                _, i0, i1 = part.split(":")
                part_tokens(load_ref("gen_smollm_blockfp_full.py"), cfg_id, int(i0), int(i1))
            else:
                part_tokens(load_ref("gen_smollm_blockfp_full.py"), cfg_id)
        elif part == "layer":
            part_layer(load_ref("gen_smollm_blockfp_full.py", max_ctx=max(inputs.LAYER_KV_POS) + 1))
        else:
            globals()["part_" + part](load_ref("gen_smollm_blockfp_full.py"))
        print(f"[golden] {part} done in {time.time() - t:.0f}s", file=sys.stderr)


if __name__ == "__main__":
    main(sys.argv[1:])
