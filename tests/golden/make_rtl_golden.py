#!/usr/bin/env python3
"""Generate tests/golden/rtl_ops.npz: golden vectors of the reference's
fixed-point ("rtl-exact") leaf ops, produced by the REFERENCE's own per-op
golden generators (jrrk2/tinyllm-fpga rtl/vc707/host/gen_*_bfp_golden.py,
which mirror the RTL modules matvec_bfp_engine.sv, rmsnorm_bfp.sv,
rope_bfp.sv, softmax_bfp.sv, swiglu_bfp.sv and the residual adder) and of
its ROM generators (rtl/vc707/sim/gen_exp_lut.py, gen_swiglu_lut.py).

Each generator script is executed (numpy only) in a scratch directory --
they read their LUTs from ./generated and write their own small vectors
there -- and its golden_* function is then called on further seeded inputs.
The RoPE frequency table is written in the generator's .svh format by the
formula of rtl/vc707/sim/gen_rope_freq_table.py (that script writes into its
own source tree).  Run once where the reference exists (REF_ROOT = its
checkout); the tests only read the .npz.

Usage:  python tests/golden/make_rtl_golden.py
"""
from __future__ import annotations

import hashlib
import math
import os
import runpy
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ["REF_ROOT"]          # the reference checkout
HOST = os.path.join(REF_ROOT, "rtl/vc707/host")
SIM = os.path.join(REF_ROOT, "rtl/vc707/sim")
TILE = 16


def run_ref(path, **env):
    old = {k: os.environ.get(k) for k in env}
    os.environ.update({k: str(v) for k, v in env.items()})
    try:
        return runpy.run_path(path, run_name="__main__")
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def freq_svh(path, base, hd=64):
    vals = []
    for j in range(hd // 2):
        f = 1.0 / (base ** (2.0 * j / hd))
        vals.append(round(f / (2.0 * math.pi) * (1 << 31)))
    with open(path, "w") as f:
        f.write("localparam logic [31:0] FREQ_TURNS_Q31 [0:31] = '{\n")
        for i, v in enumerate(vals):
            f.write(f"  32'd{v:>12}{',' if i < len(vals) - 1 else ' '}\n")
        f.write("};\n")
    return np.array(vals, np.uint32)


def tq(rng, n, scale):
    """Tile-quantized random vector (the generators' tile_quantize_raw)."""
    v = rng.standard_normal(n) * scale
    flat = v.reshape(-1, TILE)
    e = (np.floor(np.log2(np.maximum(np.abs(flat).max(axis=1), 1e-300))).astype(np.int32) + 1).clip(-127, 127)
    m = np.clip(np.round(flat / np.power(2.0, e.astype(np.float64))[:, None] * 32768.0).astype(np.int64),
                -32768, 32767)
    return m.astype(np.int16), e.astype(np.int8)


def main():
    out = {}
    work = tempfile.mkdtemp(prefix="rtl_golden_")
    os.chdir(work)
    gen = os.path.join(work, "generated")
    os.makedirs(gen, exist_ok=True)
    # ROMs, written by the reference's own generators
    run_ref(os.path.join(SIM, "gen_exp_lut.py"), OUT=gen)
    run_ref(os.path.join(SIM, "gen_swiglu_lut.py"), OUT=gen)
    exp_lut = np.array([int(x, 16) for x in open(os.path.join(gen, "exp_lut.hex")).read().split()], np.uint16)
    silu_lut = np.array([int(x, 16) for x in open(os.path.join(gen, "silu_lut.hex")).read().split()],
                        np.uint16).view(np.int16)
    out["exp_lut_sha"] = np.frombuffer(hashlib.sha256(exp_lut.tobytes()).digest(), np.uint8)
    out["silu_lut_sha"] = np.frombuffer(hashlib.sha256(silu_lut.tobytes()).digest(), np.uint8)
    out["exp_lut_head"] = exp_lut[[0, 1, 511, 767, 895, 1022, 1023]]
    out["silu_lut_probe"] = silu_lut[[0, 1, 100, 16384, 32767, 32768, 40000, 65535]]

    rng = np.random.default_rng(2027)

    # ---- matvec (matvec_bfp_engine.sv): 16 output lanes per call
    for D in (64, 576, 1536):
        g = run_ref(os.path.join(HOST, "gen_matvec_bfp_golden.py"), D=D)
        xs, ws, ys = [], [], []
        for k in ((0, 1, 2, 3) if D < 1536 else (0, 3)):
            x_m, x_e = tq(rng, D, [5.0, 1e-3, 40.0, 1.0][k])
            W_m = np.zeros((16, D // TILE, TILE), np.int16)
            W_e = np.zeros((16, D // TILE), np.int8)
            for i in range(16):
                W_m[i], W_e[i] = tq(rng, D, [0.3, 2.0, 1e-4, 0.02][k] * (1 + i % 3))
            if k == 3:                    # wide exponent spread: mask / shift edge cases
                W_e[:, ::3] -= 40
                W_e[:, 1::5] += 9
            y_m, y_e = g["golden_matvec"](x_m, x_e, W_m, W_e)
            xs.append((x_m, x_e)); ws.append((W_m, W_e)); ys.append((y_m, y_e))
        out[f"mv{D}_xm"] = np.stack([a for a, _ in xs]); out[f"mv{D}_xe"] = np.stack([b for _, b in xs])
        out[f"mv{D}_wm"] = np.stack([a for a, _ in ws]); out[f"mv{D}_we"] = np.stack([b for _, b in ws])
        out[f"mv{D}_ym"] = np.stack([a for a, _ in ys]); out[f"mv{D}_ye"] = np.stack([b for _, b in ys])

    # ---- rmsnorm (rmsnorm_bfp.sv)
    for D in (64, 576):
        g = run_ref(os.path.join(HOST, "gen_rmsnorm_bfp_golden.py"), D=D)
        cols = {"xm": [], "xe": [], "gm": [], "ge": [], "ym": [], "ye": []}
        for k in range(8):
            x_m, x_e = tq(rng, D, [3.0, 0.01, 200.0, 1.0, 1e-6, 7.0, 0.5, 50.0][k])
            g_m, g_e = tq(rng, D, 0.8)
            g_m = np.abs(g_m) if k % 2 else g_m
            y_m, y_e = g["golden_rmsnorm"](x_m, x_e, g_m, g_e)
            for n, v in zip(cols, (x_m, x_e, g_m, g_e, y_m, y_e)):
                cols[n].append(v)
        for n, v in cols.items():
            out[f"rms{D}_{n}"] = np.stack(v)

    # ---- RoPE (rope_bfp.sv), both rope bases
    for base in (10000.0, 100000.0):
        tag = int(base)
        out[f"rope{tag}_freq"] = freq_svh(os.path.join(gen, "rope_freq_turns.svh"), base)
        g = run_ref(os.path.join(HOST, "gen_rope_bfp_golden.py"), POS=3)
        poss = [0, 1, 3, 17, 100, 255, 303, 1000, 2047, 4095]
        cols = {"xm": [], "xe": [], "ym": [], "ye": []}
        for pos in poss:
            x_m, x_e = tq(rng, 64, [1.0, 30.0][pos % 2])
            y_m, y_e = g["golden_rope"](x_m, x_e, pos)
            for n, v in zip(cols, (x_m, x_e, np.array(y_m, np.int16), np.array(y_e, np.int8))):
                cols[n].append(v)
        for n, v in cols.items():
            out[f"rope{tag}_{n}"] = np.stack(v)
        out[f"rope{tag}_pos"] = np.array(poss, np.int32)

    # ---- softmax (softmax_bfp.sv): one shared exponent per vector
    g = run_ref(os.path.join(HOST, "gen_softmax_bfp_golden.py"), N=8)
    for N in (1, 8, 37, 64):
        xm, xe, ym, ye = [], [], [], []
        for k in range(6):
            v = rng.standard_normal(N) * [3.0, 0.1, 20.0, 1.0, 1e-4, 300.0][k]
            x_m, x_e = g["block_quantize_scalar_vec"](v)
            y_m, y_e = g["golden_softmax"](x_m, x_e, N)
            xm.append(x_m); xe.append(x_e); ym.append(np.array(y_m, np.int16)); ye.append(y_e)
        out[f"sm{N}_xm"] = np.stack(xm); out[f"sm{N}_xe"] = np.array(xe, np.int32)
        out[f"sm{N}_ym"] = np.stack(ym); out[f"sm{N}_ye"] = np.array(ye, np.int32)

    # ---- SwiGLU (swiglu_bfp.sv)
    for D in (64, 1536):
        g = run_ref(os.path.join(HOST, "gen_swiglu_bfp_golden.py"), D=D)
        cols = {"gm": [], "ge": [], "um": [], "ue": [], "ym": [], "ye": []}
        for k in range(6):
            g_m, g_e = tq(rng, D, [4.0, 0.05, 40.0, 1.0, 300.0, 1e-3][k])
            u_m, u_e = tq(rng, D, [1.0, 3.0, 0.01, 1.0, 1.0, 50.0][k])
            y_m, y_e = g["golden_swiglu"](g_m, g_e, u_m, u_e)
            for n, v in zip(cols, (g_m, g_e, u_m, u_e, y_m, y_e)):
                cols[n].append(v)
        for n, v in cols.items():
            out[f"sw{D}_{n}"] = np.stack(v)

    # ---- residual add
    for D in (64, 576):
        g = run_ref(os.path.join(HOST, "gen_residual_bfp_golden.py"), D=D)
        cols = {"am": [], "ae": [], "bm": [], "be": [], "ym": [], "ye": []}
        for k in range(6):
            a_m, a_e = tq(rng, D, [3.0, 1.0, 1e3, 1e-3, 1.0, 5.0][k])
            b_m, b_e = tq(rng, D, [1.5, 1.0, 1e-3, 1e3, 1.0, 5.0][k])
            if k == 4:
                b_m = -a_m; b_e = a_e.copy()          # exact cancellation
            y_m, y_e = g["golden_residual"](a_m, a_e, b_m, b_e)
            for n, v in zip(cols, (a_m, a_e, b_m, b_e, y_m, y_e)):
                cols[n].append(v)
        for n, v in cols.items():
            out[f"res{D}_{n}"] = np.stack(v)

    np.savez_compressed(os.path.join(HERE, "rtl_ops.npz"), **out)
    print("wrote", os.path.join(HERE, "rtl_ops.npz"), file=sys.stderr)


if __name__ == "__main__":
    main()
