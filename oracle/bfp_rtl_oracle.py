"""Integer restatement of the reference's fixed-point ("rtl-exact") leaf ops
(TEST ONLY -- the product never imports it).

These are the arithmetic of the FPGA modules, as pinned by the reference's
own per-op golden generators (jrrk2/tinyllm-fpga rtl/vc707/host/):

  matvec    gen_matvec_bfp_golden.py:49-104   (matvec_bfp_engine.sv)
  rmsnorm   gen_rmsnorm_bfp_golden.py:43-144  (rmsnorm_bfp.sv)
  rope      gen_rope_bfp_golden.py:25-124     (rope_bfp.sv, cordic_sincos.sv)
  softmax   gen_softmax_bfp_golden.py:34-83   (softmax_bfp.sv)
  swiglu    gen_swiglu_bfp_golden.py:45-77    (swiglu_bfp.sv)
  residual  gen_residual_bfp_golden.py:20-45
  ROMs      rtl/vc707/sim/gen_exp_lut.py, gen_swiglu_lut.py,
            gen_rope_freq_table.py

Common output step ("normalise to Q1.15"): a group of integer products is
shifted so that the largest magnitude's leading one lands on bit 14
(shift = lead - 14, arithmetic right shift or left shift), the low 16 bits
are kept as a signed mantissa, and the exponent is adjusted by the shift.
Python integers make every intermediate exact; tests compare this module
with the generators' vectors (tests/golden/rtl_ops.npz).
"""
from __future__ import annotations

import math

import numpy as np

TILE = 16
ACC_W = 48


def _lead(v: int) -> int:
    return abs(v).bit_length() - 1 if v else 0


def _wrap16(v: int) -> int:
    v &= 0xFFFF
    return v - 0x10000 if v & 0x8000 else v


def _norm_group(vals):
    """Shift a group so its largest |value| leads at bit 14; returns the 16-bit
    mantissas and the shift."""
    lead = max((_lead(v) for v in vals if v), default=0)
    sh = lead - 14
    return [_wrap16(v >> sh if sh >= 0 else v << -sh) for v in vals], sh


def _clamp8(e):
    return max(-128, min(127, e))


# ---------------------------------------------------------------------------
# ROMs
# ---------------------------------------------------------------------------
def exp_lut():
    """1024 x Q1.15: exp((i - 1023) / 128), round half to even, clamped to u16."""
    return np.array([min(65535, max(0, round(math.exp((i - 1023) / 128.0) * 32768))) for i in range(1024)],
                    np.uint16)


def silu_lut(scale=32.0):
    """65536 x int16 indexed by the 16-bit gate pattern: silu(g) at Q1.15 of scale."""
    g = np.arange(65536, dtype=np.uint16).view(np.int16).astype(np.float64) / 32768.0 * scale
    s = g * (1.0 / (1.0 + np.exp(-g)))
    return np.clip(np.round(s * 32768.0 / scale).astype(np.int64), -32768, 32767).astype(np.int16)


def rope_freq_turns(base=10000.0, hd=64):
    """Q0.31 turns per position of each rotary pair: round(base^(-2j/hd) / 2pi * 2^31)."""
    return np.array([round((1.0 / (base ** (2.0 * j / hd))) / (2.0 * math.pi) * (1 << 31)) for j in range(hd // 2)],
                    np.uint32)


# ---------------------------------------------------------------------------
# matvec: per-row running alignment of the tile sums into a 48-bit
# accumulator (the later of two exponents wins, the other side is shifted
# right, > 47 bits shifted away), saturating after every add; the result is
# normalised per row (one exponent per OUTPUT ELEMENT).
# ---------------------------------------------------------------------------
def matvec(x_m, x_e, W_m, W_e):
    hi, lo = (1 << (ACC_W - 1)) - 1, -(1 << (ACC_W - 1))
    R, NT = W_e.shape
    out_m = np.zeros(R, np.int16)
    out_e = np.zeros(R, np.int8)
    sums = (W_m.astype(np.int64) * x_m.astype(np.int64)[None]).sum(axis=2)     # exact
    for r in range(R):
        acc, acc_e = int(sums[r, 0]), int(x_e[0]) + int(W_e[r, 0])
        for t in range(1, NT):
            s, e = int(sums[r, t]), int(x_e[t]) + int(W_e[r, t])
            d = e - acc_e
            if d > 0:
                acc = 0 if d > ACC_W - 1 else acc >> d
                acc_e = e
            elif d < 0:
                s = 0 if -d > ACC_W - 1 else s >> -d
            acc = min(hi, max(lo, acc + s))
        (m,), sh = _norm_group([acc])
        out_m[r] = m
        out_e[r] = _clamp8(acc_e + sh - 15)
    return out_m, out_e


# ---------------------------------------------------------------------------
# rmsnorm: sum of squares with the same running alignment (no saturation),
# mean by a Q0.32 reciprocal of D, Q2.30 normalisation with an even total
# exponent, epsilon 10737 (1e-5 in Q2.30), three Newton-Raphson steps of
# 1/sqrt from a 26-entry leading-bit seed table (Q12.12), then per tile
# x * g * inv_rms normalised to Q1.15.
# ---------------------------------------------------------------------------
RSQRT_SEED = {31: 2365, 30: 3344, 29: 4730, 28: 6689, 27: 9459, 26: 13377, 25: 18919, 24: 26755, 23: 37837,
              22: 53510, 21: 75674, 20: 107020, 19: 151349, 18: 214040, 17: 302698, 16: 428079, 15: 605396,
              14: 856159, 13: 1210791, 12: 1712317, 11: 2421583, 10: 3424635, 9: 4843165, 8: 6849270,
              7: 9686330, 6: 13698540}
EPS_Q30 = 10737


def rms_inv(x_m, x_e, D):
    """(inv_rms as Q12.12 integer, its exponent excess)."""
    NT = D // TILE
    sq = (x_m.astype(np.int64) ** 2).sum(axis=1)
    acc, acc_e = int(sq[0]), 2 * int(x_e[0])
    for t in range(1, NT):
        s, e = int(sq[t]), 2 * int(x_e[t])
        d = e - acc_e
        if d > 0:
            acc = 0 if d > ACC_W - 1 else acc >> d
            acc_e = e
        elif d < 0:
            s = s >> -d if -d <= ACC_W - 1 else 0
        acc += s
    mean = (acc * ((1 << 32) // D)) >> 32
    lead = mean.bit_length() - 1 if mean else 0
    if (acc_e + lead) & 1:
        lead -= 1
    v = (mean >> (lead - 30) if lead >= 30 else mean << (30 - lead)) + EPS_Q30
    y = RSQRT_SEED.get(v.bit_length() - 1 if v else 0, (1 << 24) - 1)
    three_halves = (3 << 30) // 2
    for _ in range(3):
        t = (v * (y * y)) >> 24
        corr = 0 if t >= (1 << 32) else max(0, three_halves - (t >> 1))
        y = min((y * corr + (1 << 29)) >> 30, (1 << 24) - 1)
    return y, (30 - acc_e - lead) >> 1


def rmsnorm(x_m, x_e, g_m, g_e):
    D = x_m.size
    y, e_inv = rms_inv(x_m, x_e, D)
    out_m = np.zeros(D, np.int16)
    out_e = np.zeros(D // TILE, np.int8)
    for t in range(D // TILE):
        prods = [int(x_m[t, k]) * int(g_m[t, k]) * y for k in range(TILE)]
        ms, sh = _norm_group(prods)
        out_m[t * TILE:(t + 1) * TILE] = ms
        out_e[t] = _clamp8(int(x_e[t]) + int(g_e[t]) + e_inv + sh - 27)
    return out_m, out_e


# ---------------------------------------------------------------------------
# RoPE: angle = pos * turns (Q0.31, wrapped to a signed 31-bit turn count),
# scaled to a Q3.27 radian angle by pi/8 in Q2.29, 16 CORDIC rotations (gain
# pre-compensated, quadrant folded for |angle| > pi/2), rounded to Q1.15
# cos/sin; each pair is exponent-aligned (>= 16 bits shifted away), rotated
# in integers and every element normalised on its own (one exponent per
# OUTPUT ELEMENT).
# ---------------------------------------------------------------------------
CORDIC_ATAN_Q27 = [105414357, 62229729, 32880480, 16690645, 8377711, 4192939, 2096981, 1048555, 524285, 262144,
                   131072, 65536, 32768, 16384, 8192, 4096]
CORDIC_K_Q27 = 81504109
PI_Q27, HALF_PI_Q27, PI_8_Q29 = 421657428, 210828714, 210828714


def _wrap31(v):
    v &= (1 << 31) - 1
    return v - (1 << 31) if v & (1 << 30) else v


def cordic(a):
    neg = False
    if a > HALF_PI_Q27:
        a, neg = PI_Q27 - a, True
    elif a < -HALF_PI_Q27:
        a, neg = -PI_Q27 - a, True
    x, y = CORDIC_K_Q27, 0
    for i, at in enumerate(CORDIC_ATAN_Q27):
        xs, ys = x >> i, y >> i
        if a >= 0:
            x, y, a = x - ys, y + xs, a - at
        else:
            x, y, a = x + ys, y - xs, a + at
    xs, ys = (x + 2048) >> 12, (y + 2048) >> 12
    if xs > 32767:
        c = -32767 if neg else 32767
    elif xs < -32768:
        c = 32767 if neg else -32768
    else:
        c = -xs if neg else xs
    s = min(32767, max(-32768, ys))
    return c, s


def rope(x_m, x_e, pos, turns):
    HD = x_m.size
    H2 = HD // 2
    m = x_m.reshape(-1).astype(np.int64)
    e = np.repeat(x_e.astype(np.int64), TILE)
    prod = [0] * HD
    pe = [0] * HD
    for j in range(H2):
        ang = _wrap31(_wrap31(pos * int(turns[j])) * PI_8_Q29 >> 29)
        c, s = cordic(ang)
        a, b = int(m[j]), int(m[j + H2])
        ea, eb = int(e[j]), int(e[j + H2])
        em = max(ea, eb)
        a = a >> (em - ea) if em - ea < 16 else 0
        b = b >> (em - eb) if em - eb < 16 else 0
        prod[j], prod[j + H2] = a * c - b * s, b * c + a * s
        pe[j] = pe[j + H2] = em
    out_m = np.zeros(HD, np.int16)
    out_e = np.zeros(HD, np.int8)
    for k in range(HD):
        (mm,), sh = _norm_group([prod[k]])
        out_m[k] = mm
        out_e[k] = _clamp8(pe[k] + sh - 15)
    return out_m, out_e


# ---------------------------------------------------------------------------
# softmax over n scores sharing one exponent: differences to the max scaled
# to 1/128 steps (shift by e - 8), exp from the 1024-entry ROM, 1/sum by four
# Newton-Raphson steps (Q0.32 seed 2^(31 - msb)), products normalised as one
# group with exponent shift - 17.
# ---------------------------------------------------------------------------
def softmax(x_m, e, lut):
    n = x_m.size
    mx = int(x_m.max())
    ev = []
    for k in range(n):
        d = int(x_m[k]) - mx
        sh = e - 8
        d = d << sh if sh >= 0 else d >> -sh
        ev.append(int(lut[1023 if d >= 0 else (0 if d <= -1023 else d + 1023)]))
    s = sum(ev)
    y = 1 << (31 - (s.bit_length() - 1 if s else 0))
    for _ in range(4):
        y = (y * ((1 << 33) - s * y)) >> 32
    ms, sh = _norm_group([v * y for v in ev])
    return np.array(ms, np.int16), _clamp8(sh - 17)


# ---------------------------------------------------------------------------
# SwiGLU: the gate mantissa brought to the ROM's scale (shift by e_gate - 5,
# saturated to 16 bits) indexes silu; times the up mantissa; each tile
# normalised, exponent e_up + shift - 10.
# ---------------------------------------------------------------------------
def swiglu(g_m, g_e, u_m, u_e, lut):
    NT = g_e.size
    out_m = np.zeros(NT * TILE, np.int16)
    out_e = np.zeros(NT, np.int8)
    for t in range(NT):
        sh = int(g_e[t]) - 5
        prods = []
        for k in range(TILE):
            i = int(g_m[t, k])
            i = i << sh if sh >= 0 else i >> -sh
            i = max(-32768, min(32767, i))
            prods.append(int(lut[i & 0xFFFF]) * int(u_m[t, k]))
        ms, s2 = _norm_group(prods)
        out_m[t * TILE:(t + 1) * TILE] = ms
        out_e[t] = _clamp8(int(u_e[t]) + s2 - 10)
    return out_m, out_e


# ---------------------------------------------------------------------------
# residual: per tile, both operands aligned to the larger exponent (>= 16 bits
# shifted away), added, the tile normalised, exponent e_max + shift.
# ---------------------------------------------------------------------------
def residual(a_m, a_e, b_m, b_e):
    NT = a_e.size
    out_m = np.zeros(NT * TILE, np.int16)
    out_e = np.zeros(NT, np.int8)
    for t in range(NT):
        ea, eb = int(a_e[t]), int(b_e[t])
        em = max(ea, eb)
        sums = []
        for k in range(TILE):
            a = int(a_m[t, k]) >> (em - ea) if em - ea < 16 else 0
            b = int(b_m[t, k]) >> (em - eb) if em - eb < 16 else 0
            sums.append(a + b)
        ms, sh = _norm_group(sums)
        out_m[t * TILE:(t + 1) * TILE] = ms
        out_e[t] = _clamp8(em + sh)
    return out_m, out_e
