"""Fixed-point ("rtl-exact") leaf ops of the FPGA modules, on the GPU.

The reference's RTL computes RMSNorm, RoPE, softmax, SwiGLU, the matvec and
the residual add in integer arithmetic (Newton-Raphson reciprocals, CORDIC,
ROM lookups, running exponent alignment); its per-op golden generators
(rtl/vc707/host/gen_*_bfp_golden.py) pin that arithmetic.  These functions
compute the same integers through libbfp200 (csrc/rtl.cu).  Vectors are
tile-major like the generators' arrays: mantissas (..., D/16, 16) int16,
tile exponents (..., D/16) int8; leading axes are batch.

The ROMs follow the reference's ROM generators (rtl/vc707/sim/gen_exp_lut.py,
gen_swiglu_lut.py, gen_rope_freq_table.py) and can also be read from their
.hex / .svh files.
"""
from __future__ import annotations

import math
import re

import numpy as np

from . import _lib
from ._lib import check, ptr
from .ops import context

TILE = 16


# ---------------------------------------------------------------------------
# ROMs
# ---------------------------------------------------------------------------
def exp_lut():
    """exp_lut.hex: 1024 x Q1.15, entry i = exp((i - 1023) / 128)."""
    return np.array([min(65535, max(0, round(math.exp((i - 1023) / 128.0) * 32768))) for i in range(1024)],
                    np.uint16)


def silu_lut(scale=32.0):
    """silu_lut.hex: 65536 x int16 indexed by the 16-bit gate pattern, the gate
    and SiLU both Q1.15 at `scale` (same numpy expression as the generator)."""
    g = np.arange(65536, dtype=np.uint16).view(np.int16).astype(np.float64) / 32768.0 * scale
    s = g * (1.0 / (1.0 + np.exp(-g)))
    return np.clip(np.round(s * 32768.0 / scale).astype(np.int64), -32768, 32767).astype(np.int16)


def rope_freq_turns(base=10000.0, hd=64):
    """rope_freq_turns.svh: Q0.31 turns per position, round(base^(-2j/hd)/(2 pi) * 2^31)."""
    return np.array([round((1.0 / (base ** (2.0 * j / hd))) / (2.0 * math.pi) * (1 << 31)) for j in range(hd // 2)],
                    np.uint32)


def read_hex_rom(path, dtype=np.uint16):
    """A $readmemh file (one hex word per line, // comments)."""
    vals = [int(ln.split("//")[0].strip(), 16) for ln in open(path) if ln.split("//")[0].strip()]
    return np.array(vals, np.uint32).astype(np.uint16).view(np.int16 if dtype == np.int16 else np.uint16)


def read_freq_svh(path):
    return np.array([int(m) for m in re.findall(r"32'd\s*(\d+)", open(path).read())], np.uint32)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ---------------------------------------------------------------------------
# ops
# ---------------------------------------------------------------------------
def matvec(x_m, x_e, W_m, W_e):
    """matvec_bfp_engine.sv: x (..., NT, 16) / (..., NT); W (R, NT, 16) / (R, NT).
    Returns y_m (..., R) int16 and y_e (..., R) int8 (one exponent per element)."""
    W_m = _c(W_m, np.int16); W_e = _c(W_e, np.int8)
    R, NT = W_e.shape
    lead = np.shape(x_e)[:-1]
    xm = _c(x_m, np.int16).reshape(-1, NT * TILE); xe = _c(x_e, np.int8).reshape(-1, NT)
    B = xm.shape[0]
    ym = np.empty((B, R), np.int16); ye = np.empty((B, R), np.int8)
    check(_lib.lib().bfp200_rtl_matvec(context(), ptr(xm), ptr(xe), ptr(W_m), ptr(W_e), R, NT * TILE, B, ptr(ym),
                                       ptr(ye)))
    return ym.reshape(lead + (R,)), ye.reshape(lead + (R,))


def rmsnorm(x_m, x_e, g_m, g_e):
    """rmsnorm_bfp.sv: per vector (..., NT, 16); returns (m, e) in the same layout."""
    NT = np.shape(x_e)[-1]
    xm = _c(x_m, np.int16).reshape(-1, NT * TILE); xe = _c(x_e, np.int8).reshape(-1, NT)
    gm = np.broadcast_to(_c(g_m, np.int16).reshape(-1, NT * TILE), xm.shape).copy()
    ge = np.broadcast_to(_c(g_e, np.int8).reshape(-1, NT), xe.shape).copy()
    ym = np.empty_like(xm); ye = np.empty_like(xe)
    check(_lib.lib().bfp200_rtl_rmsnorm(context(), ptr(xm), ptr(xe), ptr(gm), ptr(ge), NT * TILE, xm.shape[0],
                                        ptr(ym), ptr(ye)))
    return ym.reshape(np.shape(x_m)), ye.reshape(np.shape(x_e))


def rope(x_m, x_e, pos, turns):
    """rope_bfp.sv: heads (..., HD/16, 16) at positions `pos` (broadcast to the
    leading shape).  Returns y_m (..., HD) and per-element y_e (..., HD)."""
    NTH = np.shape(x_e)[-1]
    HD = NTH * TILE
    lead = np.shape(x_e)[:-1]
    xm = _c(x_m, np.int16).reshape(-1, HD); xe = _c(x_e, np.int8).reshape(-1, NTH)
    p = _c(np.broadcast_to(np.asarray(pos), lead).reshape(-1), np.int32)
    t = _c(turns, np.uint32)
    assert t.size == HD // 2
    ym = np.empty_like(xm); ye = np.empty((xm.shape[0], HD), np.int8)
    check(_lib.lib().bfp200_rtl_rope(context(), ptr(xm), ptr(xe), ptr(p), xm.shape[0], HD, ptr(t), ptr(ym),
                                     ptr(ye)))
    return ym.reshape(lead + (HD,)), ye.reshape(lead + (HD,))


def softmax(x_m, x_e, lut=None):
    """softmax_bfp.sv: scores (..., n) sharing one exponent per vector x_e (...).
    Returns y_m (..., n) int16 and y_e (...) int."""
    lut = exp_lut() if lut is None else _c(lut, np.uint16)
    n = np.shape(x_m)[-1]
    lead = np.shape(x_m)[:-1]
    xm = _c(x_m, np.int16).reshape(-1, n)
    xe = _c(np.broadcast_to(np.asarray(x_e), lead).reshape(-1), np.int32)
    ym = np.empty_like(xm); ye = np.empty(xm.shape[0], np.int32)
    check(_lib.lib().bfp200_rtl_softmax(context(), ptr(xm), ptr(xe), n, xm.shape[0], ptr(lut), ptr(ym), ptr(ye)))
    return ym.reshape(lead + (n,)), ye.reshape(lead)


def swiglu(g_m, g_e, u_m, u_e, lut=None):
    """swiglu_bfp.sv: gate / up (..., NT, 16) + (..., NT); returns (m, e)."""
    lut = silu_lut() if lut is None else _c(lut, np.int16)
    gm = _c(g_m, np.int16).reshape(-1); um = _c(u_m, np.int16).reshape(-1)
    ge = _c(g_e, np.int8).reshape(-1); ue = _c(u_e, np.int8).reshape(-1)
    ym = np.empty_like(gm); ye = np.empty_like(ge)
    check(_lib.lib().bfp200_rtl_swiglu(context(), ptr(gm), ptr(ge), ptr(um), ptr(ue), gm.size, ptr(lut), ptr(ym),
                                       ptr(ye)))
    return ym.reshape(np.shape(g_m)), ye.reshape(np.shape(g_e))


def residual(a_m, a_e, b_m, b_e):
    """Tile-aligned residual add: (..., NT, 16) + (..., NT); returns (m, e)."""
    am = _c(a_m, np.int16).reshape(-1); bm = _c(b_m, np.int16).reshape(-1)
    ae = _c(a_e, np.int8).reshape(-1); be = _c(b_e, np.int8).reshape(-1)
    ym = np.empty_like(am); ye = np.empty_like(ae)
    check(_lib.lib().bfp200_rtl_residual(context(), ptr(am), ptr(ae), ptr(bm), ptr(be), am.size, ptr(ym), ptr(ye)))
    return ym.reshape(np.shape(a_m)), ye.reshape(np.shape(a_e))


__all__ = ["exp_lut", "silu_lut", "rope_freq_turns", "read_hex_rom", "read_freq_svh", "matvec", "rmsnorm", "rope",
           "softmax", "swiglu", "residual"]
