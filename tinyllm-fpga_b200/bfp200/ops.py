"""Op-level GPU entry points: the reference simulator's module functions
(rtl/vc707/host/gen_smollm_blockfp_full.py:90-258) computed by libbfp200.

All functions take and return numpy arrays (host memory), like the
reference.  They run on one process-wide handle opened on device
$BFP200_DEVICE (default 0); there is no CPU path.
"""
from __future__ import annotations

import os
import threading

import numpy as np

from . import _lib
from ._lib import arr, check, ptr

TILE = 16
_ctx = None
_ctx_lock = threading.Lock()


def context():
    """The process-wide op handle (small config; ops do not need an image)."""
    global _ctx
    with _ctx_lock:
        if _ctx is None:
            L = _lib.lib()
            c = _lib.Cfg()
            L.bfp200_default_cfg(c)
            c.D, c.H_Q, c.H_KV, c.FFN, c.NL, c.VOCAB, c.MAX_CTX, c.max_seqs = 64, 1, 1, 64, 1, 16, 16, 1
            h = _lib.C.c_void_p()
            check(L.bfp200_open(_lib.C.byref(c), int(os.environ.get("BFP200_DEVICE", "0")), _lib.C.byref(h)))
            _ctx = h
        return _ctx


def tile_quantize(v):
    """tile_quantize (:90-97) -> (m (n/16, 16) int16, e (n/16,) int8)."""
    v = arr(v, np.float64).reshape(-1)
    n = v.size
    if n % TILE:
        raise ValueError("length must be a multiple of 16")
    m = np.empty(n, np.int16)
    e = np.empty(n // TILE, np.int8)
    check(_lib.lib().bfp200_tile_quantize(context(), ptr(v), n, ptr(m), ptr(e)))
    return m.reshape(-1, TILE), e


def tile_decode(m_int, e_int):
    """tile_decode (:100-102) -> float64 vector."""
    m = arr(m_int, np.int16).reshape(-1)
    e = arr(e_int, np.int8).reshape(-1)
    if m.size != e.size * TILE:
        raise ValueError("need 16 mantissas per exponent")
    out = np.empty(m.size, np.float64)
    check(_lib.lib().bfp200_tile_decode(context(), ptr(m), ptr(e), m.size, ptr(out)))
    return out


def fp_quantize_vec(v):
    """fp_quantize_vec (:105-107)."""
    m, e = tile_quantize(v)
    return tile_decode(m, e)


def matvec(X_m, X_e, W_m, W_e):
    """matvec_hw_golden (:217-233) on B columns.
    X_m (B, NT, 16) int16, X_e (B, NT) int8; W_m (D_out, NT, 16), W_e (D_out, NT).
    Returns (m (B, D_out), e (B, D_out/16)) = tile_quantize of the outputs."""
    W_m = arr(W_m, np.int16)
    W_e = arr(W_e, np.int8)
    D_out, NT = W_e.shape
    X_m = arr(X_m, np.int16).reshape(-1, NT * TILE)
    B = X_m.shape[0]
    X_e = arr(X_e, np.int8).reshape(B, NT)
    om = np.empty((B, D_out), np.int16)
    oe = np.empty((B, D_out // TILE), np.int8)
    check(_lib.lib().bfp200_matvec(context(), ptr(X_m), ptr(X_e), ptr(W_m), ptr(W_e), D_out, NT * TILE, B,
                                   ptr(om), ptr(oe)))
    return om, oe


def matvec_timed(X_m, X_e, W_m, W_e, reps=20):
    """matvec plus its device time: (m, e, ms per call averaged over `reps`
    back-to-back launches after one untimed call)."""
    W_m = arr(W_m, np.int16)
    W_e = arr(W_e, np.int8)
    D_out, NT = W_e.shape
    X_m = arr(X_m, np.int16).reshape(-1, NT * TILE)
    B = X_m.shape[0]
    X_e = arr(X_e, np.int8).reshape(B, NT)
    om = np.empty((B, D_out), np.int16)
    oe = np.empty((B, D_out // TILE), np.int8)
    ms = _lib.C.c_double()
    check(_lib.lib().bfp200_matvec_timed(context(), ptr(X_m), ptr(X_e), ptr(W_m), ptr(W_e), D_out, NT * TILE, B,
                                         int(reps), ptr(om), ptr(oe), _lib.C.byref(ms)))
    return om, oe, ms.value


def matvec_hw_golden(x_m, x_e, W_m, W_e):
    """Drop-in for the reference's matvec_hw_golden: one column, returns the
    float64 vector fp_quantize_vec(out_real)."""
    om, oe = matvec(np.asarray(x_m)[None], np.asarray(x_e)[None], W_m, W_e)
    return tile_decode(om[0], oe[0])


def rmsnorm_fp(x, gamma, eps=1e-5):
    """rmsnorm_fp (:236-238); x may be (n,) or (ncols, n)."""
    x = arr(x, np.float64)
    one = x.ndim == 1
    x2 = x.reshape(1, -1) if one else x
    g = arr(gamma, np.float64).reshape(-1)
    out = np.empty_like(x2)
    check(_lib.lib().bfp200_rmsnorm_fp(context(), ptr(x2), ptr(g), x2.shape[1], x2.shape[0], float(eps), ptr(out)))
    return out[0] if one else out


def silu_fp(x):
    """silu_fp (:241-242)."""
    x = arr(x, np.float64)
    out = np.empty_like(x)
    check(_lib.lib().bfp200_silu_fp(context(), ptr(x), x.size, ptr(out)))
    return out


def softmax_fp(x):
    """softmax_fp (:245-247); x may be (n,) or (ncols, n)."""
    x = arr(x, np.float64)
    one = x.ndim == 1
    x2 = x.reshape(1, -1) if one else x
    out = np.empty_like(x2)
    check(_lib.lib().bfp200_softmax_fp(context(), ptr(x2), x2.shape[1], x2.shape[0], ptr(out)))
    return out[0] if one else out


def pairwise_sum(x):
    """numpy's float64 np.add.reduce along the last axis (pairwise summation)."""
    x = arr(x, np.float64)
    x2 = x.reshape(-1, x.shape[-1])
    out = np.empty(x2.shape[0], np.float64)
    check(_lib.lib().bfp200_pairwise_sum(context(), ptr(x2), x2.shape[1], x2.shape[0], ptr(out)))
    return out.reshape(x.shape[:-1])


def rope_fp(x, pos, base=10000.0):
    """rope_fp (:250-258); x (HD,) or (nvec, HD) with pos scalar or (nvec,)."""
    x = arr(x, np.float64)
    one = x.ndim == 1
    x2 = x.reshape(1, -1) if one else x
    p = arr(np.broadcast_to(np.asarray(pos), (x2.shape[0],)), np.int32)
    out = np.empty_like(x2)
    check(_lib.lib().bfp200_rope_fp(context(), ptr(x2), ptr(p), x2.shape[0], x2.shape[1], float(base), ptr(out)))
    return out[0] if one else out


def rope_table(n_pos, HD=64, base=10000.0):
    """(cos, sin) pairs of rope_fp (:253-254): array (n_pos, HD/2, 2).
    Host computation (same libm as Python's math module); no GPU needed."""
    out = np.empty((n_pos, HD // 2, 2), np.float64)
    check(_lib.lib().bfp200_rope_table(ptr(out), n_pos, HD, float(base)))
    return out
