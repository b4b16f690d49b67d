"""numpy restatement of the reference's bit-exact BFP simulator (TEST ONLY).

Reference: jrrk2/tinyllm-fpga, rtl/vc707/host/gen_smollm_blockfp_full.py
(twin: rtl/vc707/host/sim_rtl_fp_hw.py:28-145).  Every function below cites
the lines it restates.  The restatement keeps the reference's arithmetic
(numpy float64 / int64, same operation order, same pairwise reductions) and
only vectorises where that provably cannot change a bit:

* matvec tile sums are formed with float64 BLAS: each tile sum is at most
  16 * 2^30 = 2^34 in magnitude, so every partial sum is an exact integer
  in float64 whatever the order or FMA use;
* the attention score ``np.dot(q_h, k_t)`` is computed EXACTLY (integer
  tile-pair sums, one rounding).  The reference's BLAS dot equals this
  exact value whenever the tile-pair exponent spread is <= 17 (all partial
  sums then fit 53 bits); wider spreads are counted in ``STATS`` so tests can
  report them;
* the per-position attention accumulation ``attn += sm[t] * v`` stays a
  sequential loop over t (vectorised only across the independent lanes).

This module is the checker.  The product never imports it.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

TILE = 16            # gen_smollm_blockfp_full.py:65
ALIGN_MAX = 47       # gen_smollm_blockfp_full.py:214
SAT_HI = (1 << 47) - 1   # :229
SAT_LO = -(1 << 47)      # :230

STATS = {"score_dots": 0, "score_dots_wide_spread": 0}


# ---------------------------------------------------------------------------
# a2/a3: tile_quantize / tile_decode / fp_quantize_vec  (:90-107)
# ---------------------------------------------------------------------------
def tile_quantize(v):
    """gen_smollm_blockfp_full.py:90-97 -- per-16 shared exponent, int16 mantissa."""
    flat = np.asarray(v, dtype=np.float64).reshape(-1, TILE)
    max_abs = np.maximum(np.abs(flat).max(axis=1), 1e-300)
    e = (np.floor(np.log2(max_abs)).astype(np.int32) + 1).clip(-127, 127)
    m_scale = np.power(2.0, e.astype(np.float64))[:, None]
    m = np.clip(np.round(flat / m_scale * 32768.0).astype(np.int64), -32768, 32767)
    return m.astype(np.int16), e.astype(np.int8)


def tile_decode(m_int, e_int):
    """gen_smollm_blockfp_full.py:100-102."""
    m_scale = np.power(2.0, np.asarray(e_int).astype(np.float64))[:, None]
    return ((np.asarray(m_int).reshape(-1, TILE).astype(np.float64) / 32768.0) * m_scale).flatten()


def fp_quantize_vec(v):
    """gen_smollm_blockfp_full.py:105-107."""
    m, e = tile_quantize(v)
    return tile_decode(m, e)


def quantize_W(W):
    """gen_smollm_blockfp_full.py:110-119 (row loop vectorised: a row's tiles
    are consecutive 16-element groups, so flat tiling is identical)."""
    W = np.asarray(W, dtype=np.float64)
    D_out, D_in = W.shape
    assert D_in % TILE == 0
    m, e = tile_quantize(W.reshape(-1))
    return m.reshape(D_out, D_in // TILE, TILE), e.reshape(D_out, D_in // TILE)


def floor_log2_threshold_counts(lo=-130, hi=130):
    """For every integer j in [lo, hi]: how many doubles directly below 2^j
    does this host's ``np.log2`` round up to exactly j.  Used by tests to pin
    the GPU's emulation of ``floor(np.log2(max_abs))`` (:93)."""
    out = {}
    for j in range(lo, hi + 1):
        y = np.ldexp(1.0, j)
        n = 0
        while n < 1000:
            y = np.nextafter(y, 0.0)
            if np.floor(np.log2(np.array([y])))[0] >= j:
                n += 1
            else:
                break
        out[j] = n
    return out


# ---------------------------------------------------------------------------
# a5: matvec_hw_golden (:217-233)
# ---------------------------------------------------------------------------
def _align_accumulate(tile_sums, tile_exps):
    """Steps 3-6 of :221-232 on int64 arrays with tiles on the last axis."""
    max_e = tile_exps.max(axis=-1, keepdims=True)
    shift = max_e - tile_exps
    mask = shift <= ALIGN_MAX
    aligned = np.right_shift(tile_sums, np.clip(shift, 0, 63))
    aligned = np.where(mask, aligned, 0)
    acc = np.clip(aligned.sum(axis=-1), SAT_LO, SAT_HI)
    return acc, max_e[..., 0]


def matvec_acc(x_m, x_e, W_m, W_e):
    """Integer part of :217-231: returns (acc int64 [D_out], max_e int64 [D_out])."""
    prods = x_m[None, :, :].astype(np.int64) * W_m.astype(np.int64)
    tile_sums = prods.sum(axis=2)
    tile_exps = x_e[None, :].astype(np.int64) + W_e.astype(np.int64)
    return _align_accumulate(tile_sums, tile_exps)


def matvec_hw_golden(x_m, x_e, W_m, W_e):
    """gen_smollm_blockfp_full.py:217-233, literal restatement."""
    acc, max_e = matvec_acc(x_m, x_e, W_m, W_e)
    out_real = acc.astype(np.float64) * np.power(2.0, max_e.astype(np.float64) - 30)
    return fp_quantize_vec(out_real)


def matvec_cols(X_m, X_e, W_m, W_e, Wf=None):
    """:217-233 applied independently to B columns.

    X_m (B, NT, 16) int16, X_e (B, NT) int8 -> out (B, D_out) float64 on the
    BFP grid.  Tile sums use float64 BLAS (exact: |sum| <= 2^34)."""
    X_m = np.asarray(X_m)
    B, NT, _ = X_m.shape
    D_out = W_m.shape[0]
    if Wf is None:
        Wf = np.ascontiguousarray(W_m.astype(np.float64).transpose(1, 0, 2))  # (NT, D_out, 16)
    Xf = X_m.astype(np.float64).transpose(1, 2, 0)                            # (NT, 16, B)
    ts = np.matmul(Wf, Xf)                                                      # (NT, D_out, B)
    tile_sums = ts.transpose(2, 1, 0).astype(np.int64)                          # (B, D_out, NT)
    tile_exps = X_e.astype(np.int64)[:, None, :] + W_e.astype(np.int64)[None, :, :]
    acc, max_e = _align_accumulate(tile_sums, tile_exps)
    out_real = acc.astype(np.float64) * np.power(2.0, max_e.astype(np.float64) - 30)
    return fp_quantize_vec(out_real.reshape(-1)).reshape(B, D_out)


# ---------------------------------------------------------------------------
# a6/a10/a11: rmsnorm_fp, softmax_fp, silu_fp (:236-247)
# ---------------------------------------------------------------------------
def rmsnorm_fp(x, gamma, eps=1e-5):
    """:236-238.  np.mean is numpy's pairwise sum / n; x*gamma/s left to right."""
    v = np.mean(x * x) + eps
    return fp_quantize_vec(x * gamma / np.sqrt(v))


def silu_fp(x):
    """:241-242."""
    return fp_quantize_vec(x / (1.0 + np.exp(-x)))


def softmax_fp(x):
    """:245-247 (not quantized)."""
    e = np.exp(x - x.max())
    return e / e.sum()


# ---------------------------------------------------------------------------
# a7: rope_fp (:250-258)
# ---------------------------------------------------------------------------
def rope_cos_sin(pos, HD=64, base=10000.0):
    """The (cos, sin) pairs :253-254 evaluates with Python's math module."""
    H2 = HD // 2
    c = np.empty(H2)
    s = np.empty(H2)
    for j in range(H2):
        theta = 1.0 / (base ** (2 * j / HD)) * pos
        c[j] = math.cos(theta)
        s[j] = math.sin(theta)
    return c, s


def rope_fp(x, pos, base=10000.0, HD=64, cs=None):
    """:250-258: out[j] = a*c - b*s ; out[j+H2] = b*c + a*s ; then fpq."""
    H2 = HD // 2
    c, s = cs if cs is not None else rope_cos_sin(pos, HD, base)
    x = np.asarray(x, dtype=np.float64)
    a, b = x[:H2], x[H2:]
    out = np.empty(HD)
    out[:H2] = a * c - b * s
    out[H2:] = b * c + a * s
    return fp_quantize_vec(out)


# ---------------------------------------------------------------------------
# exact attention score (restates float(np.dot(q, k)) / math.sqrt(HD), :278)
# ---------------------------------------------------------------------------
def _grid_int(v):
    """Exact integer form of a vector of BFP grid values: v = M * 2^E per tile,
    |M| <= 2^16.  E = (requantized tile exponent) - 16 covers both the plain
    and the -32768 (exponent-bumped) case."""
    _, e = tile_quantize(v)
    E = e.astype(np.int64) - 16
    M = np.asarray(v, dtype=np.float64).reshape(-1, TILE) * np.power(2.0, -E.astype(np.float64))[:, None]
    Mi = M.astype(np.int64)
    assert np.array_equal(Mi.astype(np.float64), M), "value not on the BFP grid"
    return Mi, E


def exact_scores(q, K):
    """q (HD,) and K (T, HD) on the BFP grid -> float64 [T] = round(q.K_t) / 8.

    Exact integer tile-pair sums, combined exactly, rounded once.  Equal to the
    reference's BLAS dot whenever the pair-exponent spread is <= 17."""
    T, HD = K.shape
    qM, qE = _grid_int(q)                                   # (nt,16), (nt,)
    KM, KE = _grid_int(K.reshape(-1))
    nt = HD // TILE
    KM = KM.reshape(T, nt, TILE)
    KE = KE.reshape(T, nt)
    S = (KM * qM[None]).sum(axis=2)                         # (T, nt) int64, |S| < 2^37
    E = KE + qE[None]
    nz = S != 0
    Emax = np.where(nz, E, -10**6).max(axis=1)
    Emin = np.where(nz, E, 10**6).min(axis=1)
    spread = np.where(nz.any(axis=1), Emax - Emin, 0)
    out = (S.astype(np.float64) * np.power(2.0, E.astype(np.float64))).sum(axis=1)
    wide = spread > 15
    STATS["score_dots"] += T
    if wide.any():
        STATS["score_dots_wide_spread"] += int(wide.sum())
        from fractions import Fraction
        for t in np.nonzero(wide)[0]:
            acc = Fraction(0)
            for j in range(nt):
                if S[t, j]:
                    acc += Fraction(int(S[t, j])) * (Fraction(2) ** int(E[t, j]))
            out[t] = float(acc)
    return out / math.sqrt(HD)


# ---------------------------------------------------------------------------
# a13: fwd_layer (:261-293)
# ---------------------------------------------------------------------------
@dataclass
class Cfg:
    D: int = 576
    H_Q: int = 9
    H_KV: int = 3
    HD: int = 64
    FFN: int = 1536
    NL: int = 30
    VOCAB: int = 49152
    rope_base: float = 10000.0
    eps: float = 1e-5


def new_kv(cfg: Cfg, max_ctx: int):
    """:426-428 -- one float64 K/V cache per layer."""
    return [{"k": np.zeros((max_ctx, cfg.H_KV, cfg.HD)), "v": np.zeros((max_ctx, cfg.H_KV, cfg.HD))}
            for _ in range(cfg.NL)]


def attention(q, kv, kv_pos, cfg: Cfg):
    """:273-282: per head, exact scores, softmax_fp, sequential accumulation."""
    grp = cfg.H_Q // cfg.H_KV
    HD = cfg.HD
    T = kv_pos + 1
    attn = np.zeros((cfg.H_Q, HD))
    sm_all = np.empty((cfg.H_Q, T))
    for h_i in range(cfg.H_Q):
        kvh = h_i // grp
        scores = exact_scores(q[h_i * HD:(h_i + 1) * HD], kv["k"][:T, kvh])
        sm_all[h_i] = softmax_fp(scores)
    V = kv["v"][:T]                                  # (T, H_KV, HD)
    kvmap = np.arange(cfg.H_Q) // grp
    for t in range(T):                               # attn[h] += sm[t] * v  (:280-281)
        attn += sm_all[:, t, None] * V[t, kvmap]
    return fp_quantize_vec(attn.reshape(-1))          # :282


def fwd_layer(h, lw, pos, kv, kv_pos, cfg: Cfg = Cfg(), stages=None, cs=None):
    """gen_smollm_blockfp_full.py:261-293.  ``lw`` holds 'Wq'..'Wd' as (m, e)
    tuples and 'g1','g2' as float64 vectors (plus optional cached 'Wf_*').
    If ``stages`` is a dict, intermediate tensors are recorded in it."""
    HD = cfg.HD
    if cs is None:
        cs = rope_cos_sin(pos, HD, cfg.rope_base)
    n1 = rmsnorm_fp(h, lw["g1"], cfg.eps)
    n1_m, n1_e = tile_quantize(n1)
    q = _mv(n1_m, n1_e, lw, "Wq")
    k = _mv(n1_m, n1_e, lw, "Wk")
    v = _mv(n1_m, n1_e, lw, "Wv")
    if stages is not None:
        stages.update(n1=n1, q_pre=q.copy(), k_pre=k.copy(), v=v.copy())
    for h_i in range(cfg.H_Q):
        q[h_i * HD:(h_i + 1) * HD] = rope_fp(q[h_i * HD:(h_i + 1) * HD], pos, cfg.rope_base, HD, cs)
    for h_i in range(cfg.H_KV):
        k[h_i * HD:(h_i + 1) * HD] = rope_fp(k[h_i * HD:(h_i + 1) * HD], pos, cfg.rope_base, HD, cs)
    for h_i in range(cfg.H_KV):
        kv["k"][kv_pos, h_i] = k[h_i * HD:(h_i + 1) * HD]
        kv["v"][kv_pos, h_i] = v[h_i * HD:(h_i + 1) * HD]
    attn = attention(q, kv, kv_pos, cfg)
    a_m, a_e = tile_quantize(attn)
    o = _mv(a_m, a_e, lw, "Wo")
    h1 = fp_quantize_vec(h + o)
    n2 = rmsnorm_fp(h1, lw["g2"], cfg.eps)
    n2_m, n2_e = tile_quantize(n2)
    g_vec = _mv(n2_m, n2_e, lw, "Wg")
    u_vec = _mv(n2_m, n2_e, lw, "Wu")
    mlp = fp_quantize_vec(silu_fp(g_vec) * u_vec)
    mlp_m, mlp_e = tile_quantize(mlp)
    d_vec = _mv(mlp_m, mlp_e, lw, "Wd")
    out = fp_quantize_vec(h1 + d_vec)
    if stages is not None:
        stages.update(q=q, k=k, attn=attn, o=o, h1=h1, n2=n2, g=g_vec, u=u_vec,
                      mlp=mlp, d=d_vec, out=out)
    return out


def _mv(x_m, x_e, lw, name):
    m, e = lw[name]
    wf = lw.get("Wf_" + name)
    return matvec_cols(x_m[None], x_e[None], m, e, wf)[0]


# ---------------------------------------------------------------------------
# a14-a16: embedding, head + greedy, driver loop (:411-443)
# ---------------------------------------------------------------------------
def head_logits(h, norm_w_q, embed, eps=1e-5):
    """:438-439: ((h / sqrt(mean(h*h) + 1e-5)) * norm_w_q) @ embed.T (float64)."""
    h_normed = (h / np.sqrt(np.mean(h * h) + eps)) * norm_w_q
    return h_normed @ embed.T


def sample_token(logits, T, topk, rng):
    """sim_rtl_fp_hw.py:206-216: temperature / top-k sampling of one token
    with the legacy numpy generator `rng` (np.random.RandomState)."""
    if not T > 0:
        return int(np.argmax(logits))
    scaled = logits / T
    if topk > 0:
        idx = np.argsort(scaled)[-topk:]
        mask = np.full_like(scaled, -np.inf)
        mask[idx] = scaled[idx]
        scaled = mask
    scaled -= scaled.max()
    p = np.exp(scaled)
    p = p / p.sum()
    return int(rng.choice(len(p), p=p))


def generate_sampled(model, ids, n_gen, T, topk, seed, max_ctx=None, cfg: Cfg = Cfg()):
    """The sampling driver loop of sim_rtl_fp_hw.py:196-219 on this model:
    np.random.seed(SEED) stream, a token drawn at every step >= len(ids)-1
    (the first one discarded, as in the greedy loop :437-443), feed rule
    'sim'.  Returns prompt + n_gen ids."""
    rng = np.random.RandomState(seed)
    ids = [int(t) for t in ids]
    n_steps = len(ids) + n_gen
    kv = new_kv(cfg, n_steps if max_ctx is None else max_ctx)
    generated = list(ids)
    for step in range(n_steps):
        tid = ids[step] if step < len(ids) else generated[-1]
        h = model.embed_q(tid)
        cs = rope_cos_sin(step, cfg.HD, cfg.rope_base)
        for li in range(cfg.NL):
            h = fwd_layer(h, model.layers[li], pos=step, kv=kv[li], kv_pos=step, cfg=cfg, cs=cs)
        if step >= len(ids) - 1:
            nid = sample_token(head_logits(h, model.norm_w_q, model.embed, cfg.eps), T, topk, rng)
            if step >= len(ids):
                generated.append(nid)
    return generated


def generate(model, ids, n_gen, max_ctx=None, feed_mode="sim", cfg: Cfg = Cfg(), trace=None):
    """gen_smollm_blockfp_full.py:425-449 (feed_mode='sim', default) or the
    RTL feed rule of autoregress_bfp_top.sv:358-384 (feed_mode='rtl').

    sim: returns prompt + n_gen ids; the argmax at step len(ids)-1 is
         discarded and step len(ids) re-feeds the last prompt token.
    rtl: returns one argmax per step (len(ids) + n_gen ids); step >= len(ids)
         feeds the previous step's argmax.
    """
    ids = [int(t) for t in ids]
    n_steps = len(ids) + n_gen
    if max_ctx is None:
        max_ctx = n_steps
    assert max_ctx >= n_steps
    kv = new_kv(cfg, max_ctx)
    generated = list(ids)
    rtl_out = []
    last = 0
    for step in range(n_steps):
        if feed_mode == "sim":
            tid = ids[step] if step < len(ids) else generated[-1]
        else:
            tid = ids[step] if step < len(ids) else last
        h = model.embed_q(tid)
        cs = rope_cos_sin(step, cfg.HD, cfg.rope_base)
        for li in range(cfg.NL):
            h = fwd_layer(h, model.layers[li], pos=step, kv=kv[li], kv_pos=step, cfg=cfg, cs=cs)
        if trace is not None:
            trace.append(h.copy())
        if feed_mode == "sim":
            if step >= len(ids) - 1:
                nid = int(np.argmax(head_logits(h, model.norm_w_q, model.embed, cfg.eps)))
                if step >= len(ids):
                    generated.append(nid)
        else:
            last = int(np.argmax(head_logits(h, model.norm_w_q, model.embed, cfg.eps)))
            rtl_out.append(last)
    return generated if feed_mode == "sim" else rtl_out
