// bfp_device.cuh -- device-side arithmetic that reproduces the reference BFP
// simulator bit for bit (jrrk2/tinyllm-fpga rtl/vc707/host/
// gen_smollm_blockfp_full.py).  Everything here is exact IEEE-754 double or
// integer arithmetic; the file must be compiled with -fmad=false so no
// multiply/add pair is contracted into an FMA the simulator never performs.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace bfp {

constexpr int TILE = 16;        // elements per shared exponent (bfp_format.svh:1-27)
constexpr int ALIGN_MAX = 47;   // gen_smollm_blockfp_full.py:214
constexpr long long SAT_HI = (1LL << 47) - 1;   // :229
constexpr long long SAT_LO = -(1LL << 47);      // :230

// 2^k as a double, exact for k in [-1022, 1023].
__host__ __device__ __forceinline__ double pow2(int k) {
#ifdef __CUDA_ARCH__
  return __longlong_as_double((long long)(k + 1023) << 52);
#else
  union { long long i; double d; } u;
  u.i = (long long)(k + 1023) << 52;
  return u.d;
#endif
}

__host__ __device__ __forceinline__ int ilog2_u32(unsigned v) {
#ifdef __CUDA_ARCH__
  return 31 - __clz((int)v);
#else
  return 31 - __builtin_clz(v);
#endif
}

__host__ __device__ __forceinline__ unsigned long long dbits(double x) {
#ifdef __CUDA_ARCH__
  return (unsigned long long)__double_as_longlong(x);
#else
  union { double d; unsigned long long i; } u; u.d = x;
  return u.i;
#endif
}

// Number of doubles directly below 2^j that a correctly rounded log2 maps to
// exactly j (so floor(log2(x)) jumps to j before x reaches 2^j):
// log2(2^j (1 - n 2^-53)) = j - n 2^-53 / ln 2 rounds to j while n < ln2 * 2^b,
// b the ulp exponent of the result's binade, i.e. n = floor(ln2 * 2^b) =
// 0xB17217F7 >> (32 - b) (ln 2 in 0.32 fixed point; no fractional part of
// ln2 * 2^b is close enough to an integer for the truncation to matter).
// numpy's float64 log2 follows this exactly (checked by the tests on every
// host that generates or compares golden data).
__host__ __device__ __forceinline__ unsigned log2_roundup_count(int j) {
  const unsigned aj = (unsigned)(j < 0 ? -j : j);
  const int a = aj ? ilog2_u32(aj) : 0;
  const int b = a - ((j > 0 && (aj & (aj - 1)) == 0) ? 1 : 0);
  return (j != 0 && b >= 1) ? (0xB17217F7u >> (32 - b)) : 0u;
}

// Tile exponent of tile_quantize (:92-93) from the bit pattern of the tile's
// max |v| (sign cleared): e = clip(floor(np.log2(max(max_abs, 1e-300))) + 1).
// NaN/Inf follow numpy's x86 cast (INT32_MIN + 1, clipped to -127).  32-bit
// arithmetic on the two halves of the pattern.
__host__ __device__ __forceinline__ int tile_exponent_bits(unsigned long long abits) {
  unsigned hi = (unsigned)(abits >> 32), lo = (unsigned)abits;
  if (hi >= 0x7FF00000u) return -127;
  constexpr unsigned FHI = 0x01a56e1fu, FLO = 0xc2f8f359u;        // bits of 1e-300
  if (hi < FHI || (hi == FHI && lo < FLO)) { hi = FHI; lo = FLO; }
  const int k = (int)(hi >> 20) - 1023;                           // x in [2^k, 2^(k+1))
  const unsigned n = log2_roundup_count(k + 1);
  // fraction F >= 2^52 - n  (n < 2^10): top 20 fraction bits all ones and lo >= 2^32 - n
  const bool up = n > 0 && (hi & 0xFFFFFu) == 0xFFFFFu && lo >= 0u - n;
  const int e = k + (up ? 1 : 0) + 1;
  return e < -127 ? -127 : (e > 127 ? 127 : e);
}

__host__ __device__ __forceinline__ int tile_exponent(double max_abs) {
  return tile_exponent_bits(dbits(max_abs) & 0x7FFFFFFFFFFFFFFFULL);
}

// Mantissa of tile_quantize (:94-96): clip(rint(v / 2^e * 32768)), from v's
// bit pattern: the 53-bit significand shifted right by >= 37 bits with
// round-half-even, so only its high word enters the quotient.  Values whose
// int64 cast is undefined in numpy (NaN, Inf, |x| >= 2^63) give x86's
// INT64_MIN, i.e. -32768 after the clip.
__host__ __device__ __forceinline__ int16_t tile_mantissa_bits(unsigned long long vb, int e) {
  // computed without branches: the general case with the shift clamped to
  // its valid range, then the special cases selected in increasing precedence
  const unsigned hi = (unsigned)(vb >> 32), lo = (unsigned)vb;
  const int ex = (int)((hi >> 20) & 0x7FF);
  const bool neg = (hi >> 31) != 0;
  const int p = ex - 1023 + 15 - e;                          // x = +-M * 2^(p - 52)
  const int sh = p > 15 ? 5 : (p < -1 ? 21 : 20 - p);       // 52 - p - 32, clamped to 5 .. 21
  const unsigned Mh = (hi & 0xFFFFFu) | 0x100000u;           // significand bits 32..52
  unsigned q = Mh >> sh;
  const unsigned rh = Mh & ((1u << sh) - 1u), hh = 1u << (sh - 1);
  const bool above = rh > hh || (rh == hh && lo != 0u);
  const bool tie = rh == hh && lo == 0u;
  q += (above || (tie && (q & 1u))) ? 1u : 0u;
  int val = neg ? -(int)q : (int)q;
  val = val > 32767 ? 32767 : (val < -32768 ? -32768 : val);
  val = p <= -2 ? 0 : val;                                   // |x| < 0.5
  val = p >= 16 ? (neg ? -32768 : 32767) : val;              // saturation
  val = p >= 63 ? -32768 : val;                              // int64 cast overflow (x86 INT64_MIN)
  val = ex == 0 ? 0 : val;                                   // zero / subnormal: |x| < 2^-880
  val = ex == 0x7FF ? -32768 : val;                          // NaN / Inf
  return (int16_t)val;
}

__host__ __device__ __forceinline__ int16_t tile_mantissa(double v, int e) { return tile_mantissa_bits(dbits(v), e); }

// tile_decode (:100-102): m/32768 * 2^e, exact.
__host__ __device__ __forceinline__ double bfp_decode(int m, int e) {
  return (double)m * pow2(e - 15);
}

// tile_quantize applied to a grid value already held as (m, e): identity
// unless the tile holds -32768 (decoded -2^e), which bumps the exponent and
// halves every mantissa with round-half-even.  `has_min` = tile contains
// -32768.
__host__ __device__ __forceinline__ int requant_exp(int e, bool has_min) {
  return (has_min && e < 127) ? e + 1 : e;
}
__host__ __device__ __forceinline__ int16_t requant_mant(int m, bool bumped) {
  if (!bumped) return (int16_t)m;
  int k = m >> 1;                       // floor(m / 2)
  int odd = m & 1;                      // m/2 = k + 0.5 when odd -> round half to even
  return (int16_t)(k + (odd & (k & 1)));
}

#ifdef __CUDACC__
// ---------------------------------------------------------------------------
// Cooperative tile quantize: 16 consecutive lanes hold one tile (lane & 15 =
// element index).  Returns this lane's mantissa; *e_out gets the exponent.
// ---------------------------------------------------------------------------
// N independent tiles per 16-lane group quantized together.
//
// The tile exponent needs max|v| only through its exponent field, except in
// numpy's log2 round-up case, where the max element's top 20 fraction bits
// are all ones (tile_exponent_bits).  So the group maximum of the biased
// exponent fields is taken with two 32-bit warp reductions (one per half
// warp), and only when some lane holding that exponent has all-ones top
// fraction bits does the warp take the exact 64-bit shuffle maximum.
template <int N>
__device__ __forceinline__ void tile_quantize_16lanes_exact_n(const unsigned long long (&vb)[N], int (&e)[N]) {
  unsigned long long a[N];
  #pragma unroll
  for (int i = 0; i < N; ++i) a[i] = vb[i] & 0x7FFFFFFFFFFFFFFFULL;
  // max |v| over the 16 lanes as an unsigned max of the sign-cleared bit
  // patterns (the order of |v| for finite values; NaN > Inf > finite, so a
  // NaN propagates like np.max)
  #pragma unroll
  for (int off = 8; off >= 1; off >>= 1) {
    #pragma unroll
    for (int i = 0; i < N; ++i) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, a[i], off, 16);
      a[i] = o > a[i] ? o : a[i];
    }
  }
  #pragma unroll
  for (int i = 0; i < N; ++i) e[i] = tile_exponent_bits(a[i]);
}

template <int N>
__device__ __forceinline__ void tile_quantize_16lanes_n(const double (&v)[N], int16_t (&m)[N], int (&e)[N]) {
  const bool upper = (threadIdx.x & 16) != 0;
  unsigned long long vb[N];
  bool round_up_case = false;
  #pragma unroll
  for (int i = 0; i < N; ++i) {
    vb[i] = dbits(v[i]);
    const unsigned hi = (unsigned)(vb[i] >> 32);
    const unsigned bx = (hi >> 20) & 0x7FFu;                        // biased exponent field
    const unsigned r0 = __reduce_max_sync(0xffffffffu, upper ? 0u : bx);
    const unsigned r1 = __reduce_max_sync(0xffffffffu, upper ? bx : 0u);
    const unsigned kmax = upper ? r1 : r0;
    // NaN / Inf in the tile (field 0x7FF): exponent -127 whatever the fraction
    e[i] = kmax == 0x7FFu ? -127 : min(max((int)kmax - 1022, -127), 127);
    round_up_case |= kmax != 0x7FFu && bx == kmax && (hi & 0xFFFFFu) == 0xFFFFFu;
  }
  if (__any_sync(0xffffffffu, round_up_case)) tile_quantize_16lanes_exact_n<N>(vb, e);
  #pragma unroll
  for (int i = 0; i < N; ++i) m[i] = tile_mantissa_bits(vb[i], e[i]);
}

// tile_quantize of fpq(v) for N tiles at once: the matvec-ready form (a tile
// holding -32768 bumps its exponent and halves its mantissas).
template <int N>
__device__ __forceinline__ void tile_quantize_requant_16lanes_n(const double (&v)[N], const bool (&valid)[N],
                                                                int16_t (&m)[N], int (&e)[N]) {
  tile_quantize_16lanes_n<N>(v, m, e);
  const int lane = threadIdx.x & 31;
  #pragma unroll
  for (int i = 0; i < N; ++i) {
    const unsigned bal = __ballot_sync(0xffffffffu, valid[i] && m[i] == (int16_t)-32768);
    const bool has_min = ((bal >> (lane & 16)) & 0xFFFFu) != 0;
    m[i] = requant_mant(m[i], has_min && e[i] < 127);
    e[i] = requant_exp(e[i], has_min);
  }
}

__device__ __forceinline__ int16_t tile_quantize_16lanes(double v, int* e_out) {
  const double vv[1] = {v};
  int16_t m[1];
  int e[1];
  tile_quantize_16lanes_n<1>(vv, m, e);
  *e_out = e[0];
  return m[0];
}

// ---------------------------------------------------------------------------
// numpy pairwise summation (numpy/_core/src/umath/loops_utils.h.src,
// pairwise_sum): blocks of <= 128 summed with 8 strided accumulators, larger
// ranges split at n/2 rounded down to a multiple of 8; the reduction adds the
// result to the identity +0.0.  Valid for n <= 8192 (one ufunc buffer).
// ---------------------------------------------------------------------------
__device__ __forceinline__ double np_pw_leaf(const double* a, int n) {
  if (n < 8) {
    double res = 0.0;
    for (int i = 0; i < n; ++i) res = __dadd_rn(res, a[i]);
    return res;
  }
  double r0 = a[0], r1 = a[1], r2 = a[2], r3 = a[3], r4 = a[4], r5 = a[5], r6 = a[6], r7 = a[7];
  int i = 8;
  int lim = n - (n % 8);
  for (; i < lim; i += 8) {
    r0 = __dadd_rn(r0, a[i + 0]); r1 = __dadd_rn(r1, a[i + 1]);
    r2 = __dadd_rn(r2, a[i + 2]); r3 = __dadd_rn(r3, a[i + 3]);
    r4 = __dadd_rn(r4, a[i + 4]); r5 = __dadd_rn(r5, a[i + 5]);
    r6 = __dadd_rn(r6, a[i + 6]); r7 = __dadd_rn(r7, a[i + 7]);
  }
  double res = __dadd_rn(__dadd_rn(__dadd_rn(r0, r1), __dadd_rn(r2, r3)),
                         __dadd_rn(__dadd_rn(r4, r5), __dadd_rn(r6, r7)));
  for (; i < n; ++i) res = __dadd_rn(res, a[i]);
  return res;
}

// np_pw_leaf by 8 cooperating lanes (lane & 7 = accumulator j, the group
// aligned to 8 lanes, all 32 lanes executing): each lane runs numpy's
// accumulator j sequentially, the groups combine
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) by xor shuffles (lower lane = left
// operand), and lane 0 of the group adds the tail.  Same operations in the
// same order as np_pw_leaf; the result is valid on lane 0 of each group.
__device__ __forceinline__ double np_pw_leaf_8lanes(const double* a, int n) {
  const int j = threadIdx.x & 7;
  double v = 0.0;
  if (n >= 8) {
    // the tree's leaves hold at most 128 elements: up to 16 per accumulator,
    // all loaded before the addition chain starts
    const int cnt = n >> 3;
    double x[16];
    #pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = i < cnt ? a[8 * i + j] : 0.0;
    v = x[0];
    #pragma unroll
    for (int i = 1; i < 16; ++i)
      if (i < cnt) v = __dadd_rn(v, x[i]);
    for (int i = 128 + j; i < 8 * cnt; i += 8) v = __dadd_rn(v, a[i]);   // longer runs (not a tree leaf)
  }
  double o = __shfl_xor_sync(0xffffffffu, v, 1);
  if ((j & 1) == 0) v = __dadd_rn(v, o);
  o = __shfl_xor_sync(0xffffffffu, v, 2);
  if ((j & 3) == 0) v = __dadd_rn(v, o);
  o = __shfl_xor_sync(0xffffffffu, v, 4);
  if (j == 0) {
    if (n < 8) {
      double res = 0.0;
      for (int i = 0; i < n; ++i) res = __dadd_rn(res, a[i]);
      v = res;
    } else {
      v = __dadd_rn(v, o);
      for (int i = n - (n % 8); i < n; ++i) v = __dadd_rn(v, a[i]);
    }
  }
  return v;
}

// Enumerates the leaves of the pairwise tree of size n in order, writing
// (start, len) pairs; returns the count.  Single thread.
__device__ __forceinline__ int np_pw_leaves(int n, int* lo_out, int* len_out, int max_leaves) {
  int st_lo[24], st_n[24];
  int sp = 0, nl = 0;
  st_lo[sp] = 0; st_n[sp] = n; ++sp;
  while (sp > 0) {
    --sp;
    int lo = st_lo[sp], len = st_n[sp];
    if (len <= 128) {
      if (nl < max_leaves) { lo_out[nl] = lo; len_out[nl] = len; }
      ++nl;
    } else {
      int n2 = len / 2;
      n2 -= n2 % 8;
      st_lo[sp] = lo + n2; st_n[sp] = len - n2; ++sp;   // right (visited second)
      st_lo[sp] = lo;      st_n[sp] = n2;       ++sp;   // left (visited first)
    }
  }
  return nl;
}

// Combines leaf values in the exact order of the recursive tree (post-order
// stack machine: a node's value is left + right once both children are done).
__device__ __forceinline__ double np_pw_combine(int n, const double* leafval) {
  int st_n[24], st_s[24];
  double vals[24];
  int sp = 0, vsp = 0, li = 0;
  st_n[0] = n; st_s[0] = 0; sp = 1;
  while (sp > 0) {
    const int top = sp - 1;
    const int len = st_n[top];
    if (len <= 128) {
      vals[vsp++] = leafval[li++];
      --sp;
      continue;
    }
    int n2 = len / 2;
    n2 -= n2 % 8;
    if (st_s[top] == 0) {
      st_s[top] = 1;
      st_n[sp] = n2; st_s[sp] = 0; ++sp;
    } else if (st_s[top] == 1) {
      st_s[top] = 2;
      st_n[sp] = len - n2; st_s[sp] = 0; ++sp;
    } else {
      const double r = vals[--vsp];
      const double l = vals[--vsp];
      vals[vsp++] = __dadd_rn(l, r);
      --sp;
    }
  }
  return vals[0];
}

// Single-thread numpy sum of a[0..n) (the full reduction: 0.0 + pairwise).
__device__ __forceinline__ double np_sum_serial(const double* a, int n) {
  if (n <= 128) return __dadd_rn(0.0, np_pw_leaf(a, n));
  int lo[64], len[64];
  double val[64];
  int nl = np_pw_leaves(n, lo, len, 64);
  for (int i = 0; i < nl; ++i) val[i] = np_pw_leaf(a + lo[i], len[i]);
  return __dadd_rn(0.0, np_pw_combine(n, val));
}

// numpy's pairwise tree is "perfect" for n when every split is an exact half
// that stays a multiple of 8 down to leaves of L <= 128 (L % 8 == 0, so no
// tail): e.g. n = 576 -> 8 leaves of 72.  Returns the number of halvings k
// (<= 3, i.e. <= 8 leaves) and the leaf size, or -1.
__host__ __device__ __forceinline__ int np_pw_perfect(int n, int* leaf) {
  int k = 0;
  while (n > 128) {
    const int n2 = n / 2;
    if ((n & 1) || (n2 % 8)) return -1;
    n = n2;
    if (++k > 3) return -1;
  }
  if (n < 8 || (n % 8)) return -1;
  *leaf = n;
  return k;
}

// Warp-parallel numpy sum for a perfect tree (k halvings, leaves of L): lane
// 4*l + q holds accumulators 2q, 2q+1 of leaf l; the accumulator pairs, the
// 8-accumulator combine ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) and the leaf
// tree are all evaluated by xor shuffles with the lower lane as the left
// operand, i.e. in exactly numpy's order.  Returns 0.0 + sum on every lane.
__device__ __forceinline__ double np_sum_warp_perfect(const double* a, int k, int L) {
  const int lane = threadIdx.x & 31;
  const int leaf = lane >> 2, q = lane & 3;
  double v = 0.0;
  if (leaf < (1 << k)) {
    const double* b = a + leaf * L + 2 * q;
    double r0 = b[0], r1 = b[1];
    for (int i = 8; i < L; i += 8) { r0 = __dadd_rn(r0, b[i]); r1 = __dadd_rn(r1, b[i + 1]); }
    v = __dadd_rn(r0, r1);
  }
  double o = __shfl_xor_sync(0xffffffffu, v, 1);
  if ((q & 1) == 0) v = __dadd_rn(v, o);
  o = __shfl_xor_sync(0xffffffffu, v, 2);
  if ((q & 2) == 0) v = __dadd_rn(v, o);
  for (int lev = 0; lev < k; ++lev) {
    const int m = 4 << lev;
    o = __shfl_xor_sync(0xffffffffu, v, m);
    if ((lane & m) == 0) v = __dadd_rn(v, o);
  }
  return __dadd_rn(0.0, __shfl_sync(0xffffffffu, v, 0));
}

// numpy sum driven by a precomputed plan of its pairwise tree (built on the
// host by build_pw_plan for every length): plan = [L, H, leaf starts (L),
// internal nodes per height (H), then (left, right) value slots of every
// internal node ordered by height].  Leaves are summed by separate lanes,
// then each height level is combined in parallel; value slots: leaves
// 0..L-1, internal node j -> L + j.  sval needs 2L - 1 doubles.
__device__ __forceinline__ double np_sum_warp_plan(const double* a, int n, const unsigned short* plan, double* sval) {
  const int lane = threadIdx.x & 31;
  const int L = plan[0], H = plan[1];
  const unsigned short* starts = plan + 2;
  const unsigned short* lvl = starts + L;
  const unsigned short* ops = lvl + H;
  for (int k0 = 0; k0 < L; k0 += 4) {                 // four leaves at a time, 8 lanes each
    const int k = k0 + (lane >> 3);
    const int s0 = k < L ? starts[k] : 0, e0 = k < L ? ((k + 1 < L) ? starts[k + 1] : n) : 0;
    const double v = np_pw_leaf_8lanes(a + s0, e0 - s0);
    if (k < L && (lane & 7) == 0) sval[k] = v;
  }
  __syncwarp();
  int base = 0;
  for (int h = 0; h < H; ++h) {
    const int cnt = lvl[h];
    for (int j = lane; j < cnt; j += 32) {
      const int o = base + j;
      sval[L + o] = __dadd_rn(sval[ops[2 * o]], sval[ops[2 * o + 1]]);
    }
    base += cnt;
    __syncwarp();
  }
  const double r = H ? sval[L + base - 1] : sval[0];
  return __dadd_rn(0.0, r);
}

// Warp-cooperative numpy sum of a shared-memory array (n <= 8192).  All 32
// lanes must call it; scratch needs 3*64 words of shared memory.  Returns the
// sum on every lane.
// The general tree (lengths without the power-of-two split) is kept out of
// line: it is large and rarely taken.
static __device__ __noinline__ double np_sum_warp_generic(const double* a, int n, int* s_lo, int* s_len, double* s_val) {
  const int lane = threadIdx.x & 31;
  if (n <= 128) {
    const double r = np_pw_leaf_8lanes(a, n);
    return __dadd_rn(0.0, __shfl_sync(0xffffffffu, r, 0));
  }
  int nl = 0;
  if (lane == 0) nl = np_pw_leaves(n, s_lo, s_len, 64);
  nl = __shfl_sync(0xffffffffu, nl, 0);
  __syncwarp();
  for (int i0 = 0; i0 < nl; i0 += 4) {               // four leaves at a time, 8 lanes each
    const int i = i0 + (lane >> 3);
    const double v = np_pw_leaf_8lanes(a + (i < nl ? s_lo[i] : 0), i < nl ? s_len[i] : 0);
    if (i < nl && (lane & 7) == 0) s_val[i] = v;
  }
  __syncwarp();
  double r = 0.0;
  if (lane == 0) r = __dadd_rn(0.0, np_pw_combine(n, s_val));
  return __shfl_sync(0xffffffffu, r, 0);
}

// np_sum_warp_perfect with the leaf length a compile-time constant: each
// lane's loads are issued together ahead of its addition chain.
template <int L>
__device__ __forceinline__ double np_sum_warp_perfect_t(const double* a, int k) {
  const int lane = threadIdx.x & 31;
  const int leaf = lane >> 2, q = lane & 3;
  double v = 0.0;
  if (leaf < (1 << k)) {
    const double* b = a + leaf * L + 2 * q;
    double x0[L / 8], x1[L / 8];
    #pragma unroll
    for (int i = 0; i < L / 8; ++i) { x0[i] = b[8 * i]; x1[i] = b[8 * i + 1]; }
    double r0 = x0[0], r1 = x1[0];
    #pragma unroll
    for (int i = 1; i < L / 8; ++i) { r0 = __dadd_rn(r0, x0[i]); r1 = __dadd_rn(r1, x1[i]); }
    v = __dadd_rn(r0, r1);
  }
  double o = __shfl_xor_sync(0xffffffffu, v, 1);
  if ((q & 1) == 0) v = __dadd_rn(v, o);
  o = __shfl_xor_sync(0xffffffffu, v, 2);
  if ((q & 2) == 0) v = __dadd_rn(v, o);
  for (int lev = 0; lev < k; ++lev) {
    const int m = 4 << lev;
    o = __shfl_xor_sync(0xffffffffu, v, m);
    if ((lane & m) == 0) v = __dadd_rn(v, o);
  }
  return __dadd_rn(0.0, __shfl_sync(0xffffffffu, v, 0));
}

__device__ __forceinline__ double np_sum_warp(const double* a, int n, int* s_lo, int* s_len,
                                              double* s_val) {
  int pl = 0;
  const int pk = np_pw_perfect(n, &pl);
  if (pk >= 0) {
    switch (pl) {                                  // leaf lengths of the usual model widths
      case 72: return np_sum_warp_perfect_t<72>(a, pk);     // 576, 1152
      case 96: return np_sum_warp_perfect_t<96>(a, pk);     // 192, 384, 768, 1536
      case 128: return np_sum_warp_perfect_t<128>(a, pk);   // 128, 256, 512, 1024
      default: return np_sum_warp_perfect(a, pk, pl);
    }
  }
  return np_sum_warp_generic(a, n, s_lo, s_len, s_val);
}

// d = c + a.h0*b.b0 + a.h1*b.b1 (lo) / a.h0*b.b2 + a.h1*b.b3 (hi); a: 2 x s16
__device__ __forceinline__ int dp2a_lo_ss(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int dp2a_hi_ss(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int dp2a_lo_su(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int dp2a_hi_su(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
// Exact sum_k x[k] y[k] over one 16-element tile of int16 values, x and y
// each as two uint4 of eight 16-bit values (elements 0..7, 8..15).  y is
// split into signed high bytes and unsigned low bytes (y = 256 hi + lo) and
// each half summed by dp2a in 32 bits (at most 16 products of 2^15 x 2^8).
__device__ __forceinline__ long long tile_sum16_dp2a(const uint4 x0, const uint4 x1, const uint4 y0, const uint4 y1) {
  const unsigned h0 = __byte_perm(y0.x, y0.y, 0x7531), h1 = __byte_perm(y0.z, y0.w, 0x7531);
  const unsigned h2 = __byte_perm(y1.x, y1.y, 0x7531), h3 = __byte_perm(y1.z, y1.w, 0x7531);
  const unsigned l0 = __byte_perm(y0.x, y0.y, 0x6420), l1 = __byte_perm(y0.z, y0.w, 0x6420);
  const unsigned l2 = __byte_perm(y1.x, y1.y, 0x6420), l3 = __byte_perm(y1.z, y1.w, 0x6420);
  int A = 0, B = 0;
  A = dp2a_lo_ss(x0.x, h0, A); A = dp2a_hi_ss(x0.y, h0, A);
  A = dp2a_lo_ss(x0.z, h1, A); A = dp2a_hi_ss(x0.w, h1, A);
  A = dp2a_lo_ss(x1.x, h2, A); A = dp2a_hi_ss(x1.y, h2, A);
  A = dp2a_lo_ss(x1.z, h3, A); A = dp2a_hi_ss(x1.w, h3, A);
  B = dp2a_lo_su(x0.x, l0, B); B = dp2a_hi_su(x0.y, l0, B);
  B = dp2a_lo_su(x0.z, l1, B); B = dp2a_hi_su(x0.w, l1, B);
  B = dp2a_lo_su(x1.x, l2, B); B = dp2a_hi_su(x1.y, l2, B);
  B = dp2a_lo_su(x1.z, l3, B); B = dp2a_hi_su(x1.w, l3, B);
  return ((long long)A << 8) + (long long)B;
}

// ---------------------------------------------------------------------------
// Correct rounding of (signed 128-bit integer) * 2^scale to double.
// ---------------------------------------------------------------------------
__device__ __forceinline__ double i128_to_double_scaled(__int128 x, int scale) {
  if (x == 0) return 0.0;
  bool neg = x < 0;
  unsigned __int128 u = neg ? (unsigned __int128)(-x) : (unsigned __int128)x;
  unsigned long long hi = (unsigned long long)(u >> 64), lo = (unsigned long long)u;
  int p = hi ? 127 - __clzll((long long)hi) : 63 - __clzll((long long)lo);  // top bit index
  double r;
  if (p < 53) {
    r = (double)lo;                                  // exact
    r = r * pow2(scale);
  } else {
    int sh = p - 52;
    unsigned __int128 mant = u >> sh;
    unsigned __int128 rem = u - (mant << sh);
    unsigned __int128 half = (unsigned __int128)1 << (sh - 1);
    unsigned long long m = (unsigned long long)mant;
    if (rem > half || (rem == half && (m & 1))) ++m;
    if (m >> 53) { m >>= 1; ++sh; }
    r = (double)m * pow2(sh + scale);                // exact: m < 2^53, power-of-two scale
  }
  return neg ? -r : r;
}

// Exact BFP dot of two 64-element head vectors given as 4 tiles each:
// sum_j S_j * 2^(E_j - 30) with S_j = sum_k qm*km (|S_j| <= 2^34) and
// E_j = qe_j + ke_j, rounded once to double.  This equals the reference's
// BLAS np.dot whenever the pair-exponent spread is <= 17 (then every partial
// sum is exact in double); wider spreads are rounded exactly here.
__device__ __forceinline__ double exact_tile_dot4(const long long S[4], const int E[4]) {
  int emax = -100000, emin = 100000;
  #pragma unroll
  for (int j = 0; j < 4; ++j)
    if (S[j] != 0) { emax = E[j] > emax ? E[j] : emax; emin = E[j] < emin ? E[j] : emin; }
  if (emax == -100000) return 0.0;
  if (emax - emin <= 17) {
    double s = 0.0;
    #pragma unroll
    for (int j = 0; j < 4; ++j) s = __dadd_rn(s, (double)S[j] * pow2(E[j] - 30));
    return s;
  }
  int base = emax - 90 > emin ? emax - 90 : emin;   // terms below 2^-90 of the top are dropped
  __int128 acc = 0;
  #pragma unroll
  for (int j = 0; j < 4; ++j)
    if (S[j] != 0 && E[j] >= base) acc += ((__int128)S[j]) << (E[j] - base);
  return i128_to_double_scaled(acc, base - 30);
}
#endif  // __CUDACC__

}  // namespace bfp
