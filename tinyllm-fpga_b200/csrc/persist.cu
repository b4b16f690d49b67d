// persist.cu -- persistent small-batch (1..4 sequences) decode kernel.
//
// One cooperative launch runs every decode step of a generate call.  Per step
// and layer the work is five phases (gen_smollm_blockfp_full.py:261-293):
//   P1  n1 = tile_quantize(rmsnorm_fp(h, g1)); q|k|v = matvec       one CTA per 16-row group
//   P2  rope_fp(q), rope_fp(k), KV write, attention, requant          one CTA per (column, q head)
//   P3  h1 = fpq(h + matvec(attn, Wo))                                one CTA per 16-row group
//   P4  mlp = tile_quantize(fpq(fpq(silu_fp(g)) * u)), g|u = matvec(tile_quantize(rmsnorm_fp(h1, g2)))
//                                                                     one CTA per gate/up group pair
//   P5  h = fpq(h1 + matvec(mlp, Wd))                                 one CTA per 16-row group
// followed by the head (:437-443): every CTA forms hn and scans a share of
// the vocabulary; every CTA then reduces the shares to the argmax and feeds
// it back as the next step's token.
//
// Phases are ordered by monotone per-phase completion counters instead of a
// grid-wide barrier: a producer CTA publishes (fence + atomic add) when its
// outputs are written, and a consumer waits (acquire load) only for the
// phase it reads.  CTAs without work in a phase skip it.  Every wait is
// bounded; a timeout sets the error flag and the kernel winds down.
//
// Each CTA streams the weight slice of its next matvec -- mantissa planes,
// tile exponents and, for the normalising phases, the gamma vector -- into
// one of two shared-memory buffers with a 1-D TMA bulk copy as soon as the
// buffer is free, so weight traffic overlaps the phases before it.  The
// attention CTAs (chosen among those idle in P1) stage the cached K/V rows
// of their head with cp.async before they wait for P1.
//
// Arithmetic is the one of the multi-kernel path (gemv.cu, attention_kernel,
// head kernels): the same device helpers in the same order, so the token
// streams are identical.  Data written inside the kernel is read with
// ld.global.cg (L2), never from a possibly stale L1 line.
#include "bfp_device.cuh"
#include "kernels.cuh"

namespace bfp {

namespace {

constexpr int PT = 256;                  // threads per CTA
constexpr int ATT_CH = 256;              // attention positions per shared-memory chunk
constexpr long long SPIN_LIMIT = 1LL << 22;

enum { C_P1 = 0, C_P2, C_P3, C_P4, C_P5, C_HEAD, C_COUNT };

// Per-CTA control block in static shared memory: column state, small
// scratch, and the views of the dynamic shared memory (so the out-of-line
// phase functions take one pointer).
struct Ctl {
  int tok[4], pos[4], slot[4];
  double red[16];
  double hnn[4];
  int lo[64], len[64];
  double val[160];
  int qk_m[128];
  int qk_e[8];
  double *xs, *sq, *sc, *hnT;
  int16_t* nm;
  int8_t* ne;
  int* ms;
  long long* acc;
  uint4 *attk, *attv;
  unsigned *attke, *attve;
  unsigned char* wbest;
};

// ---------------------------------------------------------------------------
// synchronisation primitives
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Publishes this CTA's completed global writes: counter += inc.
__device__ __forceinline__ void publish(unsigned* c, unsigned inc) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(c, inc);
  }
}

// Waits until counter >= target.  Returns false (on every thread) when the
// wait gave up or another CTA has already raised the error flag.
__device__ __forceinline__ bool wait_count(const unsigned* c, unsigned target, int* err) {
  int ok = 1;
  if (threadIdx.x == 0) {
    long long it = 0;
    while ((int)(ld_acquire_u32(c) - target) < 0) {
      if ((++it & 255) == 0) {
        if (ld_volatile_i32(err)) { ok = 0; break; }
        if (it > SPIN_LIMIT) { atomicExch(err, 2); ok = 0; break; }
      }
    }
    __threadfence();
  }
  return __syncthreads_and(ok) != 0;
}

__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

// the CTA's weight-slice buffer: TMA copies complete on one mbarrier
struct Bufs {
  unsigned char* p[2];
  unsigned long long* bar;
  unsigned par[2];
  bool pend[2];
};

__device__ __forceinline__ void buf_wait(Bufs& B, int b, int* err) {
  const unsigned bar = smem_u32(&B.bar[b]);
  long long it = 0;
  for (;;) {
    unsigned ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(bar), "r"(B.par[b]) : "memory");
    if (ok) break;
    if (++it > SPIN_LIMIT) {
      if (threadIdx.x == 0) atomicExch(err, 3);
      break;
    }
  }
  B.par[b] ^= 1u;
  B.pend[b] = false;
}

// ---------------------------------------------------------------------------
// exact 16-term tile sum (x int16, w as signed-high / unsigned-low byte planes)
// ---------------------------------------------------------------------------
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
__device__ __forceinline__ long long tile_sum(const uint4 x0, const uint4 x1, const uint4 wh, const uint4 wl) {
  int A = 0, B = 0;
  A = dp2a_lo_ss(x0.x, wh.x, A); A = dp2a_hi_ss(x0.y, wh.x, A);
  A = dp2a_lo_ss(x0.z, wh.y, A); A = dp2a_hi_ss(x0.w, wh.y, A);
  A = dp2a_lo_ss(x1.x, wh.z, A); A = dp2a_hi_ss(x1.y, wh.z, A);
  A = dp2a_lo_ss(x1.z, wh.w, A); A = dp2a_hi_ss(x1.w, wh.w, A);
  B = dp2a_lo_su(x0.x, wl.x, B); B = dp2a_hi_su(x0.y, wl.x, B);
  B = dp2a_lo_su(x0.z, wl.y, B); B = dp2a_hi_su(x0.w, wl.y, B);
  B = dp2a_lo_su(x1.x, wl.z, B); B = dp2a_hi_su(x1.y, wl.z, B);
  B = dp2a_lo_su(x1.z, wl.w, B); B = dp2a_hi_su(x1.w, wl.w, B);
  return ((long long)A << 8) + (long long)B;
}

// ---------------------------------------------------------------------------
// Roles.  Every CTA keeps one role for the whole launch, so each SM only
// ever executes one phase's code and its instruction caches stay warm:
//   role 0 (P1)  QKV matvec, gpc[0] row groups per CTA
//   role 1 (P3)  O matvec,   gpc[1] row groups
//   role 2 (P4)  gate/up,    gpc[2] g/u group pairs
//   role 3 (P5)  down,       gpc[3] row groups
//   role 4 (P2)  attention,  one (column, q head) per CTA
// Remaining CTAs only take part in the head.
// ---------------------------------------------------------------------------
constexpr int N_MV_ROLES = 4;

__host__ __device__ inline int role_units(const PersistArgs& a, int r) {   // row groups (role 2: pairs)
  return r == 0 ? (a.HQ + 2 * a.HKV) * 4 : r == 1 ? a.D / 16 : r == 2 ? a.FFN / 16 : a.D / 16;
}
__host__ __device__ inline int role_nt(const PersistArgs& a, int r) {      // K tiles of the role's matrix
  return r == 0 ? a.NTD : r == 1 ? a.HQ * 4 : r == 2 ? a.NTD : a.NTF;
}
__host__ __device__ inline int role_gpu(int r) { return r == 2 ? 2 : 1; } // weight groups per unit
__host__ __device__ inline bool role_gamma(int r) { return r == 0 || r == 2; }

struct Roles {
  int n[N_MV_ROLES];      // CTAs per matvec role
  int first[N_MV_ROLES + 2];   // first CTA of roles 0..3, attention, end of attention
  int items;
};

__host__ __device__ inline Roles roles_of(const PersistArgs& a) {
  Roles R;
  int c = 0;
  for (int r = 0; r < N_MV_ROLES; ++r) {
    R.n[r] = (role_units(a, r) + a.gpc[r] - 1) / a.gpc[r];
    R.first[r] = c;
    c += R.n[r];
  }
  R.items = a.ncols * a.HQ;
  R.first[N_MV_ROLES] = c;
  R.first[N_MV_ROLES + 1] = c + R.items;
  return R;
}

// one CTA's weight slice: mantissa planes [RG][NT][512], exponents
// [RG][NT][16], then (roles 0, 2) the layer's gamma
__host__ __device__ inline size_t slice_bytes(const PersistArgs& a, int r) {
  return (size_t)a.gpc[r] * role_gpu(r) * role_nt(a, r) * 528 + (role_gamma(r) ? (size_t)a.D * 8 : 0);
}

// ---------------------------------------------------------------------------
// shared memory: [mbarrier][weight slice][phase scratch U]
//   U: matvec scratch (xs, sq, nm, ne, ms, acc) | attention scratch |
//      head scratch (xs, sq, hnT, wbest)
// ---------------------------------------------------------------------------
struct PLayout {
  size_t bar, buf, xs, sq, nm, ne, ms, acc, sc, attk, attke, attv, attve, hnT, wbest, total;
};

__host__ __device__ inline size_t p_al(size_t x) { return (x + 127) & ~size_t(127); }
// doubles per column of the transposed hn: [ceil(D/256)][8][32]
__host__ __device__ inline int hnT_stride(int D) { return ((D / 8 + 31) / 32) * 256; }

__host__ __device__ inline PLayout p_layout(const PersistArgs& a, int NC) {
  PLayout L;
  const int NTmax = a.NTF > a.NTD ? a.NTF : a.NTD;
  const int Kmax = NTmax * 16;
  size_t sl = 0;
  for (int r = 0; r < N_MV_ROLES; ++r) sl = sl > slice_bytes(a, r) ? sl : slice_bytes(a, r);
  L.bar = 0;
  L.buf = 128;
  const size_t u0 = L.buf + p_al(sl);
  // matvec view
  L.xs = u0;
  L.sq = L.xs + p_al((size_t)NC * a.D * 8);
  L.nm = L.sq + p_al((size_t)NC * a.D * 8);
  L.ne = L.nm + p_al((size_t)NC * Kmax * 2);
  L.ms = L.ne + p_al((size_t)NC * NTmax);
  L.acc = L.ms + p_al((size_t)64 * NC * 4);
  const size_t mv_end = L.acc + p_al((size_t)PT * NC * 8);
  // head view: xs, sq, then the transposed hn and the per-warp bests
  L.hnT = L.nm;
  L.wbest = L.hnT + p_al((size_t)NC * hnT_stride(a.D) * 8);
  const size_t head_end = L.wbest + p_al((size_t)(PT / 32) * NC * 24);
  // attention view
  L.sc = u0;
  L.attk = L.sc + p_al((size_t)a.MAXC * 8);
  L.attke = L.attk + p_al((size_t)ATT_CH * 128);
  L.attv = L.attke + p_al((size_t)ATT_CH * 4);
  L.attve = L.attv + p_al((size_t)ATT_CH * 128);
  const size_t att_end = L.attve + p_al((size_t)ATT_CH * 4);
  size_t end = mv_end > head_end ? mv_end : head_end;
  end = end > att_end ? end : att_end;
  L.total = end;
  return L;
}

// ---------------------------------------------------------------------------
// out-of-line helpers: each exists once in the kernel, so the code of a
// phase stays small enough for the instruction caches
// ---------------------------------------------------------------------------
// tile_quantize of one 16-lane tile: (mantissa, exponent)
__device__ __noinline__ int2 q16(double v) {
  int e;
  const int16_t m = tile_quantize_16lanes(v, &e);
  return make_int2(m, e);
}

// tile_quantize(fpq(v)): the quantized tile, then the requant of a tile
// holding -32768 (valid = this lane's value takes part)
__device__ __noinline__ int2 q16_requant(double v, bool valid) {
  int e;
  int16_t m = tile_quantize_16lanes(v, &e);
  const unsigned bal = __ballot_sync(0xffffffffu, valid && m == (int16_t)-32768);
  const bool has_min = ((bal >> (threadIdx.x & 16)) & 0xFFFFu) != 0;
  m = requant_mant(m, has_min && e < 127);
  return make_int2(m, requant_exp(e, has_min));
}

// three independent tiles of tile_quantize(fpq(y)) per 16-lane group, their
// shuffle trees overlapped
struct Q3 { int2 q[3]; };
__device__ __noinline__ Q3 q16_requant3(double y0, double y1, double y2, bool v0, bool v1, bool v2) {
  const double y[3] = {y0, y1, y2};
  const bool v[3] = {v0, v1, v2};
  int16_t m[3];
  int e[3];
  tile_quantize_requant_16lanes_n<3>(y, v, m, e);
  Q3 r;
  #pragma unroll
  for (int i = 0; i < 3; ++i) r.q[i] = make_int2(m[i], e[i]);
  return r;
}

// silu_fp (:241-242): x / (1 + exp(-x))
__device__ __noinline__ double silu1(double x) { return __ddiv_rn(x, __dadd_rn(1.0, exp(-x))); }

// float(np.dot(q, k)) / math.sqrt(HD) from four exact tile sums
__device__ __noinline__ double score1(long long s0, long long s1, long long s2, long long s3, int e0, int e1, int e2,
                                      int e3, double sqrt_hd) {
  const long long S[4] = {s0, s1, s2, s3};
  const int E[4] = {e0, e1, e2, e3};
  return __ddiv_rn(exact_tile_dot4(S, E), sqrt_hd);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
}

// Stages NC columns of a BFP vector (K elements, column c at xm + c*K or, for
// the embedding, the row of ctl->tok[c]) into nm / ne; columns >= ncols are
// left unset.  One memory round trip: 16-byte cp.async for the mantissas,
// L2 loads for the exponents.
template <int NC>
__device__ __forceinline__ void stage_columns(const PersistArgs* a, Ctl* ctl, bool emb, const int16_t* xm,
                                              const int8_t* xe, int K) {
  const int NT = K / 16, NU = K / 8, tid = threadIdx.x;
  #pragma unroll 1
  for (int i = tid; i < NC * NU; i += PT) {
    const int c = i / NU, u = i - c * NU;
    if (c < a->ncols) {
      const int16_t* row = emb ? a->emb_m + (size_t)ctl->tok[c] * K : xm + (size_t)c * K;
      cp_async16(ctl->nm + (size_t)i * 8, row + (size_t)u * 8);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  #pragma unroll 1
  for (int i0 = tid; i0 < NC * NT; i0 += 2 * PT) {
    int8_t e[2];
    #pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = i0 + j * PT, c = i / NT, t = i - c * NT;
      e[j] = -127;
      if (i < NC * NT && c < a->ncols)
        e[j] = emb ? a->emb_e[(size_t)ctl->tok[c] * NT + t] : __ldcg(xe + (size_t)c * NT + t);
    }
    #pragma unroll
    for (int j = 0; j < 2; ++j)
      if (i0 + j * PT < NC * NT) ctl->ne[i0 + j * PT] = e[j];
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
}

// ---------------------------------------------------------------------------
// phase building blocks
// ---------------------------------------------------------------------------
// tile_quantize(rmsnorm_fp(x, gamma)) of NC columns -> nm / ne   (:236-238, :263-264, :286-287)
// x: the embedding rows of ctl->tok (emb) or xm / xe (column stride D)
template <int NC>
__device__ __noinline__ void norm_input(const PersistArgs* a, Ctl* ctl, bool emb, const int16_t* xm, const int8_t* xe,
                                        const double* gamma) {
  const int D = a->D, NT = D / 16, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  double* xs = ctl->xs;
  double* sq = ctl->sq;
  stage_columns<NC>(a, ctl, emb, xm, xe, D);
  #pragma unroll 1
  for (int i = tid; i < NC * D; i += PT) {
    const double x = (i / D < a->ncols) ? bfp_decode(ctl->nm[i], ctl->ne[i >> 4]) : 0.0;
    xs[i] = x;
    sq[i] = __dmul_rn(x, x);
  }
  __syncthreads();
  if (warp < NC) {
    const double sum = np_sum_warp(sq + (size_t)warp * D, D, ctl->lo, ctl->len, ctl->val);
    if (lane == 0) ctl->red[warp] = __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)D), a->eps));
  }
  __syncthreads();
  #pragma unroll 1
  for (int base = 0; base < NC * D; base += PT * 3) {
    double y[3];
    bool valid[3];
    #pragma unroll
    for (int q = 0; q < 3; ++q) {
      const int i = base + tid + q * PT;
      valid[q] = i < NC * D;
      const int c = valid[q] ? i / D : 0, k = valid[q] ? i - c * D : 0;
      y[q] = valid[q] ? __ddiv_rn(__dmul_rn(xs[i], gamma[k]), ctl->red[c]) : 0.0;
    }
    const Q3 r = q16_requant3(y[0], y[1], y[2], valid[0], valid[1], valid[2]);
    #pragma unroll
    for (int q = 0; q < 3; ++q) {
      const int i = base + tid + q * PT;
      if (valid[q]) {
        ctl->nm[i] = (int16_t)r.q[q].x;
        if ((i & 15) == 0) ctl->ne[i >> 4] = (int8_t)r.q[q].y;
      }
    }
  }
  __syncthreads();
  (void)NT;
}

// matvec input already in BFP form (column stride K)
template <int NC>
__device__ __noinline__ void load_input(const PersistArgs* a, Ctl* ctl, const int16_t* xm, const int8_t* xe, int K) {
  stage_columns<NC>(a, ctl, false, xm, xe, K);
}

// matvec_hw_golden (:217-233) of RG row groups x NC columns; weights and
// exponents in shared memory (buf: [RG][NT][512] mantissa planes, then
// [RG][NT][16] exponents).  Thread tid handles row tid % (16 RG) and every
// (16 RG)-th K tile; its partial int64 sums go to ctl->acc[tid][c] and the
// max exponents to ctl->ms.  Input columns >= ncols hold garbage; their sums
// are never read.
template <int NC, int RG>
__device__ __noinline__ void slice_matvec(Ctl* ctl, const unsigned char* buf, int NT) {
  constexpr int ROWS = 16 * RG, TPR = PT / ROWS;
  const int tid = threadIdx.x;
  const int row = tid % ROWS, tl = tid / ROWS, gi = row >> 4, ri = row & 15;
  const uint4* W = reinterpret_cast<const uint4*>(buf);
  const int8_t* WE = reinterpret_cast<const int8_t*>(buf + (size_t)RG * NT * 512);
  const int8_t* ne = ctl->ne;
  int* ms = ctl->ms;
  for (int i = tid; i < ROWS * NC; i += PT) ms[i] = -100000;
  __syncthreads();
  #pragma unroll
  for (int c = 0; c < NC; ++c) {
    int m = -100000;
    #pragma unroll 1
    for (int t = tl; t < NT; t += TPR) {
      const int e = (int)ne[c * NT + t] + (int)WE[(gi * NT + t) * 16 + ri];
      m = e > m ? e : m;
    }
    atomicMax(&ms[row * NC + c], m);
  }
  __syncthreads();
  long long acc[NC];
  int Mr[NC];
  #pragma unroll
  for (int c = 0; c < NC; ++c) { acc[c] = 0; Mr[c] = ms[row * NC + c]; }
  #pragma unroll 2
  for (int t = tl; t < NT; t += TPR) {
    const uint4 wh = W[(gi * NT + t) * 32 + ri], wl = W[(gi * NT + t) * 32 + 16 + ri];
    const int we = (int)WE[(gi * NT + t) * 16 + ri];
    #pragma unroll
    for (int c = 0; c < NC; ++c) {
      const uint4* xp = reinterpret_cast<const uint4*>(ctl->nm + (size_t)c * NT * 16 + t * 16);
      const long long Sm = tile_sum(xp[0], xp[1], wh, wl);
      const int sh = Mr[c] - (int)ne[c * NT + t] - we;
      acc[c] += (sh > ALIGN_MAX) ? 0LL : (Sm >> sh);
    }
  }
  #pragma unroll
  for (int c = 0; c < NC; ++c) ctl->acc[tid * NC + c] = acc[c];
  __syncthreads();
}

// clip and scale of slice row r (:229-232), exact
template <int NC, int RG>
__device__ __forceinline__ double slice_total(const Ctl* ctl, int r, int c) {
  constexpr int ROWS = 16 * RG, TPR = PT / ROWS;
  long long s = 0;
  #pragma unroll
  for (int k = 0; k < TPR; ++k) s += ctl->acc[(r + k * ROWS) * NC + c];
  s = s > SAT_HI ? SAT_HI : (s < SAT_LO ? SAT_LO : s);
  return (double)s * pow2(ctl->ms[r * NC + c] - 30);
}

// ---- epilogues: 16 lanes per (row group, column) pair; called by the first
// 32 * ceil(NPAIR / 2) threads (whole warps) --------------------------------
template <int NPAIR>
__device__ __forceinline__ bool epi_threads() { return threadIdx.x < 32 * ((NPAIR + 1) / 2); }

// q|k|v rows of groups g0 .. g0+ng-1: quant(matvec)  (:265-267)
template <int NC, int RG>
__device__ __noinline__ void epi_qkv(const PersistArgs* a, const Ctl* ctl, int g0, int ng, int R) {
  const int tid = threadIdx.x, p = tid >> 4, l16 = tid & 15, go = p / NC, c = p % NC;
  const bool valid = go < ng && c < a->ncols;
  const int2 q = q16(valid ? slice_total<NC, RG>(ctl, go * 16 + l16, c) : 0.0);
  if (valid) {
    a->qkv_m[(size_t)c * R + (g0 + go) * 16 + l16] = (int16_t)q.x;
    if (l16 == 0) a->qkv_e[(size_t)c * (R / 16) + g0 + go] = (int8_t)q.y;
  }
}

// out = fpq(res + quant(matvec)) for groups g0 .. g0+ng-1 (:285, :293); res
// is the embedding row of the fed token (emb) or rm / re
template <int NC, int RG>
__device__ __noinline__ void epi_residual(const PersistArgs* a, const Ctl* ctl, int g0, int ng, bool emb,
                                          const int16_t* rm, const int8_t* re, int16_t* om, int8_t* oe) {
  const int tid = threadIdx.x, p = tid >> 4, l16 = tid & 15, go = p / NC, c0 = p % NC;
  const bool valid = go < ng && c0 < a->ncols;
  const int c = valid ? c0 : 0, g = g0 + (valid ? go : 0);
  const int D = a->D, NTD = a->NTD;
  const size_t orow = (size_t)g * 16 + l16;
  double hv = 0.0;
  if (valid) {
    if (emb) {
      const size_t t = (size_t)ctl->tok[c];
      hv = bfp_decode(a->emb_m[t * D + orow], a->emb_e[t * NTD + g]);
    } else {
      hv = bfp_decode(__ldcg(rm + (size_t)c * D + orow), __ldcg(re + (size_t)c * NTD + g));
    }
  }
  const int2 q = q16(valid ? slice_total<NC, RG>(ctl, go * 16 + l16, c0) : 0.0);
  const int2 r = q16(__dadd_rn(hv, bfp_decode(q.x, q.y)));
  if (valid) {
    om[(size_t)c * D + orow] = (int16_t)r.x;
    if (l16 == 0) oe[(size_t)c * NTD + g] = (int8_t)r.y;
  }
}

// mlp groups u0 .. u0+nu-1 = tile_quantize(fpq(fpq(silu_fp(g)) * u))  (:288-291);
// slice rows: pair j = gate rows 32j..32j+15, up rows 32j+16..32j+31
template <int NC, int RG>
__device__ __noinline__ void epi_swiglu(const PersistArgs* a, const Ctl* ctl, int u0, int nu) {
  const int tid = threadIdx.x, p = tid >> 4, l16 = tid & 15, j = p / NC, c0 = p % NC;
  const bool valid = j < nu && c0 < a->ncols;
  const int c = valid ? c0 : 0, u = u0 + (valid ? j : 0);
  const int2 gq = q16(valid ? slice_total<NC, RG>(ctl, j * 32 + l16, c0) : 0.0);
  const int2 uq = q16(valid ? slice_total<NC, RG>(ctl, j * 32 + 16 + l16, c0) : 0.0);
  const int2 s = q16(silu1(bfp_decode(gq.x, gq.y)));
  const int2 r = q16_requant(__dmul_rn(bfp_decode(s.x, s.y), bfp_decode(uq.x, uq.y)), valid);
  if (valid) {
    a->mlp_m[(size_t)c * a->FFN + (size_t)u * 16 + l16] = (int16_t)r.x;
    if (l16 == 0) a->mlp_e[(size_t)c * a->NTF + u] = (int8_t)r.y;
  }
}

// ---------------------------------------------------------------------------
// attention of (column c, q head) at position pos (:268-283).  K and V are
// processed in chunks of ATT_CH positions staged in shared memory; the
// current position's rotated k and raw v are inserted into their chunk.
// ---------------------------------------------------------------------------
struct AttItem {
  int c, head, kvh, pos, T, kpre;
  size_t kbase;
};

__device__ __forceinline__ AttItem att_item(const PersistArgs* a, const Ctl* ctl, int layer, int item) {
  AttItem it;
  it.c = item / a->HQ;
  it.head = item - it.c * a->HQ;
  it.kvh = it.head / (a->HQ / a->HKV);
  it.pos = ctl->pos[it.c];
  it.T = it.pos + 1;
  it.kpre = it.pos < ATT_CH ? it.pos : ATT_CH;
  it.kbase = (((size_t)ctl->slot[it.c] * a->kv.NL + layer) * a->HKV + it.kvh) * a->kv.MAX_CTX;
  return it;
}

// issues the copies of cached rows [r0, r0 + n) of K (and V) into shared
// memory; the exponent words are loaded by the caller's threads directly
__device__ __noinline__ void att_stage(const PersistArgs* a, Ctl* ctl, size_t kbase, int r0, int n, bool k, bool v) {
  const int tid = threadIdx.x;
  const uint4* ksrc = reinterpret_cast<const uint4*>(a->kv.km + (kbase + r0) * 64);
  const uint4* vsrc = reinterpret_cast<const uint4*>(a->kv.vm + (kbase + r0) * 64);
  #pragma unroll 1
  for (int i = tid; i < n * 8; i += PT) {
    if (k) cp_async16(ctl->attk + i, ksrc + i);
    if (v) cp_async16(ctl->attv + i, vsrc + i);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const unsigned* kesrc = reinterpret_cast<const unsigned*>(a->kv.ke + (kbase + r0) * 4);
  const unsigned* vesrc = reinterpret_cast<const unsigned*>(a->kv.ve + (kbase + r0) * 4);
  #pragma unroll 1
  for (int i = tid; i < n; i += PT) {
    if (k) ctl->attke[i] = __ldcg(kesrc + i);
    if (v) ctl->attve[i] = __ldcg(vesrc + i);
  }
}

__device__ __noinline__ void att_compute(const PersistArgs* a, Ctl* ctl, int layer, int item, bool prefetched) {
  const AttItem it = att_item(a, ctl, layer, item);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int HQ = a->HQ, HKV = a->HKV;
  const int R = (HQ + 2 * HKV) * 64;
  const int16_t* qm = a->qkv_m + (size_t)it.c * R;
  const int8_t* qe = a->qkv_e + (size_t)it.c * (R / 16);
  const int pos = it.pos, T = it.T;
  const int vrow0 = (HQ + HKV + it.kvh) * 64;
  if (!prefetched) att_stage(a, ctl, it.kbase, 0, it.kpre, true, true);
  // rope_fp of q (this head) and k (its kv head) at `pos` (:250-258, :268-269), then fpq
  if (tid < 128) {
    const int which = tid >> 6, d = tid & 63;
    const int row0 = which == 0 ? it.head * 64 : (HQ + it.kvh) * 64;
    const int jj = d < 32 ? d : d - 32, pd = d < 32 ? d + 32 : d - 32;
    const double own = bfp_decode(__ldcg(qm + row0 + d), __ldcg(qe + (row0 + d) / 16));
    const double partner = bfp_decode(__ldcg(qm + row0 + pd), __ldcg(qe + (row0 + pd) / 16));
    const double cs = a->rope_cs[((size_t)pos * 32 + jj) * 2], sn = a->rope_cs[((size_t)pos * 32 + jj) * 2 + 1];
    const double av = d < 32 ? own : partner, bv = d < 32 ? partner : own;
    const double y = d < 32 ? __dsub_rn(__dmul_rn(av, cs), __dmul_rn(bv, sn))
                            : __dadd_rn(__dmul_rn(bv, cs), __dmul_rn(av, sn));
    const int2 q = q16(y);
    ctl->qk_m[tid] = q.x;
    if ((d & 15) == 0) ctl->qk_e[which * 4 + d / 16] = q.y;
    if (which == 1 && it.head % (HQ / HKV) == 0) {     // KV write (:270-272), once per kv head
      const size_t kvrow = it.kbase + pos;
      a->kv.km[kvrow * 64 + d] = (int16_t)q.x;
      if ((d & 15) == 0) a->kv.ke[kvrow * 4 + d / 16] = (int8_t)q.y;
      a->kv.vm[kvrow * 64 + d] = __ldcg(qm + vrow0 + d);
      if ((d & 15) == 0) a->kv.ve[kvrow * 4 + d / 16] = __ldcg(qe + vrow0 / 16 + d / 16);
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  // scores[t] = float(np.dot(q, k_t)) / math.sqrt(HD)   (:278), exact
  double* sc = ctl->sc;
  const int* qk_m = ctl->qk_m;
  const int* qk_e = ctl->qk_e;
  double lmax = -INFINITY;
  #pragma unroll 1
  for (int c0 = 0; c0 < T; c0 += ATT_CH) {
    const int n = min(ATT_CH, T - c0);
    if (c0 > 0) {
      __syncthreads();
      att_stage(a, ctl, it.kbase, c0, min(n, pos - c0), true, false);
      asm volatile("cp.async.wait_all;" ::: "memory");
    }
    if (pos - c0 < n && tid < 32) {                    // the current position's rotated k
      int16_t* kr = reinterpret_cast<int16_t*>(ctl->attk + (size_t)(pos - c0) * 8);
      kr[2 * tid] = (int16_t)qk_m[64 + 2 * tid];
      kr[2 * tid + 1] = (int16_t)qk_m[64 + 2 * tid + 1];
      if (tid == 0)
        ctl->attke[pos - c0] = (unsigned)(qk_e[4] & 0xFF) | ((unsigned)(qk_e[5] & 0xFF) << 8) |
                               ((unsigned)(qk_e[6] & 0xFF) << 16) | ((unsigned)(qk_e[7] & 0xFF) << 24);
    }
    __syncthreads();
    #pragma unroll 1
    for (int t = tid; t < n; t += PT) {
      const uint4* kr = ctl->attk + t * 8;
      const unsigned ke4 = ctl->attke[t];
      long long Sx[4];
      #pragma unroll
      for (int jt = 0; jt < 4; ++jt) {
        const uint4 k0 = kr[2 * jt], k1 = kr[2 * jt + 1];
        const unsigned w[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
        long long s = 0;
        #pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int lo = (int)(int16_t)(w[u] & 0xFFFF), hi = (int)(int16_t)(w[u] >> 16);
          s += (long long)(qk_m[jt * 16 + 2 * u] * lo) + (long long)(qk_m[jt * 16 + 2 * u + 1] * hi);
        }
        Sx[jt] = s;
      }
      const double v = score1(Sx[0], Sx[1], Sx[2], Sx[3], qk_e[0] + (int)(int8_t)(ke4), qk_e[1] + (int)(int8_t)(ke4 >> 8),
                              qk_e[2] + (int)(int8_t)(ke4 >> 16), qk_e[3] + (int)(int8_t)(ke4 >> 24), a->sqrt_hd);
      sc[c0 + t] = v;
      lmax = v > lmax ? v : lmax;
    }
  }
  // softmax_fp (:245-247): e = exp(x - max); e / e.sum()
  for (int off = 16; off; off >>= 1) {
    const double o = __shfl_xor_sync(0xffffffffu, lmax, off);
    lmax = o > lmax ? o : lmax;
  }
  if (lane == 0) ctl->red[warp] = lmax;
  __syncthreads();
  double mx = ctl->red[0];
  #pragma unroll 1
  for (int w = 1; w < PT / 32; ++w) mx = ctl->red[w] > mx ? ctl->red[w] : mx;
  #pragma unroll 1
  for (int t = tid; t < T; t += PT) sc[t] = exp(__dsub_rn(sc[t], mx));
  __syncthreads();
  if (warp == 0) {
    const double Ssum = np_sum_warp_plan(sc, T, a->pw_data + a->pw_off[T], ctl->val);
    if (lane == 0) ctl->red[8] = Ssum;
  }
  __syncthreads();
  const double Ssum = ctl->red[8];
  #pragma unroll 1
  for (int t = tid; t < T; t += PT) sc[t] = __ddiv_rn(sc[t], Ssum);
  // attn += sm[t] * v[t], sequential in t (:280-281)
  double acc = 0.0;
  #pragma unroll 1
  for (int c0 = 0; c0 < T; c0 += ATT_CH) {
    const int n = min(ATT_CH, T - c0);
    __syncthreads();
    if (c0 > 0) {
      att_stage(a, ctl, it.kbase, c0, min(n, pos - c0), false, true);
      asm volatile("cp.async.wait_all;" ::: "memory");
    }
    if (pos - c0 < n) {                                // the current position's v (:272)
      if (tid < 32)
        reinterpret_cast<unsigned*>(ctl->attv + (size_t)(pos - c0) * 8)[tid] =
            __ldcg(reinterpret_cast<const unsigned*>(qm + vrow0) + tid);
      if (tid == 0) {
        unsigned e4 = 0;
        #pragma unroll
        for (int j = 0; j < 4; ++j) e4 |= (unsigned)(uint8_t)__ldcg(qe + vrow0 / 16 + j) << (8 * j);
        ctl->attve[pos - c0] = e4;
      }
    }
    __syncthreads();
    if (tid < 64) {
      const int16_t* vr = reinterpret_cast<const int16_t*>(ctl->attv) + tid;
      const unsigned* ve = ctl->attve;
      const int sh = 8 * (tid >> 4);
      #pragma unroll 8
      for (int t = 0; t < n; ++t) {
        const int e = (int)(int8_t)(ve[t] >> sh);
        acc = __dadd_rn(acc, __dmul_rn(sc[c0 + t], bfp_decode(vr[(size_t)t * 64], e)));
      }
    }
  }
  if (tid < 64) {
    const int2 q = q16_requant(acc, true);           // tile_quantize(fpq(attn)) (:282-283)
    a->a_m[(size_t)it.c * HQ * 64 + it.head * 64 + tid] = (int16_t)q.x;
    if ((tid & 15) == 0) a->a_e[(size_t)it.c * HQ * 4 + it.head * 4 + tid / 16] = (int8_t)q.y;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// head (:437-440): hn = (h / sqrt(mean(h*h) + eps)) * norm_w_q in every CTA;
// fp64 logits of this CTA's share of the vocabulary -> (best, index, runner-up).
// hn is held transposed (hnT[c][k/256][k%8][(k/8)%32]) so the lanes of a
// warp, which handle consecutive 8-element chunks of an embedding row, read
// consecutive doubles.
// ---------------------------------------------------------------------------
template <int NC>
__device__ __noinline__ void head_scan(const PersistArgs* a, Ctl* ctl, int par) {
  const int D = a->D, NT = D / 16, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int HS = hnT_stride(D);
  double* xs = ctl->xs;
  double* sq = ctl->sq;
  double* hnT = ctl->hnT;
  stage_columns<NC>(a, ctl, false, a->h_m, a->h_e, D);
  #pragma unroll 1
  for (int i = tid; i < NC * D; i += PT) {
    const double x = (i / D < a->ncols) ? bfp_decode(ctl->nm[i], ctl->ne[i >> 4]) : 0.0;
    xs[i] = x;
    sq[i] = __dmul_rn(x, x);
  }
  __syncthreads();                                   // hnT overlays the staged input
  #pragma unroll 1
  for (int i = tid; i < NC * HS; i += PT) hnT[i] = 0.0;
  if (warp < NC) {
    const double sum = np_sum_warp(sq + (size_t)warp * D, D, ctl->lo, ctl->len, ctl->val);
    if (lane == 0) ctl->red[warp] = __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)D), a->eps));
  }
  __syncthreads();
  #pragma unroll 1
  for (int i = tid; i < NC * D; i += PT) {
    const int c = i / D, k = i - c * D, u = k >> 3;
    hnT[c * HS + ((u >> 5) * 8 + (k & 7)) * 32 + (u & 31)] = __dmul_rn(__ddiv_rn(xs[i], ctl->red[c]), a->nw[k]);
  }
  __syncthreads();
  // ||hn|| for the certificate (any summation order; rounding covered by the 1e-12 factor)
  if (blockIdx.x == 0) {
    #pragma unroll 1
    for (int c = 0; c < NC; ++c) {
      double ss = 0.0;
      #pragma unroll 1
      for (int k = tid; k < HS; k += PT) ss = fma(hnT[c * HS + k], hnT[c * HS + k], ss);
      for (int off = 16; off; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      if (lane == 0) ctl->red[8 + warp] = ss;
      __syncthreads();
      if (tid == 0) {
        double t = 0.0;
        for (int w = 0; w < PT / 32; ++w) t += ctl->red[8 + w];
        ctl->hnn[c] = sqrt(t) * (1.0 + 1e-12);
      }
      __syncthreads();
    }
  }
  double best[NC], sec[NC];
  int bidx[NC];
  #pragma unroll
  for (int c = 0; c < NC; ++c) { best[c] = -INFINITY; sec[c] = -INFINITY; bidx[c] = 0x7fffffff; }
  const int NU = D / 8;
  const int gw = blockIdx.x * (PT / 32) + warp, nw = gridDim.x * (PT / 32);
  constexpr int RF = 4;                                  // rows in flight per warp
  #pragma unroll 1
  for (int v0 = gw; v0 < a->V; v0 += RF * nw) {
    double acc[RF][NC];
    #pragma unroll
    for (int q = 0; q < RF; ++q)
      #pragma unroll
      for (int c = 0; c < NC; ++c) acc[q][c] = 0.0;
    #pragma unroll 1
    for (int ub = 0; ub < NU; ub += 96) {
      uint4 w[RF][3];
      int ex[RF][3];
      #pragma unroll
      for (int q = 0; q < RF; ++q)
        #pragma unroll
        for (int j = 0; j < 3; ++j) {
          const int v = v0 + q * nw, u = ub + lane + 32 * j;
          if (v < a->V && u < NU) {
            w[q][j] = reinterpret_cast<const uint4*>(a->emb_m + (size_t)v * D)[u];
            ex[q][j] = a->emb_e[(size_t)v * NT + u / 2];
          } else {                                     // zero mantissas: contribute nothing
            w[q][j] = make_uint4(0, 0, 0, 0);
            ex[q][j] = 0;
          }
        }
      #pragma unroll
      for (int j = 0; j < 3; ++j) {
        if (ub + 32 * j >= NU) break;                  // chunks beyond the row (warp-uniform)
        const double* hp = hnT + ((ub >> 5) + j) * 256 + lane;   // zero-filled beyond D
        #pragma unroll
        for (int q = 0; q < RF; ++q) {
          const double scl = pow2(ex[q][j] - 15);
          const unsigned ww[4] = {w[q][j].x, w[q][j].y, w[q][j].z, w[q][j].w};
          #pragma unroll
          for (int t = 0; t < 8; ++t) {
            const double ev = (double)(int)(int16_t)((ww[t >> 1] >> (16 * (t & 1))) & 0xFFFF) * scl;
            #pragma unroll
            for (int c = 0; c < NC; ++c) acc[q][c] = fma(ev, hp[c * HS + t * 32], acc[q][c]);
          }
        }
      }
    }
    #pragma unroll
    for (int q = 0; q < RF; ++q) {
      const int v = v0 + q * nw;
      #pragma unroll
      for (int c = 0; c < NC; ++c) {
        double x = acc[q][c];
        #pragma unroll
        for (int off = 16; off; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
        if (v < a->V) {
          if (x > best[c]) { sec[c] = best[c]; best[c] = x; bidx[c] = v; }
          else if (x > sec[c]) sec[c] = x;
        }
      }
    }
  }
  double* wb = reinterpret_cast<double*>(ctl->wbest);
  if (lane == 0)
    #pragma unroll
    for (int c = 0; c < NC; ++c) {
      wb[(warp * NC + c) * 3 + 0] = best[c];
      wb[(warp * NC + c) * 3 + 1] = sec[c];
      wb[(warp * NC + c) * 3 + 2] = (double)bidx[c];
    }
  __syncthreads();
  if (tid < NC && tid < a->ncols) {
    double b = -INFINITY, s2 = -INFINITY;
    int bi = 0x7fffffff;
    #pragma unroll 1
    for (int w = 0; w < PT / 32; ++w) {
      const double x = wb[(w * NC + tid) * 3], xs2 = wb[(w * NC + tid) * 3 + 1];
      const int xi = (int)wb[(w * NC + tid) * 3 + 2];
      if (x > b || (x == b && xi < bi)) { s2 = fmax(s2, b); b = x; bi = xi; }
      else s2 = fmax(s2, x);
      s2 = fmax(s2, xs2);
    }
    const size_t o = ((size_t)par * 4 + tid) * gridDim.x + blockIdx.x;
    a->part_val[o] = b;
    a->part_idx[o] = bi;
    a->part_sec[o] = s2;
  }
}

// every CTA: argmax over all shares (lowest index on ties), token feedback;
// CTA 0 also records the token and the certificate (:439-443).  The grid has
// at most 32 * HR_MAX CTAs.
constexpr int HR_MAX = 8;
__device__ __noinline__ void head_reduce(const PersistArgs* a, Ctl* ctl, int par, int step) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (warp < 4 && warp < a->ncols) {
    const int c = warp, nrb = gridDim.x;
    double xv[HR_MAX], xsv[HR_MAX];
    int xiv[HR_MAX];
    #pragma unroll
    for (int j = 0; j < HR_MAX; ++j) {
      const int r = lane + 32 * j;
      const size_t o = ((size_t)par * 4 + c) * nrb + r;
      xv[j] = -INFINITY; xsv[j] = -INFINITY; xiv[j] = 0x7fffffff;
      if (r < nrb) { xv[j] = __ldcg(a->part_val + o); xiv[j] = __ldcg(a->part_idx + o); xsv[j] = __ldcg(a->part_sec + o); }
    }
    double best = -INFINITY, sec = -INFINITY;
    int bi = 0x7fffffff;
    #pragma unroll
    for (int j = 0; j < HR_MAX; ++j) {
      if (xv[j] > best || (xv[j] == best && xiv[j] < bi)) { sec = fmax(sec, best); best = xv[j]; bi = xiv[j]; }
      else sec = fmax(sec, xv[j]);
      sec = fmax(sec, xsv[j]);
    }
    #pragma unroll 1
    for (int off = 16; off; off >>= 1) {
      const double ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      const double os = __shfl_xor_sync(0xffffffffu, sec, off);
      if (ob > best || (ob == best && oi < bi)) { sec = fmax(sec, best); best = ob; bi = oi; }
      else sec = fmax(sec, ob);
      sec = fmax(sec, os);
    }
    if (lane == 0) {
      const bool ok = bi >= 0 && bi < a->V;          // no index: every logit was NaN
      if (!ok) bi = 0;
      if (blockIdx.x == 0) {
        // |fl(dot) - dot| <= gamma_D ||hn|| ||e_v|| for every summation order
        const double u = 1.1102230246251565e-16;
        const double gam = (a->D + 2) * u / (1.0 - (a->D + 2) * u);
        const double margin = 4.0 * gam * ctl->hnn[c] * a->emb_norm_max * (1.0 + 1e-6);
        if (!ok || !((best - sec) > margin)) atomicAdd(reinterpret_cast<unsigned long long*>(a->uncert), 1ULL);
        a->gen_out[(size_t)c * a->n_gen + step] = bi;
      }
      ctl->tok[c] = bi;
      ctl->pos[c] += 1;
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// One TMA transaction for the whole slice: mantissas and exponents of the nu
// units (exponents placed after a full gpc-unit mantissa block) and gamma.
__device__ __forceinline__ void fetch_slice(const PersistArgs* a, Bufs& B, int r, int l, int u0, int nu) {
  const int NT = role_nt(*a, r), gpu = role_gpu(r), G = role_units(*a, r) * gpu;
  const uint8_t* wm = r == 0 ? a->wm_qkv : r == 1 ? a->wm_o : r == 2 ? a->wm_gu : a->wm_d;
  const int8_t* we = r == 0 ? a->we_qkv : r == 1 ? a->we_o : r == 2 ? a->we_gu : a->we_d;
  const size_t gi = ((size_t)l * G + (size_t)u0 * gpu) * NT;
  const unsigned nt = (unsigned)(nu * gpu * NT), full = (unsigned)(a->gpc[r] * gpu * NT);
  if (threadIdx.x == 0) {
    const unsigned bar = smem_u32(&B.bar[0]);
    const unsigned ng = role_gamma(r) ? (unsigned)a->D * 8 : 0u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(nt * 528 + ng) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(B.p[0])), "l"(wm + gi * 512), "r"(nt * 512), "r"(bar) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(B.p[0] + (size_t)full * 512)), "l"(we + gi * 16), "r"(nt * 16), "r"(bar) : "memory");
    if (ng)
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   :: "r"(smem_u32(B.p[0] + (size_t)full * 528)), "l"((r == 0 ? a->g1 : a->g2) + (size_t)l * a->D),
                      "r"(ng), "r"(bar) : "memory");
  }
  B.pend[0] = true;
}

// matvec of this CTA's slice with the RG-group instantiation that covers it
template <int NC>
__device__ __forceinline__ void run_matvec(Ctl* ctl, const unsigned char* buf, int rg, int NT) {
  if (rg == 1) slice_matvec<NC, 1>(ctl, buf, NT);
  else if (rg == 2) slice_matvec<NC, 2>(ctl, buf, NT);
  else slice_matvec<NC, 4>(ctl, buf, NT);
}

template <int NC>
__device__ __forceinline__ void run_epilogue(const PersistArgs* a, Ctl* ctl, int r, int rg, int u0, int nu, bool emb) {
  const int D = a->D;
  (void)D;
  #define PERSIST_EPI(RGV)                                                                          \
    if (rg == RGV) {                                                                                \
      if (r == 0) { if (epi_threads<RGV * NC>()) epi_qkv<NC, RGV>(a, ctl, u0, nu, role_units(*a, 0) * 16); } \
      else if (r == 1) { if (epi_threads<RGV * NC>()) epi_residual<NC, RGV>(a, ctl, u0, nu, emb, a->h_m, a->h_e, a->h1_m, a->h1_e); } \
      else if (r == 2) { if (epi_threads<(RGV >= 2 ? RGV / 2 : 1) * NC>()) epi_swiglu<NC, RGV>(a, ctl, u0, nu); } \
      else { if (epi_threads<RGV * NC>()) epi_residual<NC, RGV>(a, ctl, u0, nu, false, a->h1_m, a->h1_e, a->h_m, a->h_e); } \
    }
  PERSIST_EPI(1) else PERSIST_EPI(2) else PERSIST_EPI(4)
  #undef PERSIST_EPI
}

template <int NC>
__global__ void __launch_bounds__(PT, 1) persistent_decode_kernel(const __grid_constant__ PersistArgs args) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ Ctl ctl_s;
  const PersistArgs* a = &args;
  Ctl* ctl = &ctl_s;
  const int tid = threadIdx.x, cta = blockIdx.x, ncta = gridDim.x;
  const PLayout L = p_layout(args, NC);
  if (tid == 0) {
    ctl->xs = reinterpret_cast<double*>(smem + L.xs);
    ctl->sq = reinterpret_cast<double*>(smem + L.sq);
    ctl->nm = reinterpret_cast<int16_t*>(smem + L.nm);
    ctl->ne = reinterpret_cast<int8_t*>(smem + L.ne);
    ctl->ms = reinterpret_cast<int*>(smem + L.ms);
    ctl->acc = reinterpret_cast<long long*>(smem + L.acc);
    ctl->sc = reinterpret_cast<double*>(smem + L.sc);
    ctl->attk = reinterpret_cast<uint4*>(smem + L.attk);
    ctl->attke = reinterpret_cast<unsigned*>(smem + L.attke);
    ctl->attv = reinterpret_cast<uint4*>(smem + L.attv);
    ctl->attve = reinterpret_cast<unsigned*>(smem + L.attve);
    ctl->hnT = reinterpret_cast<double*>(smem + L.hnT);
    ctl->wbest = smem + L.wbest;
  }
  Bufs B;
  B.p[0] = B.p[1] = smem + L.buf;
  B.bar = reinterpret_cast<unsigned long long*>(smem + L.bar);
  B.par[0] = B.par[1] = 0;
  B.pend[0] = B.pend[1] = false;
  const Roles R = roles_of(args);
  // this CTA's role
  int role = -1, u0 = 0, nu = 0, item = -1;
  for (int r = 0; r < N_MV_ROLES; ++r)
    if (cta >= R.first[r] && cta < R.first[r] + R.n[r]) {
      role = r;
      u0 = (cta - R.first[r]) * a->gpc[r];
      nu = min(a->gpc[r], role_units(args, r) - u0);
    }
  if (cta >= R.first[N_MV_ROLES] && cta < R.first[N_MV_ROLES + 1]) { role = N_MV_ROLES; item = cta - R.first[N_MV_ROLES]; }
  const int rg = role >= 0 && role < N_MV_ROLES ? a->gpc[role] * role_gpu(role) : 0;
  const int NT = role >= 0 && role < N_MV_ROLES ? role_nt(args, role) : 0;
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_u32(&B.bar[0])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid < 4) {
    const bool v = tid < a->ncols;
    ctl->tok[tid] = v ? a->col_tok[tid] : 0;
    ctl->pos[tid] = v ? a->col_pos[tid] : 0;
    ctl->slot[tid] = v ? a->col_slot[tid] : 0;
  }
  __syncthreads();
  if (rg > 0 && a->n_gen > 0) fetch_slice(a, B, role, 0, u0, nu);
  unsigned* cnt = a->sync;
  // counter of each phase and the units it counts per layer instance
  const int in_ctr[5] = {C_P5, C_P2, C_P3, C_P4, C_P1};      // what role r waits for
  const unsigned in_per[5] = {(unsigned)R.n[3], (unsigned)R.items, (unsigned)R.n[1], (unsigned)R.n[2],
                              (unsigned)R.n[0]};
  const int out_ctr[5] = {C_P1, C_P3, C_P4, C_P5, C_P2};
  bool ok = true;
  bool att_staged = false;
  for (int step = 0; step < a->n_gen && ok; ++step) {
    for (int l = 0; l < a->NL && ok; ++l) {
      const unsigned inst = (unsigned)(step * a->NL + l);
      const bool emb = l == 0;
      if (role >= 0 && role < N_MV_ROLES) {
        buf_wait(B, 0, a->err);
        // role 0 reads h of the previous layer (layer 0: the embedding, known locally)
        const unsigned target = role == 0 ? inst * in_per[0] : (inst + 1) * in_per[role];
        if (!(role == 0 && emb) && !wait_count(cnt + in_ctr[role] * 32, target, a->err)) { ok = false; break; }
        const unsigned char* buf = B.p[0];
        const double* gamma = reinterpret_cast<const double*>(buf + (size_t)a->gpc[role] * role_gpu(role) * NT * 528);
        if (role == 0) norm_input<NC>(a, ctl, emb, a->h_m, a->h_e, gamma);
        else if (role == 1) load_input<NC>(a, ctl, a->a_m, a->a_e, a->HQ * 64);
        else if (role == 2) norm_input<NC>(a, ctl, false, a->h1_m, a->h1_e, gamma);
        else load_input<NC>(a, ctl, a->mlp_m, a->mlp_e, a->FFN);
        run_matvec<NC>(ctl, buf, rg, NT);
        // the slice buffer is free: fetch the next layer's (or next step's layer 0)
        if (l + 1 < a->NL || step + 1 < a->n_gen) fetch_slice(a, B, role, l + 1 < a->NL ? l + 1 : 0, u0, nu);
        run_epilogue<NC>(a, ctl, role, rg, u0, nu, emb);
        publish(cnt + out_ctr[role] * 32, 1);
      } else if (role == N_MV_ROLES) {
        const AttItem it = att_item(a, ctl, l, item);
        if (!att_staged) att_stage(a, ctl, it.kbase, 0, it.kpre, true, true);
        if (!wait_count(cnt + C_P1 * 32, (inst + 1) * in_per[4], a->err)) {
          asm volatile("cp.async.wait_all;" ::: "memory");
          ok = false;
          break;
        }
        att_compute(a, ctl, l, item, true);
        publish(cnt + C_P2 * 32, 1);
        // stage the next layer's cached rows while the other phases run
        att_staged = l + 1 < a->NL;
        if (att_staged) {
          const AttItem nx = att_item(a, ctl, l + 1, item);
          att_stage(a, ctl, nx.kbase, 0, nx.kpre, true, true);
        }
      }
    }
    if (!ok) break;
    // ---- head (:437-443)
    if (!wait_count(cnt + C_P5 * 32, (unsigned)((step + 1) * a->NL) * R.n[3], a->err)) break;
    head_scan<NC>(a, ctl, step & 1);
    publish(cnt + C_HEAD * 32, 1);
    if (!wait_count(cnt + C_HEAD * 32, (unsigned)(step + 1) * ncta, a->err)) break;
    head_reduce(a, ctl, step & 1, step);
    att_staged = false;
  }
  // drain copies still in flight before the CTA's shared memory is released
  if (B.pend[0]) buf_wait(B, 0, a->err);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  if (cta == 0 && tid < a->ncols) {
    a->col_tok[tid] = ctl->tok[tid];
    a->col_pos[tid] = ctl->pos[tid];
  }
}

template <int NC>
cudaError_t set_smem(size_t smem) {
  return cudaFuncSetAttribute(persistent_decode_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

}  // namespace

size_t persistent_smem_bytes(const PersistArgs& a) { return p_layout(a, a.ncols <= 1 ? 1 : 4).total; }

// Every matvec role gets 1, 2 or 4 units per CTA; among the plans whose CTAs
// (plus one per attention item) fit the grid and whose shared memory fits,
// the one with the smallest largest per-CTA weight slice wins.
bool persistent_plan(PersistArgs& a, int nctas, int smem_optin) {
  if (a.ncols < 1 || a.ncols > 4 || nctas > 32 * HR_MAX || a.HQ % a.HKV) return false;
  const int opts[3] = {1, 2, 4};
  bool found = false;
  long best_cost = 0;
  int best[4] = {1, 1, 1, 1};
  PersistArgs t = a;
  for (int i0 = 0; i0 < 3; ++i0)
    for (int i1 = 0; i1 < 3; ++i1)
      for (int i2 = 0; i2 < 3; ++i2)
        for (int i3 = 0; i3 < 3; ++i3) {
          t.gpc[0] = opts[i0]; t.gpc[1] = opts[i1]; t.gpc[2] = opts[i2]; t.gpc[3] = opts[i3];
          if (t.gpc[2] * 2 > 4) continue;                       // slice_matvec covers up to 4 groups
          const Roles R = roles_of(t);
          if (R.first[N_MV_ROLES + 1] > nctas) continue;
          if (persistent_smem_bytes(t) + sizeof(Ctl) > (size_t)smem_optin) continue;
          long cost = 0;
          for (int r = 0; r < N_MV_ROLES; ++r) {
            const long c = (long)t.gpc[r] * role_gpu(r) * role_nt(t, r);
            cost = cost > c ? cost : c;
          }
          if (!found || cost < best_cost) { found = true; best_cost = cost; for (int r = 0; r < 4; ++r) best[r] = t.gpc[r]; }
        }
  if (!found) return false;
  for (int r = 0; r < 4; ++r) a.gpc[r] = best[r];
  return true;
}

cudaError_t launch_persistent_decode(const PersistArgs& a, int nctas, cudaStream_t s) {
  const int NC = a.ncols <= 1 ? 1 : 4;
  const size_t smem = p_layout(a, NC).total;
  cudaError_t e = NC == 1 ? set_smem<1>(smem) : set_smem<4>(smem);
  if (e != cudaSuccess) return e;
  int per = 0;
  e = NC == 1 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, persistent_decode_kernel<1>, PT, smem)
              : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, persistent_decode_kernel<4>, PT, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, nsm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (per < 1 || nctas > per * nsm || roles_of(a).first[N_MV_ROLES + 1] > nctas)
    return cudaErrorCooperativeLaunchTooLarge;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nctas);
  cfg.blockDim = dim3(PT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (NC == 1) return cudaLaunchKernelEx(&cfg, persistent_decode_kernel<1>, a);
  return cudaLaunchKernelEx(&cfg, persistent_decode_kernel<4>, a);
}

}  // namespace bfp
