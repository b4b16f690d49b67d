// layer1.cu -- the attention half of one decode layer for a single sequence
// (one column), in ONE launch of one thread-block cluster:
//
//   n1 = tile_quantize(rmsnorm_fp(h, g1))                 (gen_smollm_blockfp_full.py:263-264)
//   q, k, v = matvec(n1, Wq | Wk | Wv)                     (:265-267)
//   rope_fp on q and k, K/V row written at kv_pos          (:268-272)
//   attention over positions 0..pos, tile_quantize(fpq)    (:273-283)
//   h1 = fpq(h + matvec(attn, Wo))                         (:284-285)
//
// Why one cluster: at one column the layer is a chain of short dependent
// stages, and every kernel boundary costs about a microsecond.  Here the
// stages hand over through distributed shared memory and cluster barriers
// instead of kernel boundaries.
//
// Roles.  The cluster has one CTA per 64-row "unit" of the fused Q|K|V
// matrix: units 0..HQ-1 are the query heads, HQ..HQ+HKV-1 the key heads and
// the rest the value heads (rows 64 r .. 64 r + 63).  Every CTA computes the
// RMSNorm of h itself (no exchange needed), then the 64 rows of its unit, so
// RoPE's pairs (d, d + 32) are inside one CTA.  Key / value CTAs write their
// row to the KV arena and expose it in shared memory; each query CTA then
// runs the attention of its head with the cached rows staged in shared
// memory before the dependency wait, and exposes its 64 outputs.  Finally
// every CTA gathers the whole attention vector and computes its share of
// the O row groups with the residual add.
//
// Every weight byte a CTA needs (its Q/K/V unit, its O row groups, gamma)
// and the cached K/V rows are in flight by TMA bulk copies / cp.async
// before griddepcontrol.wait, so they overlap the previous kernel.
//
// Arithmetic is the reference's, operation for operation (the same device
// helpers as the multi-kernel path); compile with -fmad=false.
#include "bfp_device.cuh"
#include "kernels.cuh"
#include "stamps.cuh"

#include <cooperative_groups.h>

namespace bfp {

namespace {

constexpr int A_THREADS = 512;
constexpr int A_HD = 64;
constexpr int A_PLAN_MAX = 512;      // pairwise-sum plan entries kept in shared memory
// First thread of the 64 that accumulate attn: warps 2 and 3.  Measured:
// the same loop on warps 0 and 1 ran at twice the cycles per position on
// warp 0 (warp 1 unaffected); warps 2 / 3 run it at the warp-1 rate.
#ifndef BFP200_VW
#define BFP200_VW 64
#endif
constexpr int A_VW = BFP200_VW;
constexpr int A_SW = 0;              // the warp that runs the single-warp reductions

__device__ __forceinline__ void a_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void a_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ unsigned a_smem(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void a_cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void a_cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

__device__ __forceinline__ void a_mbar_init(unsigned long long* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(a_smem(bar)) : "memory");
}
__device__ __forceinline__ void a_mbar_expect(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(a_smem(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void a_bulk(void* dst, const void* src, unsigned bytes, unsigned long long* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(a_smem(dst)), "l"(src), "r"(bytes), "r"(a_smem(bar)) : "memory");
}
// Bounded wait for phase 0 of a local copy barrier; false when it gave up.
__device__ __forceinline__ bool a_mbar_wait(unsigned long long* bar) {
  for (long long it = 0; it < (1LL << 26); ++it) {
    unsigned ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok) : "r"(a_smem(bar)) : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ __forceinline__ int a_dp2a_lo_ss(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int a_dp2a_hi_ss(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int a_dp2a_lo_su(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int a_dp2a_hi_su(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
// exact 16-term tile sum of x (int16) against w given as signed-high /
// unsigned-low byte planes: 256 * sum x*(w>>8) + sum x*(w&255)
__device__ __forceinline__ long long a_tile_sum(const uint4 x0, const uint4 x1, const uint4 wh, const uint4 wl) {
  int A = 0, B = 0;
  A = a_dp2a_lo_ss(x0.x, wh.x, A); A = a_dp2a_hi_ss(x0.y, wh.x, A);
  A = a_dp2a_lo_ss(x0.z, wh.y, A); A = a_dp2a_hi_ss(x0.w, wh.y, A);
  A = a_dp2a_lo_ss(x1.x, wh.z, A); A = a_dp2a_hi_ss(x1.y, wh.z, A);
  A = a_dp2a_lo_ss(x1.z, wh.w, A); A = a_dp2a_hi_ss(x1.w, wh.w, A);
  B = a_dp2a_lo_su(x0.x, wl.x, B); B = a_dp2a_hi_su(x0.y, wl.x, B);
  B = a_dp2a_lo_su(x0.z, wl.y, B); B = a_dp2a_hi_su(x0.w, wl.y, B);
  B = a_dp2a_lo_su(x1.x, wl.z, B); B = a_dp2a_hi_su(x1.y, wl.z, B);
  B = a_dp2a_lo_su(x1.z, wl.w, B); B = a_dp2a_hi_su(x1.w, wl.w, B);
  return ((long long)A << 8) + (long long)B;
}

// m * 2^(e-15) exactly (|m| <= 32768, |e| <= 127) with one double addition
// and integer bit assembly: the double 2^(52+k) + (m + 2^31) 2^k (biased
// exponent 1075 + k, fraction m + 2^31) minus (2^52 + 2^31) 2^k; both lie
// on the 2^k grid within a factor two of each other, so the difference is
// exact.  Equals bfp_decode(m, e) for every input, without the int -> double
// conversion (a slow instruction inside the accumulation loop).
__device__ __forceinline__ double a_decode(int m, int e) {
  const unsigned hi = (unsigned)(1060 + e) << 20;             // 1075 + (e - 15)
  const double big = __hiloint2double((int)hi, (int)((unsigned)m ^ 0x80000000u));
  const double neg = __hiloint2double((int)(hi | 0x80000000u), (int)0x80000000u);
  return __dadd_rn(big, neg);
}

}  // namespace

// ---------------------------------------------------------------------------
// shared-memory layout.  Everything up to `wo` is common to all CTAs
// (distributed shared memory addresses a peer by the same offsets); the rest
// depends on the CTA's role.
// ---------------------------------------------------------------------------
struct L1Layout {
  int bar, wq, wqe, gam, hx, nm, ne, cs, rowm, rowe, attm, atte, red_acc, red_max, rot, misc;
  int wo, woe;                      // this CTA's O row groups (og of them)
  int plan, sc, ks, kes, vs, ves;   // query CTAs only (after the O weights)
  int total;
};

// og: O row groups of the CTA; att: a query (attention) CTA; ch: cached K/V
// positions staged in shared memory.
__host__ __device__ inline L1Layout l1_layout(int D, int og, bool att, int maxc, int ch) {
  const int NT = D / 16;
  L1Layout L;
  int off = 0;
  auto take = [&](int b) { const int o = off; off = (off + b + 127) & ~127; return o; };
  L.bar = take(32);
  L.wq = take(4 * NT * 512);
  L.wqe = take(4 * NT * 16);
  L.gam = take(D * 8);
  L.hx = take(D * 8);
  L.nm = take(D * 2);
  L.ne = take(NT + 16);
  L.cs = take(64 * 8);
  L.rowm = take(64 * 2);
  L.rowe = take(16);
  L.attm = take(64 * 2);
  L.atte = take(16);
  // the RMSNorm squares (D doubles) share this area with the matvec reductions
  const int red = 8 * 64 * 8 + 8 * 64 * 4;
  L.red_acc = take(red > D * 8 ? red : D * 8);
  L.red_max = L.red_acc + 8 * 64 * 8;
  L.rot = take(64 * 8);
  L.misc = take(2048);
  L.wo = take(og * NT * 512);
  L.woe = take(og * NT * 16);
  L.plan = L.sc = L.ks = L.kes = L.vs = L.ves = off;
  if (att) {
    L.plan = take(A_PLAN_MAX * 2);
    L.sc = take(maxc * 8);
    L.ks = take(ch * 128);
    L.kes = take(ch * 4);
    L.vs = take(ch * 128);
    L.ves = take(ch * 4);
  }
  L.total = off;
  return L;
}

// O row groups of CTA r: the units are ordered key/value CTAs first, then the
// query CTAs (whose shared memory also holds the attention buffers); the
// first (OG % NU) of that order take one group more.
__host__ __device__ inline void l1_o_groups(int r, int HQ, int NU, int OG, int* start, int* cnt) {
  const int p = r >= HQ ? r - HQ : (NU - HQ) + r;
  const int base = OG / NU, extra = OG % NU;
  *cnt = base + (p < extra ? 1 : 0);
  *start = p * base + (p < extra ? p : extra);
}

// K staging: 16-byte chunk u of position t at u ^ (t & 7) (a thread per
// position reads a 128-byte row without bank conflicts).
__device__ __forceinline__ int l1_kswz(int i) { return (i & ~7) | ((i ^ (i >> 3)) & 7); }

// Stage-dump offsets within one column (bfp200_fwd_layer's stage layout:
// n1 q k v attn o h1 ... with lengths D D KVD KVD D D D ...; here QD = D).
__device__ __forceinline__ int l1_stage_off(int s, int D, int KVD) {
  const int len[7] = {D, D, KVD, KVD, D, D, D};
  int o = 0;
  for (int i = 0; i < s; ++i) o += len[i];
  return o;
}

// ---------------------------------------------------------------------------
// Matvec of up to 64 rows (4 row groups of one DevMat, weights in shared
// memory) against one quantized column x (shared memory), matvec_hw_golden
// (:217-232): thread (row = tid & 63, sub = tid >> 6) takes K tiles sub,
// sub + 8, ...; the row maximum of the tile exponents and the int64 sums of
// floor-shifted tile sums are combined through shared memory.  Returns the
// exact real output clip(acc) * 2^(M - 30) on threads tid < nrows.
// ---------------------------------------------------------------------------
template <int MAXJ>
__device__ __forceinline__ double l1_matvec64(const uint8_t* wsm, const int8_t* wesm, int nrows, int NT,
                                              const int16_t* xm, const int8_t* xe, long long* red_acc,
                                              int* red_max) {
  const int tid = threadIdx.x;
  const int row = tid & 63, sub = tid >> 6;
  const int g = row >> 4, ri = row & 15;
  const bool live = row < nrows;
  long long S[MAXJ];
  int E[MAXJ];
  int M = -100000;
  #pragma unroll
  for (int j = 0; j < MAXJ; ++j) {
    const int t = sub + 8 * j;
    S[j] = 0;
    E[j] = -100000;
    if (live && t < NT) {
      const uint4* wp = reinterpret_cast<const uint4*>(wsm + ((size_t)g * NT + t) * 512);
      const uint4* xp = reinterpret_cast<const uint4*>(xm + t * 16);
      S[j] = a_tile_sum(xp[0], xp[1], wp[ri], wp[16 + ri]);
      E[j] = (int)xe[t] + (int)wesm[(g * NT + t) * 16 + ri];
      M = E[j] > M ? E[j] : M;
    }
  }
  red_max[sub * 64 + row] = M;
  __syncthreads();
  M = red_max[row];
  #pragma unroll
  for (int s = 1; s < 8; ++s) M = max(M, red_max[s * 64 + row]);
  long long acc = 0;
  #pragma unroll
  for (int j = 0; j < MAXJ; ++j) {
    const int sh = M - E[j];
    acc += (sh > ALIGN_MAX) ? 0LL : (S[j] >> sh);     // :223-228 (dead tiles: E = -1e5, sh > 47)
  }
  red_acc[sub * 64 + row] = acc;
  __syncthreads();
  double out = 0.0;
  if (tid < nrows) {
    long long s = 0;
    #pragma unroll
    for (int k = 0; k < 8; ++k) s += red_acc[k * 64 + tid];
    s = s > SAT_HI ? SAT_HI : (s < SAT_LO ? SAT_LO : s);          // :229-231
    out = (double)s * pow2(M - 30);                             // :232, exact
  }
  return out;
}

// attn_d = sum_t sm[t] * v[t][d], sequential in t (:280-281), over the
// staged rows 0..nv-1 (int16 mantissas [t][64] and packed tile exponents
// [t]) of dimension d = this thread.  Out of line: inside the kernel body
// the loop competes for registers with everything live around it, and
// spilled operands serialise it; as a call it gets its own allocation.
__device__ __noinline__ double l1_attn_accumulate(const int16_t* vs, const unsigned* ves, const double* sc,
                                                   int nv, int d) {
  const int sh = 8 * (d >> 4);
  const int16_t* vrow = vs + d;
  double acc = 0.0;
  int t = 0;
  // 16 rows' loads and decodes issued ahead of their 16 dependent adds
  // (groups of 4: +23 us per token)
  for (; t + 16 <= nv; t += 16) {
    int m16[16], e16[16];
    double s16[16];
    #pragma unroll
    for (int u = 0; u < 16; ++u) {
      m16[u] = vrow[(t + u) * A_HD];
      e16[u] = (int)(int8_t)(ves[t + u] >> sh);
      s16[u] = sc[t + u];
    }
    #pragma unroll
    for (int u = 0; u < 16; ++u) acc = __dadd_rn(acc, __dmul_rn(s16[u], a_decode(m16[u], e16[u])));
  }
  for (; t < nv; ++t) acc = __dadd_rn(acc, __dmul_rn(sc[t], a_decode(vrow[t * A_HD], (int)(int8_t)(ves[t] >> sh))));
  return acc;
}

// ---------------------------------------------------------------------------
// The kernel.  Grid = one cluster of NU = HQ + 2 HKV CTAs.
// ---------------------------------------------------------------------------
template <int MAXJ>
__global__ void __launch_bounds__(A_THREADS, 1)
bfp_attn_block_kernel(L1Args a) {
  extern __shared__ __align__(128) unsigned char smem[];
  namespace cg = cooperative_groups;
  cg::cluster_group cl = cg::this_cluster();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = (int)cl.block_rank();
  const int D = a.D, NT = D / 16, HQ = a.HQ, HKV = a.HKV, NU = HQ + 2 * HKV, KVD = HKV * A_HD;
  const int grp = HQ / HKV;
  const bool is_q = r < HQ, is_k = r >= HQ && r < HQ + HKV;
  const bool rope = r < HQ + HKV;
  int og0, ogn;
  l1_o_groups(r, HQ, NU, NT, &og0, &ogn);
  const L1Layout L = l1_layout(D, ogn, is_q, a.kv.MAX_CTX, a.ch);
  unsigned long long* bar = reinterpret_cast<unsigned long long*>(smem + L.bar);
  uint8_t* wq = smem + L.wq;
  int8_t* wqe = reinterpret_cast<int8_t*>(smem + L.wqe);
  double* gam = reinterpret_cast<double*>(smem + L.gam);
  double* hx = reinterpret_cast<double*>(smem + L.hx);
  int16_t* nm = reinterpret_cast<int16_t*>(smem + L.nm);
  int8_t* ne = reinterpret_cast<int8_t*>(smem + L.ne);
  double* cs = reinterpret_cast<double*>(smem + L.cs);
  int16_t* rowm = reinterpret_cast<int16_t*>(smem + L.rowm);
  int8_t* rowe = reinterpret_cast<int8_t*>(smem + L.rowe);
  int16_t* attm = reinterpret_cast<int16_t*>(smem + L.attm);
  int8_t* atte = reinterpret_cast<int8_t*>(smem + L.atte);
  long long* red_acc = reinterpret_cast<long long*>(smem + L.red_acc);
  int* red_max = reinterpret_cast<int*>(smem + L.red_max);
  double* sq = reinterpret_cast<double*>(smem + L.red_acc);      // RMSNorm squares (before the matvec)
  double* rot = reinterpret_cast<double*>(smem + L.rot);
  double* s_misc = reinterpret_cast<double*>(smem + L.misc);       // [0] r, [1] sum, [2..17] maxima
  int* s_lo = reinterpret_cast<int*>(smem + L.misc + 256);
  int* s_len = s_lo + 96;
  double* s_val = reinterpret_cast<double*>(smem + L.misc + 1024);   // 128 doubles
  uint8_t* wo = smem + L.wo;
  int8_t* woe = reinterpret_cast<int8_t*>(smem + L.woe);
  unsigned short* s_plan = reinterpret_cast<unsigned short*>(smem + L.plan);
  double* sc = reinterpret_cast<double*>(smem + L.sc);
  uint4* ks = reinterpret_cast<uint4*>(smem + L.ks);
  unsigned* kes = reinterpret_cast<unsigned*>(smem + L.kes);
  uint4* vs = reinterpret_cast<uint4*>(smem + L.vs);
  unsigned* ves = reinterpret_cast<unsigned*>(smem + L.ves);
  __shared__ __align__(16) int16_t s_qm[64];
  __shared__ int s_qe[4];
  __shared__ int s_fail;

  const int slot = a.col_slot[0], pos = a.col_pos[0];   // written by an earlier, completed launch
  const int T = pos + 1;
  const int kvh = is_q ? r / grp : (is_k ? r - HQ : r - HQ - HKV);
  const size_t kbase = (((size_t)slot * a.kv.NL + a.layer) * HKV + kvh) * a.kv.MAX_CTX;

  BFP_STAMP(0, a.layer, r, 0);
  a_pdl_trigger();
  // ---- 0. before the dependency wait: weights, gamma, RoPE factors, cached K/V
  if (tid == 0) {
    s_fail = 0;
    a_mbar_init(&bar[0]);
    a_mbar_init(&bar[1]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    const unsigned wqb = 4u * NT * 512, wqeb = 4u * NT * 16, gb = (unsigned)D * 8;
    a_mbar_expect(&bar[0], wqb + wqeb + gb);
    a_bulk(wq, a.Wqkv.wm + (size_t)(4 * r) * NT * 512, wqb, &bar[0]);
    a_bulk(wqe, a.Wqkv.we + (size_t)(4 * r) * NT * 16, wqeb, &bar[0]);
    a_bulk(gam, a.gamma, gb, &bar[0]);
    const unsigned wob = (unsigned)ogn * NT * 512, woeb = (unsigned)ogn * NT * 16;
    a_mbar_expect(&bar[1], wob + woeb);
    if (ogn > 0) {
      a_bulk(wo, a.Wo.wm + (size_t)og0 * NT * 512, wob, &bar[1]);
      a_bulk(woe, a.Wo.we + (size_t)og0 * NT * 16, woeb, &bar[1]);
    }
  }
  if (rope && tid < 64) cs[tid] = a.rope_cs[(size_t)pos * 64 + tid];   // (cos, sin) of the 32 pairs (:253-254)
  const unsigned short* plan = nullptr;
  if (is_q) {
    const int nst = min(pos, a.ch);                     // cached rows staged
    const uint4* ksrc = reinterpret_cast<const uint4*>(a.kv.km + kbase * A_HD);
    const uint4* vsrc = reinterpret_cast<const uint4*>(a.kv.vm + kbase * A_HD);
    for (int i = tid; i < nst * 8; i += A_THREADS) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(a_smem(ks + l1_kswz(i))), "l"(ksrc + i) : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(a_smem(vs + i)), "l"(vsrc + i) : "memory");
    }
    const unsigned* kesrc = reinterpret_cast<const unsigned*>(a.kv.ke + kbase * 4);
    const unsigned* vesrc = reinterpret_cast<const unsigned*>(a.kv.ve + kbase * 4);
    for (int i = tid; i < nst; i += A_THREADS) {
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(a_smem(kes + i)), "l"(kesrc + i) : "memory");
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(a_smem(ves + i)), "l"(vesrc + i) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    const unsigned short* gp = a.pw_data + a.pw_off[T];
    const int np = 3 * (int)gp[0] + (int)gp[1];
    if (np <= A_PLAN_MAX) {
      for (int i = tid; i < np; i += A_THREADS) s_plan[i] = gp[i];
      plan = s_plan;
    } else {
      plan = gp;
    }
  }
  // Two passes over the same code.  Pass 0 ("dry") runs before the
  // dependency wait, on placeholder inputs in shared memory and a short V
  // loop, with no global, peer or cluster-barrier side effects: it only
  // pulls the kernel's instructions into this SM's instruction caches while
  // the previous kernel finishes (the real pass, run once per layer, would
  // otherwise stall on instruction fetches at every new code line).  Pass 1
  // is the real computation.  The loop must stay a loop (unroll 1): both
  // passes have to execute the same instruction addresses.
  #pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
  const bool dry = pass == 0;
  if (!dry) {
    a_pdl_wait();
    BFP_STAMP(0, a.layer, r, 1);
  }
  // (the dry pass must not read h from global memory: a line cached before
  // the previous kernel's write would be stale)
  const int16_t* hin_m = dry ? nm : a.hm;
  const int8_t* hin_e = dry ? ne : a.he;

  // ---- 1. n1 = tile_quantize(rmsnorm_fp(h, g1))   (:236-238, :263-264)
  for (int i = tid; i < D; i += A_THREADS) {
    const double x = bfp_decode(hin_m[i], hin_e[i >> 4]);
    hx[i] = x;
    sq[i] = __dmul_rn(x, x);
  }
  if (!dry && tid == 0 && !a_mbar_wait(&bar[0])) s_fail = 1;
  __syncthreads();
  if (warp == A_SW) {
    const double sum = np_sum_warp(sq, D, s_lo, s_len, s_val);
    if (lane == 0) s_misc[0] = __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)D), a.eps));
  }
  __syncthreads();
  {
    const double rr = s_misc[0];
    for (int base = 0; base < NT; base += 64) {
      double y[2];
      bool valid[2];
      #pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int tile = base + q * 32 + (tid >> 4);
        valid[q] = tile < NT;
        const int i = valid[q] ? tile * 16 + (tid & 15) : 0;
        y[q] = valid[q] ? __ddiv_rn(__dmul_rn(hx[i], gam[i]), rr) : 0.0;
      }
      int16_t m[2];
      int e[2];
      tile_quantize_requant_16lanes_n<2>(y, valid, m, e);
      __syncthreads();                                  // (the dry pass reads nm / ne as its input)
      #pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int tile = base + q * 32 + (tid >> 4);
        if (valid[q]) {
          nm[tile * 16 + (tid & 15)] = m[q];
          if ((tid & 15) == 0) ne[tile] = (int8_t)e[q];
        }
      }
    }
  }
  __syncthreads();
  if (!dry) BFP_STAMP(0, a.layer, r, 2);
  if (!dry && a.dbg && r == 0)
    for (int i = tid; i < D; i += A_THREADS) a.dbg[l1_stage_off(0, D, KVD) + i] = bfp_decode(nm[i], ne[i >> 4]);

  // ---- 2. this unit's 64 rows of q | k | v   (:265-267), RoPE (:268-269)
  // The warming pass leaves this matvec out: the next layer's dependency wait
  // returns when that pass ends, and fetching this code cold in the real pass
  // costs less than running the 64 x 36-tile matvec here (same-box A/B:
  // -12 us per token).
  const double out = dry ? 0.0 : l1_matvec64<MAXJ>(wq, wqe, 64, NT, nm, ne, red_acc, red_max);
  if (tid < 64) {
    int qe;
    const int16_t qm = tile_quantize_16lanes(out, &qe);           // fp_quantize_vec of the matvec (:233)
    if (rope) {
      // rope_fp (:250-258): out[j] = a c - b s, out[j + 32] = b c + a s
      // (a = x[j], b = x[j + 32]), then fpq
      const double own = bfp_decode(qm, qe);
      rot[tid] = own;
      asm volatile("bar.sync 1, 64;" ::: "memory");
      const double partner = rot[tid ^ 32];
      const int jj = tid & 31;
      const double c = cs[2 * jj], s = cs[2 * jj + 1];
      const double y = tid < 32 ? __dsub_rn(__dmul_rn(own, c), __dmul_rn(partner, s))
                                : __dadd_rn(__dmul_rn(own, c), __dmul_rn(partner, s));
      int re;
      const int16_t rm = tile_quantize_16lanes(y, &re);
      rowm[tid] = rm;
      if ((tid & 15) == 0) rowe[tid >> 4] = (int8_t)re;
      if (!dry && a.dbg) a.dbg[l1_stage_off(1, D, KVD) + r * 64 + tid] = bfp_decode(rm, re);   // q | k rows
    } else {
      rowm[tid] = qm;                                   // v: stored as produced (:272)
      if ((tid & 15) == 0) rowe[tid >> 4] = (int8_t)qe;
      if (!dry && a.dbg) a.dbg[l1_stage_off(1, D, KVD) + r * 64 + tid] = bfp_decode(qm, qe);
    }
  }
  __syncthreads();
  if (!dry && !is_q) {                                  // K / V row at kv_pos (:270-272)
    int16_t* dm = is_k ? a.kv.km : a.kv.vm;
    int8_t* de = is_k ? a.kv.ke : a.kv.ve;
    if (tid < 8) reinterpret_cast<uint4*>(dm + (kbase + pos) * A_HD)[tid] = reinterpret_cast<const uint4*>(rowm)[tid];
    else if (tid == 8) *reinterpret_cast<unsigned*>(de + (kbase + pos) * 4) = *reinterpret_cast<const unsigned*>(rowe);
  }
  if (!dry) {
    BFP_STAMP(0, a.layer, r, 3);
    a_cluster_arrive();                                 // #1: K / V rows are in shared memory
    a_cluster_wait();
    BFP_STAMP(0, a.layer, r, 4);
  }

  // ---- 3. attention of query head r   (:273-283)
  if (is_q) {
    const int krank = HQ + kvh, vrank = HQ + HKV + kvh;
    const int16_t* rk = dry ? rowm : cl.map_shared_rank(rowm, krank);
    const int8_t* rke = dry ? rowe : cl.map_shared_rank(rowe, krank);
    const int16_t* rv = dry ? rowm : cl.map_shared_rank(rowm, vrank);
    const int8_t* rve = dry ? rowe : cl.map_shared_rank(rowe, vrank);
    if (tid < 64) s_qm[tid] = rowm[tid];
    if (tid < 4) s_qe[tid] = rowe[tid];
    if (!dry) {
      if (pos < a.ch) {                                 // the new row joins the staged rows
        if (tid < 8) ks[l1_kswz(pos * 8 + tid)] = reinterpret_cast<const uint4*>(rk)[tid];
        else if (tid < 16) vs[pos * 8 + tid - 8] = reinterpret_cast<const uint4*>(rv)[tid - 8];
        else if (tid == 16) kes[pos] = *reinterpret_cast<const unsigned*>(rke);
        else if (tid == 17) ves[pos] = *reinterpret_cast<const unsigned*>(rve);
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    }
    __syncthreads();
    if (!dry) BFP_STAMP(0, a.layer, r, 5);
    // the dry pass reads no row beyond the staged chunk (arena or peer)
    const int Tp = dry ? min(T, a.ch) : T;
    const int nin = min(Tp, a.ch);                      // positions read from shared memory
    // scores[t] = float(np.dot(q, k_t)) / math.sqrt(HD) (:278): exact tile
    // sums, one rounding; dividing by 8 = multiplying by 1/8 (exact)
    const bool pow2_hd = a.inv_hd != 0.0;
    double lmax = -INFINITY;
    for (int t = tid; t < Tp; t += A_THREADS) {
      uint4 kk[8];
      unsigned ke4;
      if (t < nin) {
        #pragma unroll
        for (int u = 0; u < 8; ++u) kk[u] = ks[t * 8 + (u ^ (t & 7))];
        ke4 = kes[t];
      } else {                                          // beyond the staged chunk: the arena / the peer
        const uint4* kr = t == pos ? reinterpret_cast<const uint4*>(rk)
                                   : reinterpret_cast<const uint4*>(a.kv.km + (kbase + t) * A_HD);
        #pragma unroll
        for (int u = 0; u < 8; ++u) kk[u] = kr[u];
        ke4 = t == pos ? *reinterpret_cast<const unsigned*>(rke)
                       : *reinterpret_cast<const unsigned*>(a.kv.ke + (kbase + t) * 4);
      }
      long long S[4];
      int E[4];
      #pragma unroll
      for (int jt = 0; jt < 4; ++jt) {
        const uint4* qp = reinterpret_cast<const uint4*>(s_qm) + 2 * jt;   // q of tile jt, 16-bit pairs
        S[jt] = tile_sum16_dp2a(qp[0], qp[1], kk[2 * jt], kk[2 * jt + 1]);
        E[jt] = s_qe[jt] + (int)(int8_t)(ke4 >> (8 * jt));
      }
      const double dot = exact_tile_dot4(S, E);
      const double v = pow2_hd ? __dmul_rn(dot, a.inv_hd) : __ddiv_rn(dot, a.sqrt_hd);
      sc[t] = v;
      lmax = v > lmax ? v : lmax;
    }
    // softmax_fp (:245-247): e = exp(x - max); e / e.sum()
    for (int off = 16; off; off >>= 1) {
      const double o = __shfl_xor_sync(0xffffffffu, lmax, off);
      lmax = o > lmax ? o : lmax;
    }
    if (lane == 0) s_misc[2 + warp] = lmax;
    __syncthreads();
    if (!dry) BFP_STAMP(0, a.layer, r, 6);
    double mx = s_misc[2];
    for (int w = 1; w < A_THREADS / 32; ++w) mx = s_misc[2 + w] > mx ? s_misc[2 + w] : mx;
    for (int t = tid; t < Tp; t += A_THREADS) sc[t] = exp(__dsub_rn(sc[t], mx));
    __syncthreads();
    if (warp == A_SW) {
      const double S = np_sum_warp_plan(sc, T, plan, s_val);    // (dry: the entries past Tp are stale)
      if (lane == 0) s_misc[1] = S;
    }
    __syncthreads();
    if (!dry) BFP_STAMP(0, a.layer, r, 7);
    const double Ssum = s_misc[1];
    for (int t = tid; t < Tp; t += A_THREADS) sc[t] = __ddiv_rn(sc[t], Ssum);
    __syncthreads();
    if (!dry) BFP_STAMP(0, a.layer, r, 8);
    // attn[h] += sm[t] * v[t], sequential in t (:280-281)
    if (tid >= A_VW && tid < A_VW + A_HD) {
      const int d = tid - A_VW;                         // this thread's dimension
      const int nv = dry ? min(nin, 16) : nin;            // (dry: one whole group of the loop)
      const int Tv = dry ? nv : Tp;
      if (!dry) { BFP_STAMP_T(A_VW, 3, a.layer, r, 0); BFP_STAMP_T(A_VW + 32, 3, a.layer, r, 4); }
      double acc = l1_attn_accumulate(reinterpret_cast<const int16_t*>(vs), ves, sc, nv, d);
#ifdef BFP200_STAMPS
      if (!dry) { s_misc[20 + (d >> 5)] = acc; __syncwarp(); BFP_STAMP_T(A_VW, 3, a.layer, r, 2); BFP_STAMP_T(A_VW + 32, 3, a.layer, r, 6); }
#endif
      for (int t = nv; t < Tv; ++t) {                   // rows beyond the staged chunk
        const int m = t == pos ? rv[d] : a.kv.vm[(kbase + t) * A_HD + d];
        const int e = t == pos ? (int)rve[d >> 4] : (int)a.kv.ve[(kbase + t) * 4 + (d >> 4)];
        acc = __dadd_rn(acc, __dmul_rn(sc[t], a_decode(m, e)));
      }
      int e;
      int16_t m = tile_quantize_16lanes(acc, &e);        // fpq(attn)   (:282)
      const unsigned bal = __ballot_sync(0xffffffffu, m == (int16_t)-32768);
      const bool has_min = ((bal >> (lane & 16)) & 0xFFFFu) != 0;
      m = requant_mant(m, has_min && e < 127);           // tile_quantize(attn)   (:283)
      e = requant_exp(e, has_min);
      attm[d] = m;
      if ((d & 15) == 0) atte[d >> 4] = (int8_t)e;
      if (!dry && a.dbg) a.dbg[l1_stage_off(4, D, KVD) + r * 64 + d] = bfp_decode(m, e);
      if (!dry) { BFP_STAMP_T(A_VW, 3, a.layer, r, 3); BFP_STAMP_T(A_VW + 32, 3, a.layer, r, 7); }
    }
    __syncthreads();
    if (!dry) BFP_STAMP(0, a.layer, r, 9);
  }
  if (!dry) {
    a_cluster_arrive();                                 // #2: attention outputs are in shared memory
    a_cluster_wait();
    BFP_STAMP(0, a.layer, r, 10);
  }

  // ---- 4. gather the attention vector, O rows of this CTA, residual (:284-285)
  {
    int16_t* am = nm;                                   // n1 is dead: reuse its buffer
    int8_t* ae = ne;
    if (tid < HQ * 32) {
      const int h = tid >> 5;
      const unsigned* src = reinterpret_cast<const unsigned*>(dry ? attm : cl.map_shared_rank(attm, h));
      reinterpret_cast<unsigned*>(am + h * A_HD)[lane] = src[lane];
    } else if (tid < HQ * 32 + HQ) {
      const int h = tid - HQ * 32;
      const unsigned* src = reinterpret_cast<const unsigned*>(dry ? atte : cl.map_shared_rank(atte, h));
      reinterpret_cast<unsigned*>(ae)[h] = src[0];
    }
    if (!dry && tid == 0 && ogn > 0 && !a_mbar_wait(&bar[1])) s_fail = 1;
    __syncthreads();
    if (!dry) {
      BFP_STAMP(0, a.layer, r, 11);
      a_cluster_arrive();                               // #3: peers may exit once everyone has gathered
    }
    if (ogn > 0) {
      const int nrows = 16 * ogn;
      const double o_real = l1_matvec64<MAXJ>(wo, woe, nrows, NT, am, ae, red_acc, red_max);
      if (warp * 32 < nrows) {                          // whole warps: the quantizer shuffles
        const bool live = tid < nrows;
        int qe;
        int16_t qm = tile_quantize_16lanes(o_real, &qe);             // o = matvec (:284)
        const int orow = og0 * 16 + (live ? tid : 0);
        if (!dry && a.dbg && live) a.dbg[l1_stage_off(5, D, KVD) + orow] = bfp_decode(qm, qe);
        const double y = __dadd_rn(live ? hx[orow] : 0.0, bfp_decode(qm, qe));   // fpq(h + o)   (:285)
        qm = tile_quantize_16lanes(y, &qe);
        if (!dry && live) {
          a.h1m[orow] = qm;
          if ((tid & 15) == 0) a.h1e[orow >> 4] = (int8_t)qe;
          if (a.dbg) a.dbg[l1_stage_off(6, D, KVD) + orow] = bfp_decode(qm, qe);
        }
      }
    }
    __syncthreads();                                    // (idle warps wait on the CTA barrier)
  }
  }   // pass
  BFP_STAMP(0, a.layer, r, 12);
  if (tid == 0 && s_fail) atomicExch(a.err, 4);
  a_cluster_wait();
  BFP_STAMP(0, a.layer, r, 13);
}

BFP_STAMP_READER(bfp200_stamps_layer1)

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// Fills the role-dependent fields of `a` (O groups, staged K/V positions);
// false when the configuration does not fit this kernel.  smem_budget: the
// dynamic shared memory a CTA may use.
bool attn_block_plan(L1Args& a, int smem_budget) {
  const int D = a.D, NT = D / 16, NU = a.HQ + 2 * a.HKV;
  if (D % 64 || a.HQ * 64 != D || a.HKV <= 0 || a.HQ % a.HKV || NU > 16 || NT > 8 * 5) return false;
  int ca = 0, co = 0;
  for (int r = 0; r < NU; ++r) {
    int s0, c;
    l1_o_groups(r, a.HQ, NU, NT, &s0, &c);
    if (r < a.HQ) ca = c > ca ? c : ca;
    else co = c > co ? c : co;
  }
  const int maxc = a.kv.MAX_CTX;
  if (l1_layout(D, co, false, maxc, 0).total > smem_budget) return false;
  int ch = maxc;
  while (ch > 0 && l1_layout(D, ca, true, maxc, ch).total > smem_budget) --ch;
  if (ch < maxc && ch < 64) return false;
  a.og_other = co;
  a.og_att = ca;
  a.ch = ch;
  return true;
}

size_t attn_block_smem(const L1Args& a) {
  const int m1 = l1_layout(a.D, a.og_other, false, a.kv.MAX_CTX, a.ch).total;
  const int m2 = l1_layout(a.D, a.og_att, true, a.kv.MAX_CTX, a.ch).total;
  return (size_t)(m1 > m2 ? m1 : m2);
}

cudaError_t launch_attn_block(const L1Args& a, cudaStream_t s, bool pdl) {
  const int NU = a.HQ + 2 * a.HKV;
  const int NT = a.D / 16;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(NU);
  cfg.blockDim = dim3(A_THREADS);
  cfg.dynamicSmemBytes = attn_block_smem(a);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = NU;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  switch ((NT + 7) / 8) {
    case 1: return cudaLaunchKernelEx(&cfg, bfp_attn_block_kernel<1>, a);
    case 2: return cudaLaunchKernelEx(&cfg, bfp_attn_block_kernel<2>, a);
    case 3: return cudaLaunchKernelEx(&cfg, bfp_attn_block_kernel<3>, a);
    case 4: return cudaLaunchKernelEx(&cfg, bfp_attn_block_kernel<4>, a);
    case 5: return cudaLaunchKernelEx(&cfg, bfp_attn_block_kernel<5>, a);
    default: return cudaErrorInvalidValue;
  }
}

// Raises the kernel's dynamic shared memory limit (the opt-in limit minus
// its static shared memory, returned in *dyn_budget) and allows its
// non-portable cluster size.
cudaError_t init_attn_block_attributes(int smem_optin, int* dyn_budget) {
  cudaError_t e = cudaSuccess;
  int budget = smem_optin;
  auto set = [&](const void* f) {
    cudaFuncAttributes fa;
    cudaError_t r = cudaFuncGetAttributes(&fa, f);
    const int dyn = smem_optin - (int)fa.sharedSizeBytes;
    budget = dyn < budget ? dyn : budget;
    if (r == cudaSuccess) r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (r == cudaSuccess) r = cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (r != cudaSuccess) e = r;
  };
  set((const void*)bfp_attn_block_kernel<1>);
  set((const void*)bfp_attn_block_kernel<2>);
  set((const void*)bfp_attn_block_kernel<3>);
  set((const void*)bfp_attn_block_kernel<4>);
  set((const void*)bfp_attn_block_kernel<5>);
  if (dyn_budget) *dyn_budget = budget;
  return e;
}

}  // namespace bfp
