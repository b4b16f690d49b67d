// gemv.cu -- small-batch (1..4 columns) BFP matvec family of the bs1 decode.
//
// Same arithmetic as bfp_matmul_kernel (matvec_hw_golden, gen_smollm_blockfp_full.py
// :217-233), arranged for latency instead of throughput:
//   * one CTA per 16-row group (two groups for the gate/up pair), full K;
//   * every weight tile a thread needs is loaded into registers BEFORE the
//     programmatic-launch wait, so weight streaming overlaps the previous
//     kernel entirely;
//   * optional RMSNorm prologue on the input columns (rmsnorm_fp +
//     tile_quantize, :263-264 / :286-287), computed by every CTA, so no
//     separate normalisation kernel sits between two matvecs;
//   * fused epilogues: store, residual (:285, :293), SwiGLU (:290-291), and
//     RoPE + KV write (:268-272) for the fused Q/K/V matrix, where the four
//     CTAs of one head form a thread-block cluster and exchange the rotated
//     halves through distributed shared memory.
#include "bfp_device.cuh"
#include "kernels.cuh"
#include "stamps.cuh"

#include <cooperative_groups.h>

namespace bfp {

__device__ __forceinline__ void gv_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void gv_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ int gv_dp2a_lo_ss(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int gv_dp2a_hi_ss(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int gv_dp2a_lo_su(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}
__device__ __forceinline__ int gv_dp2a_hi_su(unsigned a, unsigned b, int c) {
  int d; asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c)); return d;
}

// exact 16-term tile sum x . w with w given as hi / lo byte planes
__device__ __forceinline__ long long gv_tile_sum(const uint4 x0, const uint4 x1, const uint4 wh, const uint4 wl) {
  int A = 0, B = 0;
  A = gv_dp2a_lo_ss(x0.x, wh.x, A); A = gv_dp2a_hi_ss(x0.y, wh.x, A);
  A = gv_dp2a_lo_ss(x0.z, wh.y, A); A = gv_dp2a_hi_ss(x0.w, wh.y, A);
  A = gv_dp2a_lo_ss(x1.x, wh.z, A); A = gv_dp2a_hi_ss(x1.y, wh.z, A);
  A = gv_dp2a_lo_ss(x1.z, wh.w, A); A = gv_dp2a_hi_ss(x1.w, wh.w, A);
  B = gv_dp2a_lo_su(x0.x, wl.x, B); B = gv_dp2a_hi_su(x0.y, wl.x, B);
  B = gv_dp2a_lo_su(x0.z, wl.y, B); B = gv_dp2a_hi_su(x0.w, wl.y, B);
  B = gv_dp2a_lo_su(x1.x, wl.z, B); B = gv_dp2a_hi_su(x1.y, wl.z, B);
  B = gv_dp2a_lo_su(x1.z, wl.w, B); B = gv_dp2a_hi_su(x1.w, wl.w, B);
  return ((long long)A << 8) + (long long)B;
}

constexpr int GV_THREADS = 256;
constexpr int GV_MAX_NT = 96;     // K <= 1536

struct GvSmem {
  size_t we, gam, xs, sq, nm, ne, ms, red, vals, r, total;
};

__host__ __device__ inline GvSmem gv_layout(int RG, int NC, int K, bool norm) {
  GvSmem L;
  size_t off = 0;
  auto take = [&](size_t b) { size_t o = off; off = (off + b + 15) & ~size_t(15); return o; };
  const int NT = K / 16;
  L.we = take((size_t)RG * NT * 16);
  L.gam = take(norm ? (size_t)K * 8 : 0);
  L.xs = take(norm ? (size_t)NC * K * 8 : 0);
  L.sq = take(norm ? (size_t)NC * K * 8 : 0);
  L.nm = take((size_t)NC * K * 2);
  L.ne = take((size_t)NC * NT);
  L.ms = take((size_t)16 * RG * NC * 4);
  L.red = take((size_t)(GV_THREADS / 32) * 16 * RG * NC * 8);
  L.vals = take((size_t)NC * 16 * 8);
  L.r = take((size_t)NC * 8);
  L.total = off;
  return L;
}

size_t gemv_smem_bytes(int rg, int nc, int K, bool norm) { return gv_layout(rg, nc, K, norm).total; }

// MAXU: K tiles per thread (NT <= MAXU * threads-per-row)
template <int NC, int RG, int MODE, bool NORM, int MAXU>
__global__ void __launch_bounds__(GV_THREADS)
bfp_gemv_small_kernel(GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int ROWS = 16 * RG;
  constexpr int TPR = GV_THREADS / ROWS;                 // threads per row
  const int NT = a.W.NT, K = NT * 16;
  const int g0 = blockIdx.x * RG;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = tid % ROWS, tl = tid / ROWS;
  const int gi = row >> 4, ri = row & 15;
  const GvSmem L = gv_layout(RG, NC, K, NORM);
  int8_t* WeS = reinterpret_cast<int8_t*>(smem + L.we);
  double* gs = reinterpret_cast<double*>(smem + L.gam);
  double* xs = reinterpret_cast<double*>(smem + L.xs);
  double* sq = reinterpret_cast<double*>(smem + L.sq);
  int16_t* nm = reinterpret_cast<int16_t*>(smem + L.nm);
  int8_t* ne = reinterpret_cast<int8_t*>(smem + L.ne);
  int* Ms = reinterpret_cast<int*>(smem + L.ms);
  long long* red = reinterpret_cast<long long*>(smem + L.red);
  double* vals = reinterpret_cast<double*>(smem + L.vals);
  double* rs = reinterpret_cast<double*>(smem + L.r);
  __shared__ int s_lo[96], s_len[96];
  __shared__ double s_val[96];

  constexpr int SK = MODE == GV_SWIGLU ? 1 : (MODE == GV_RESIDUAL ? 2 : 3);
  BFP_STAMP(SK, a.layer, blockIdx.x, 0);
  gv_pdl_trigger();
  // ---- weights: registers and shared memory, before the dependency wait
  uint4 wh[MAXU], wl[MAXU];
  #pragma unroll
  for (int j = 0; j < MAXU; ++j) {
    const int t = tl + j * TPR;
    if (t < NT) {
      const uint4* wp = reinterpret_cast<const uint4*>(a.W.wm + ((size_t)(g0 + gi) * NT + t) * 512);
      wh[j] = wp[ri];
      wl[j] = wp[16 + ri];
    }
  }
  for (int i = tid; i < RG * NT; i += GV_THREADS)
    reinterpret_cast<uint4*>(WeS)[i] = reinterpret_cast<const uint4*>(a.W.we + (size_t)g0 * NT * 16)[i];
  if constexpr (NORM)
    for (int i = tid; i < K; i += GV_THREADS) gs[i] = a.gamma[i];
  for (int i = tid; i < ROWS * NC; i += GV_THREADS) Ms[i] = -100000;

  gv_pdl_wait();
  BFP_STAMP(SK, a.layer, blockIdx.x, 1);
  // ---- input columns (optionally RMS-normalised) into shared memory
  if constexpr (NORM) {
    constexpr int PER = 4;            // loads in flight per thread per round
    for (int base = 0; base < NC * K; base += GV_THREADS * PER) {
      int16_t mv[PER];
      int8_t ev[PER];
      #pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int i = base + tid + q * GV_THREADS;
        const int c = i / K, k = i % K;
        mv[q] = 0; ev[q] = 0;
        if (i < NC * K && c < a.ncols) { mv[q] = a.xm[(size_t)c * a.x_ld + k]; ev[q] = a.xe[(size_t)c * a.x_lde + k / 16]; }
      }
      #pragma unroll
      for (int q = 0; q < PER; ++q) {
        const int i = base + tid + q * GV_THREADS;
        if (i < NC * K) {
          const double x = bfp_decode(mv[q], ev[q]);
          xs[i] = x;
          sq[i] = __dmul_rn(x, x);
        }
      }
    }
    __syncthreads();
    if (warp < NC) {   // column `warp`: r = sqrt(mean(x*x) + eps)   (:237)
      const double sum = np_sum_warp(sq + (size_t)warp * K, K, s_lo, s_len, s_val);
      if (lane == 0) rs[warp] = __dsqrt_rn(__dadd_rn(__ddiv_rn(sum, (double)K), a.eps));
    }
    __syncthreads();
    constexpr int QN = 3;             // tiles quantized together per lane (overlapping latencies)
    for (int base = 0; base < NC * K; base += GV_THREADS * QN) {
      double y[QN];
      bool valid[QN];
      #pragma unroll
      for (int q = 0; q < QN; ++q) {                         // tiles never straddle columns (K % 16 == 0)
        const int i = base + tid + q * GV_THREADS;
        valid[q] = i < NC * K;
        const int c = valid[q] ? i / K : 0, k = valid[q] ? i % K : 0;
        y[q] = valid[q] ? __ddiv_rn(__dmul_rn(xs[i], gs[k]), rs[c]) : 0.0;
      }
      int16_t m[QN];
      int e[QN];
      tile_quantize_requant_16lanes_n<QN>(y, valid, m, e);   // tile_quantize(fpq(y)) (:238, :264)
      #pragma unroll
      for (int q = 0; q < QN; ++q) {
        const int i = base + tid + q * GV_THREADS;
        if (valid[q]) {
          const int c = i / K, k = i % K;
          nm[i] = m[q];
          if ((k & 15) == 0) ne[c * NT + k / 16] = (int8_t)e[q];
          if (a.dbg_in && blockIdx.x == 0 && c < a.ncols) a.dbg_in[(size_t)c * a.dbg_ld + k] = bfp_decode(m[q], e[q]);
        }
      }
    }
  } else {
    for (int i = tid; i < NC * K / 8; i += GV_THREADS) {
      const int c = i / (K / 8), k8 = i % (K / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (c < a.ncols) v = reinterpret_cast<const uint4*>(a.xm + (size_t)c * a.x_ld)[k8];
      reinterpret_cast<uint4*>(nm)[i] = v;
    }
    for (int i = tid; i < NC * NT; i += GV_THREADS) {
      const int c = i / NT, t = i % NT;
      ne[i] = (c < a.ncols) ? a.xe[(size_t)c * a.x_lde + t] : (int8_t)-127;
    }
  }
  __syncthreads();
  BFP_STAMP(SK, a.layer, blockIdx.x, 2);
  // ---- max tile exponent per (row, column) over the full K (:221-222)
  #pragma unroll
  for (int c = 0; c < NC; ++c) {
    int m = -100000;
    for (int t = tl; t < NT; t += TPR) {
      const int e = (int)ne[c * NT + t] + (int)WeS[(gi * NT + t) * 16 + ri];
      m = e > m ? e : m;
    }
    atomicMax(&Ms[row * NC + c], m);
  }
  __syncthreads();
  BFP_STAMP(SK, a.layer, blockIdx.x, 3);
  // ---- tile sums, per-tile floor shift, int64 accumulation (:219-228)
  long long acc[NC];
  int Mr[NC];
  #pragma unroll
  for (int c = 0; c < NC; ++c) { acc[c] = 0; Mr[c] = Ms[row * NC + c]; }
  #pragma unroll
  for (int j = 0; j < MAXU; ++j) {
    const int t = tl + j * TPR;
    if (t < NT) {
      const int we = (int)WeS[(gi * NT + t) * 16 + ri];
      #pragma unroll
      for (int c = 0; c < NC; ++c) {
        const uint4* xp = reinterpret_cast<const uint4*>(nm + (size_t)c * K + t * 16);
        const long long S = gv_tile_sum(xp[0], xp[1], wh[j], wl[j]);
        const int sh = Mr[c] - (int)ne[c * NT + t] - we;
        acc[c] += (sh > ALIGN_MAX) ? 0LL : (S >> sh);
      }
    }
  }
  // reduce the TPR partials of each row: lanes r and r+16 of a warp (RG = 1),
  // then across warps
  #pragma unroll
  for (int c = 0; c < NC; ++c) {
    long long v = acc[c];
    if (ROWS == 16) v += __shfl_xor_sync(0xffffffffu, v, 16);
    acc[c] = v;
  }
  if (ROWS == 32 || lane < 16) {
    #pragma unroll
    for (int c = 0; c < NC; ++c) red[((size_t)warp * ROWS + row) * NC + c] = acc[c];
  }
  __syncthreads();
  BFP_STAMP(SK, a.layer, blockIdx.x, 4);

  // ---- epilogue: 16 lanes per (row group, column) pair
  constexpr int NPAIR = (MODE == GV_SWIGLU ? 1 : RG) * NC;
  const int p = tid >> 4;                  // pair index (warps 0..NPAIR/2)
  const int l16 = tid & 15;
  if (p >= ((NPAIR + 1) & ~1)) {
    if constexpr (MODE == GV_QKV_ROPE) {   // every thread takes part in the cluster barriers
      namespace cg = cooperative_groups;
      cg::this_cluster().sync();
      cg::this_cluster().sync();
    }
    return;
  }
  const bool valid = p < NPAIR && (p % NC) < a.ncols;
  auto total = [&](int r, int c) -> double {      // clip, scale: exact (:229-232)
    long long s = 0;
    #pragma unroll
    for (int w = 0; w < GV_THREADS / 32; ++w) s += red[((size_t)w * ROWS + r) * NC + c];
    s = s > SAT_HI ? SAT_HI : (s < SAT_LO ? SAT_LO : s);
    return (double)s * pow2(Ms[r * NC + c] - 30);
  };
  if constexpr (MODE == GV_STORE || MODE == GV_RESIDUAL) {
    const int c = p % NC, go = p / NC;
    const int r = go * 16 + l16;
    const double out_real = valid ? total(r, c) : 0.0;
    int qe;
    int16_t qm = tile_quantize_16lanes(out_real, &qe);               // :233
    const size_t orow = (size_t)(g0 + go) * 16 + l16;
    if (a.dbg_mid && valid) a.dbg_mid[(size_t)c * a.dbg_ld + orow] = bfp_decode(qm, qe);
    if constexpr (MODE == GV_RESIDUAL) {
      const double hv = valid ? bfp_decode(a.rm[(size_t)c * a.o_ld + orow], a.re[(size_t)c * a.o_lde + g0 + go]) : 0.0;
      const double y = __dadd_rn(hv, bfp_decode(qm, qe));            // fpq(h + o)
      qm = tile_quantize_16lanes(y, &qe);
    }
    if (valid) {
      a.om[(size_t)c * a.o_ld + orow] = qm;
      if (l16 == 0) a.oe[(size_t)c * a.o_lde + g0 + go] = (int8_t)qe;
    }
  } else if constexpr (MODE == GV_SWIGLU) {
    const int c = p;
    const double gu_r[2] = {valid ? total(l16, c) : 0.0, valid ? total(16 + l16, c) : 0.0};
    int16_t gu_m[2];
    int gu_e[2], se, pe;
    tile_quantize_16lanes_n<2>(gu_r, gu_m, gu_e);                    // g, u = matvec (:288-289)
    if (a.dbg_mid && valid) {
      a.dbg_mid[(size_t)c * a.dbg_ld + (size_t)g0 / 2 * 16 + l16] = bfp_decode(gu_m[0], gu_e[0]);
      a.dbg_mid2[(size_t)c * a.dbg_ld + (size_t)g0 / 2 * 16 + l16] = bfp_decode(gu_m[1], gu_e[1]);
    }
    const double gv = bfp_decode(gu_m[0], gu_e[0]), uv = bfp_decode(gu_m[1], gu_e[1]);
    const double sv = __ddiv_rn(gv, __dadd_rn(1.0, exp(-gv)));       // silu_fp (:241-242)
    const int16_t sm = tile_quantize_16lanes(sv, &se);
    const double prod = __dmul_rn(bfp_decode(sm, se), uv);           // fpq(silu * u) (:290)
    int16_t pm = tile_quantize_16lanes(prod, &pe);
    const unsigned bal = __ballot_sync(0xffffffffu, pm == (int16_t)-32768);
    const bool has_min = ((bal >> (lane & 16)) & 0xFFFFu) != 0;
    pm = requant_mant(pm, has_min && pe < 127);                      // tile_quantize(mlp) (:291)
    pe = requant_exp(pe, has_min);
    if (valid) {
      const size_t og = (size_t)g0 / 2;
      a.om[(size_t)c * a.o_ld + og * 16 + l16] = pm;
      if (l16 == 0) a.oe[(size_t)c * a.o_lde + og] = (int8_t)pe;
    }
  } else {   // GV_QKV_ROPE: 4 CTAs (the 4 row groups of one head) per cluster
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const int c = p;
    const int unit = blockIdx.x >> 2, rank = blockIdx.x & 3;
    const double out_real = valid ? total(l16, c) : 0.0;
    int qe;
    const int16_t qm = tile_quantize_16lanes(out_real, &qe);          // q/k/v = matvec (:265-267)
    const double own = bfp_decode(qm, qe);
    if (p < NC) vals[c * 16 + l16] = own;
    cl.sync();
    const double partner = (p < NC) ? cl.map_shared_rank(vals, rank ^ 2)[c * 16 + l16] : 0.0;
    const int HQ = a.HQ, HKV = a.HKV;
    const int slot = valid ? a.col_slot[c] : 0, pos = valid ? a.col_pos[c] : 0;
    const int d = rank * 16 + l16;
    if (unit < HQ + HKV) {
      // rope_fp (:250-258): out[j] = a*c - b*s, out[j+32] = b*c + a*s, then fpq
      const int jj = d < 32 ? d : d - 32;
      const double cs = valid ? a.rope_cs[((size_t)pos * 32 + jj) * 2 + 0] : 0.0;
      const double sn = valid ? a.rope_cs[((size_t)pos * 32 + jj) * 2 + 1] : 0.0;
      const double av = d < 32 ? own : partner, bv = d < 32 ? partner : own;
      const double y = d < 32 ? __dsub_rn(__dmul_rn(av, cs), __dmul_rn(bv, sn))
                              : __dadd_rn(__dmul_rn(bv, cs), __dmul_rn(av, sn));
      int re;
      const int16_t rm = tile_quantize_16lanes(y, &re);
      if (a.dbg_mid && valid) a.dbg_mid[(size_t)c * a.dbg_ld + unit * 64 + d] = bfp_decode(rm, re);
      if (valid) {
        if (unit < HQ) {
          a.qr_m[(size_t)c * HQ * 64 + unit * 64 + d] = rm;
          if (l16 == 0) a.qr_e[(size_t)c * HQ * 4 + unit * 4 + rank] = (int8_t)re;
        } else {
          const size_t base = (((size_t)slot * a.kv.NL + a.layer) * HKV + (unit - HQ)) * a.kv.MAX_CTX + pos;
          a.kv.km[base * 64 + d] = rm;
          if (l16 == 0) a.kv.ke[base * 4 + rank] = (int8_t)re;
        }
      }
    } else if (valid) {   // v heads: stored as produced (:272)
      if (a.dbg_mid) a.dbg_mid[(size_t)c * a.dbg_ld + unit * 64 + d] = bfp_decode(qm, qe);
      const size_t base = (((size_t)slot * a.kv.NL + a.layer) * HKV + (unit - HQ - HKV)) * a.kv.MAX_CTX + pos;
      a.kv.vm[base * 64 + d] = qm;
      if (l16 == 0) a.kv.ve[base * 4 + rank] = (int8_t)qe;
    }
    cl.sync();                               // partners stay resident until the exchange is done
  }
}

template <int NC, int RG, int MODE, bool NORM, int MAXU>
static cudaError_t launch_gemv_t(const GemvArgs& a, cudaStream_t s, bool pdl) {
  const size_t smem = gv_layout(RG, NC, a.W.NT * 16, NORM).total;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.W.G / RG);
  cfg.blockDim = dim3(GV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (MODE == GV_QKV_ROPE) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 4;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, bfp_gemv_small_kernel<NC, RG, MODE, NORM, MAXU>, a);
}

// instantiation table: (NC, RG, MODE, NORM, MAXU)
#define GV_FOR_EACH(X)                                                                   \
  X(1, 1, GV_STORE, false, 6) X(4, 1, GV_STORE, false, 6)                                \
  X(1, 1, GV_RESIDUAL, false, 3) X(4, 1, GV_RESIDUAL, false, 3)                          \
  X(1, 1, GV_RESIDUAL, false, 6) X(4, 1, GV_RESIDUAL, false, 6)                          \
  X(1, 2, GV_SWIGLU, true, 5) X(4, 2, GV_SWIGLU, true, 5)                                \
  X(1, 1, GV_QKV_ROPE, true, 3) X(4, 1, GV_QKV_ROPE, true, 3)

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t s, bool pdl) {
  if (a.ncols < 1 || a.ncols > 4 || a.W.NT > GV_MAX_NT) return cudaErrorInvalidValue;
  const int NC = a.ncols == 1 ? 1 : 4;
  const int RG = a.mode == GV_SWIGLU ? 2 : 1;
  const int tpr = GV_THREADS / (16 * RG);
  const int need = (a.W.NT + tpr - 1) / tpr;
  int maxu = -1;
  const bool norm = a.norm != 0;
#define GV_PICK(nc, rg, md, nrm, mu)                                                      \
  if (maxu < 0 && NC == nc && RG == rg && a.mode == md && norm == nrm && need <= mu) {   \
    maxu = mu;                                                                           \
    return launch_gemv_t<nc, rg, md, nrm, mu>(a, s, pdl);                                \
  }
  GV_FOR_EACH(GV_PICK)
#undef GV_PICK
  return cudaErrorInvalidValue;
}

bool gemv_supported(int mode, bool norm, int NT, int ncols) {
  if (ncols < 1 || ncols > 4) return false;
  const int RG = mode == GV_SWIGLU ? 2 : 1;
  const int tpr = GV_THREADS / (16 * RG);
  const int need = (NT + tpr - 1) / tpr;
  bool ok = false;
#define GV_CHECK(nc, rg, md, nrm, mu) ok = ok || (rg == RG && md == mode && nrm == norm && need <= mu);
  GV_FOR_EACH(GV_CHECK)
#undef GV_CHECK
  return ok;
}

cudaError_t init_gemv_attributes() {
  int dev = 0, optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return e;
#define GV_ATTR(nc, rg, md, nrm, mu)                                                        \
  {                                                                                         \
    const void* f = (const void*)bfp_gemv_small_kernel<nc, rg, md, nrm, mu>;                          \
    cudaFuncAttributes fa;                                                                  \
    cudaError_t r = cudaFuncGetAttributes(&fa, f);                                          \
    if (r == cudaSuccess)                                                                   \
      r = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes); \
    if (r != cudaSuccess) e = r;                                                            \
  }
  GV_FOR_EACH(GV_ATTR)
#undef GV_ATTR
  return e;
}

BFP_STAMP_READER(bfp200_stamps_gemv)

}  // namespace bfp
