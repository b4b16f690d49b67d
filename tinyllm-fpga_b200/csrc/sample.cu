// sample.cu -- temperature / top-k sampling of the next token, the non-greedy
// head of the reference's hardware emulator (sim_rtl_fp_hw.py:204-216):
//
//   scaled = logits / T
//   if TOPK > 0: keep scaled[argsort(scaled)[-TOPK:]], the rest -inf
//   scaled -= scaled.max();  p = exp(scaled);  p = p / p.sum()
//   nid = np.random.choice(len(p), p=p)
//
// np.random.choice (legacy RandomState) draws u = random_sample() and
// returns searchsorted(cdf / cdf[-1], u, side='right') with cdf = cumsum(p),
// a sequential sum; p.sum() is numpy's pairwise sum.  The uniforms are
// generated on the host (MT19937 seeded like np.random.seed, 53-bit
// random_sample), one per sampled step, and read on the device by step.
//
// One CTA per sequence.  Top-k keeps the k largest scaled logits (radix
// select on order-preserving 64-bit keys); among values equal to the k-th
// largest the lowest indices are kept (numpy's unstable argsort leaves that
// order unspecified).  The logits come from the fp64 head, whose summation
// order differs from BLAS by a bounded amount; a draw is certified when u is
// farther than that bound's effect from the neighbouring cdf values (and, with
// top-k, the kept set is separated from the rest by more than the bound).
#include "bfp_device.cuh"
#include "kernels.cuh"

#include <cstdint>

namespace bfp {

namespace {

constexpr int SM_THREADS = 1024;
constexpr int SM_WARPS = SM_THREADS / 32;

__device__ __forceinline__ unsigned long long order_key(double x) {
  const unsigned long long b = (unsigned long long)__double_as_longlong(x);
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

// block-wide exclusive scan of one int per thread; returns the prefix and
// sets *total
__device__ int block_exclusive_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
  #pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < SM_WARPS ? s_warp[lane] : 0;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < SM_WARPS) s_warp[lane] = w;        // inclusive warp prefix
  }
  __syncthreads();
  const int before = (warp ? s_warp[warp - 1] : 0) + x - v;
  *total = s_warp[SM_WARPS - 1];
  __syncthreads();
  return before;
}

__device__ double block_max(double v, double* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  double m = s_red[0];
  for (int w = 1; w < SM_WARPS; ++w) m = fmax(m, s_red[w]);
  __syncthreads();
  return m;
}

__device__ int block_min_int(int v, int* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  int m = s_red[0];
  for (int w = 1; w < SM_WARPS; ++w) m = min(m, s_red[w]);
  __syncthreads();
  return m;
}

// numpy's pairwise sum of a[0..n) (global memory) from the host-built plan of
// its tree (same plan format as the attention sums): leaves by separate
// threads, then one level of internal nodes at a time.  sval: 2L-1 doubles
// of shared memory.
__device__ double block_np_sum_plan(const double* a, int n, const unsigned short* plan, double* sval) {
  const int L = plan[0], H = plan[1];
  const unsigned short* starts = plan + 2;
  const unsigned short* lvl = starts + L;
  const unsigned short* ops = lvl + H;
  for (int k = threadIdx.x; k < L; k += SM_THREADS) {
    const int s0 = starts[k], e0 = (k + 1 < L) ? starts[k + 1] : n;
    sval[k] = np_pw_leaf(a + s0, e0 - s0);
  }
  __syncthreads();
  int base = 0;
  for (int hgt = 0; hgt < H; ++hgt) {
    const int cnt = lvl[hgt];
    for (int j = threadIdx.x; j < cnt; j += SM_THREADS) {
      const int o = base + j;
      sval[L + o] = __dadd_rn(sval[ops[2 * o]], sval[ops[2 * o + 1]]);
    }
    base += cnt;
    __syncthreads();
  }
  const double r = H ? sval[L + base - 1] : sval[0];
  __syncthreads();
  return __dadd_rn(0.0, r);
}

__global__ void __launch_bounds__(SM_THREADS)
sample_kernel(SampleArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  double* sval = reinterpret_cast<double*>(smem);                 // [2 L]
  __shared__ int s_hist[256];
  __shared__ int s_wi[SM_WARPS];
  __shared__ double s_wd[SM_WARPS];
  __shared__ unsigned long long s_prefix;
  __shared__ int s_krem;
  const int c = blockIdx.x, tid = threadIdx.x;
  const int V = a.V;
  const double* lg = a.logits + (size_t)c * a.ld;
  double* p = a.work + (size_t)c * a.ld;
  int* incl = a.incl + (size_t)c * a.ld;
  double* cdf = a.cdf + (size_t)c * a.ld;
  const int CH = (V + SM_THREADS - 1) / SM_THREADS;               // contiguous chunk per thread
  const int i0 = min(V, tid * CH), i1 = min(V, i0 + CH);
  // scaled = logits / T   (:207)
  for (int i = tid; i < V; i += SM_THREADS) p[i] = __ddiv_rn(lg[i], a.temperature);
  __syncthreads();
  const bool topk = a.top_k > 0 && a.top_k < V;
  // ---- top-k: the k-th largest key by radix select, 8 bits per pass
  unsigned long long thr = 0;
  int need_eq = 0;
  if (topk) {
    if (tid == 0) { s_prefix = 0; s_krem = a.top_k; }
    for (int pass = 0; pass < 8; ++pass) {
      const int sh = 56 - 8 * pass;
      for (int b = tid; b < 256; b += SM_THREADS) s_hist[b] = 0;
      __syncthreads();
      const unsigned long long pre = s_prefix;
      const unsigned long long hmask = pass ? (~0ull << (sh + 8)) : 0ull;
      for (int i = tid; i < V; i += SM_THREADS) {
        const unsigned long long k = order_key(p[i]);
        if ((k & hmask) == pre) atomicAdd(&s_hist[(k >> sh) & 255], 1);
      }
      __syncthreads();
      if (tid == 0) {
        int rem = s_krem, d = 255;
        for (; d > 0; --d) {
          if (s_hist[d] >= rem) break;
          rem -= s_hist[d];
        }
        s_krem = rem;
        s_prefix = pre | ((unsigned long long)d << sh);
      }
      __syncthreads();
    }
    thr = s_prefix;
    need_eq = s_krem;                 // how many of the values equal to the threshold are kept
  }
  // ---- kept set (ascending index order), its maximum, and
  // p = exp(scaled - max) on it, 0 elsewhere   (:208-213)
  int n_keep = V;
  double mx = -INFINITY, out_max = -INFINITY, kth = -INFINITY;
  if (topk) {
    int neq = 0;
    for (int i = i0; i < i1; ++i) neq += order_key(p[i]) == thr;
    int tot;
    const int eq_before = block_exclusive_scan(neq, s_wi, &tot);
    int e = eq_before, nk = 0;
    for (int i = i0; i < i1; ++i) {
      const unsigned long long k = order_key(p[i]);
      nk += k > thr || (k == thr && e < need_eq);
      e += k == thr;
    }
    const int keep_before = block_exclusive_scan(nk, s_wi, &n_keep);
    e = eq_before;
    int q = keep_before;
    double lm = -INFINITY, lout = -INFINITY;
    for (int i = i0; i < i1; ++i) {
      const double x = p[i];
      const unsigned long long k = order_key(x);
      const bool keep = k > thr || (k == thr && e < need_eq);
      e += k == thr;
      if (keep) { incl[q++] = i; lm = fmax(lm, x); }
      else lout = fmax(lout, x);
    }
    mx = block_max(lm, s_wd);
    out_max = block_max(lout, s_wd);
    e = eq_before;
    for (int i = i0; i < i1; ++i) {
      const double x = p[i];
      const unsigned long long k = order_key(x);
      const bool keep = k > thr || (k == thr && e < need_eq);
      e += k == thr;
      p[i] = keep ? exp(__dsub_rn(x, mx)) : 0.0;
    }
    const unsigned long long kb = (thr >> 63) ? (thr & 0x7fffffffffffffffull) : ~thr;
    kth = __longlong_as_double((long long)kb);     // the k-th largest scaled value
  } else {
    double lm = -INFINITY;
    for (int i = tid; i < V; i += SM_THREADS) lm = fmax(lm, p[i]);
    mx = block_max(lm, s_wd);
    for (int i = tid; i < V; i += SM_THREADS) p[i] = exp(__dsub_rn(p[i], mx));
  }
  __syncthreads();
  // p = p / p.sum()   (pairwise sum, :213)
  const double total = block_np_sum_plan(p, V, a.plan, sval);
  for (int i = tid; i < V; i += SM_THREADS) p[i] = __ddiv_rn(p[i], total);
  __syncthreads();
  // cdf = cumsum(p) (sequential); entries outside the kept set add 0.0 and
  // leave the running sum unchanged, so only kept entries are visited
  if (tid == 0) {
    double s = 0.0;
    if (topk) {
      for (int j = 0; j < n_keep; ++j) { s = __dadd_rn(s, p[incl[j]]); cdf[j] = s; }
    } else {
      int i = 0;
      for (; i + 4 <= V; i += 4) {
        const double x0 = p[i], x1 = p[i + 1], x2 = p[i + 2], x3 = p[i + 3];
        s = __dadd_rn(s, x0); cdf[i] = s;
        s = __dadd_rn(s, x1); cdf[i + 1] = s;
        s = __dadd_rn(s, x2); cdf[i + 2] = s;
        s = __dadd_rn(s, x3); cdf[i + 3] = s;
      }
      for (; i < V; ++i) { s = __dadd_rn(s, p[i]); cdf[i] = s; }
    }
    sval[0] = s;
  }
  __syncthreads();
  const double last = sval[0];
  const int nq = topk ? n_keep : V;
  const int step = *a.step;
  const double u = a.uniforms[(size_t)c * a.u_ld + step + 1];
  // first kept position whose cdf / cdf[-1] exceeds u (searchsorted, side='right')
  int first = nq;
  for (int q = tid; q < nq; q += SM_THREADS)
    if (__ddiv_rn(cdf[q], last) > u) { first = q; break; }
  first = block_min_int(first, s_wi);
  if (tid == 0) {
    const int qq = first < nq ? first : nq - 1;
    const int tok = topk ? incl[qq] : qq;
    // certificate: logits may differ from BLAS by 2 gamma ||hn|| max||e_v||,
    // scaled ones by that / T; p, the sums and the cdf move by at most a few
    // times that (plus rounding, bounded by 1e-10 here)
    const double uu = 1.1102230246251565e-16;
    const double gam = (a.D + 2) * uu / (1.0 - (a.D + 2) * uu);
    const double dl = 2.0 * gam * a.hn_norm[c] * a.emb_norm_max / a.temperature;
    const double m = 8.0 * dl + 1e-10;
    const double hi = __ddiv_rn(cdf[qq], last);
    const double lo = qq > 0 ? __ddiv_rn(cdf[qq - 1], last) : 0.0;
    bool ok = first < nq && (hi - u) > m && (qq == 0 || (u - lo) > m);
    if (topk && out_max > -INFINITY) ok = ok && (kth - out_max) > 2.0 * dl;   // kept set vs the largest dropped
    a.tok[c] = tok;
    a.cert[c] = ok ? 1 : 0;
  }
}

}  // namespace

cudaError_t launch_sample(const SampleArgs& a, int ncols, int plan_leaves, cudaStream_t s) {
  const size_t smem = (size_t)(2 * plan_leaves + 2) * sizeof(double);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  sample_kernel<<<ncols, SM_THREADS, smem, s>>>(a);
  return cudaGetLastError();
}

// numpy's legacy global generator: np.random.seed(seed) = MT19937
// init_genrand(seed); random_sample() = (a >> 5, b >> 6) of two 32-bit draws
// as a 53-bit fraction (Matsumoto & Nishimura's genrand_res53).
void mt19937_uniforms(uint32_t seed, int n, double* out) {
  constexpr int N = 624, M = 397;
  uint32_t mt[N];
  mt[0] = seed;
  for (int i = 1; i < N; ++i) mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
  int idx = N;
  auto next = [&]() -> uint32_t {
    if (idx >= N) {
      for (int k = 0; k < N; ++k) {
        const uint32_t y = (mt[k] & 0x80000000u) | (mt[(k + 1) % N] & 0x7fffffffu);
        mt[k] = mt[(k + M) % N] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
      }
      idx = 0;
    }
    uint32_t y = mt[idx++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
  };
  for (int i = 0; i < n; ++i) {
    const uint32_t a = next() >> 5, b = next() >> 6;
    out[i] = ((double)a * 67108864.0 + (double)b) / 9007199254740992.0;
  }
}

}  // namespace bfp
