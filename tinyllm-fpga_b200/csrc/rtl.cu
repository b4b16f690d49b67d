// rtl.cu -- the FPGA's fixed-point leaf ops ("rtl-exact" mode), batched.
//
// The reference pins each RTL module with a per-op golden generator
// (rtl/vc707/host/gen_*_bfp_golden.py); these kernels compute the same
// integers:
//   matvec    running-alignment 48-bit matvec, one exponent per output
//             element (gen_matvec_bfp_golden.py:49-104, matvec_bfp_engine.sv)
//   rmsnorm   sum of squares, Q0.32 1/D, Newton-Raphson 1/sqrt from a seed
//             table (gen_rmsnorm_bfp_golden.py:43-144, rmsnorm_bfp.sv)
//   rope      Q0.31 turn table, CORDIC sin/cos, per-element output exponent
//             (gen_rope_bfp_golden.py:25-124, rope_bfp.sv)
//   softmax   exp ROM, Newton-Raphson 1/sum, one shared exponent
//             (gen_softmax_bfp_golden.py:34-83, softmax_bfp.sv)
//   swiglu    SiLU ROM at 2^5 scale, per-tile output
//             (gen_swiglu_bfp_golden.py:45-77, swiglu_bfp.sv)
//   residual  per-tile aligned add (gen_residual_bfp_golden.py:20-45)
// Every group output is "normalised to Q1.15": shifted so the largest
// magnitude leads at bit 14, low 16 bits kept as the signed mantissa.
#include "bfp_device.cuh"
#include "kernels.cuh"

#include <cstdint>

namespace bfp {

namespace {

constexpr int RT_ACC_W = 48;

__device__ __forceinline__ int lead64(long long v) {
  if (v == 0) return 0;
  const unsigned long long a = v < 0 ? (unsigned long long)(-(v + 1)) + 1ull : (unsigned long long)v;
  return 63 - __clzll((long long)a);
}
__device__ __forceinline__ int16_t norm_mant(long long v, int sh) {
  const long long s = sh >= 0 ? (v >> sh) : (long long)((unsigned long long)v << (-sh));
  return (int16_t)(uint16_t)(s & 0xFFFF);
}
__device__ __forceinline__ int8_t clamp8(int e) { return (int8_t)(e < -128 ? -128 : (e > 127 ? 127 : e)); }

// max over the 16 lanes of a half warp
__device__ __forceinline__ int half_max(int v) {
  #pragma unroll
  for (int o = 8; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_max_i(int v) {
  #pragma unroll
  for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- matvec: one warp per (output row, column); lanes form the tile sums,
// lane 0 folds them in tile order
__global__ void __launch_bounds__(256)
rtl_matvec_kernel(const int16_t* xm, const int8_t* xe, const int16_t* wm, const int8_t* we, int R, int NT, int batch,
                  int16_t* ym, int8_t* ye) {
  __shared__ long long s_sum[8][96];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * 8 + warp;
  if (item >= (long long)R * batch) return;
  const int r = (int)(item % R), c = (int)(item / R);
  const int16_t* x = xm + (size_t)c * NT * 16;
  const int16_t* w = wm + (size_t)r * NT * 16;
  for (int t = lane; t < NT; t += 32) {
    long long s = 0;
    #pragma unroll
    for (int k = 0; k < 16; ++k) s += (long long)x[t * 16 + k] * (long long)w[t * 16 + k];
    s_sum[warp][t] = s;
  }
  __syncwarp();
  if (lane) return;
  const long long hi = (1LL << (RT_ACC_W - 1)) - 1, lo = -(1LL << (RT_ACC_W - 1));
  long long acc = s_sum[warp][0];
  int acc_e = (int)xe[(size_t)c * NT] + (int)we[(size_t)r * NT];
  for (int t = 1; t < NT; ++t) {
    long long s = s_sum[warp][t];
    const int e = (int)xe[(size_t)c * NT + t] + (int)we[(size_t)r * NT + t];
    const int d = e - acc_e;
    if (d > 0) {
      acc = d > RT_ACC_W - 1 ? 0 : (acc >> d);
      acc_e = e;
    } else if (d < 0) {
      s = -d > RT_ACC_W - 1 ? 0 : (s >> -d);
    }
    acc += s;
    acc = acc > hi ? hi : (acc < lo ? lo : acc);
  }
  const int sh = lead64(acc) - 14;
  ym[(size_t)c * R + r] = norm_mant(acc, sh);
  ye[(size_t)c * R + r] = clamp8(acc_e + sh - 15);
}

// ---- rmsnorm: one warp per vector
__device__ const int RSQRT_SEED_Q12[26] = {13698540, 9686330, 6849270, 4843165, 3424635, 2421583, 1712317,
                                           1210791,  856159,  605396,  428079,  302698,  214040,  151349,
                                           107020,   75674,   53510,   37837,   26755,   18919,   13377,
                                           9459,     6689,    4730,    3344,    2365};   // leading bit 6 .. 31

__global__ void __launch_bounds__(128)
rtl_rmsnorm_kernel(const int16_t* xm, const int8_t* xe, const int16_t* gm, const int8_t* ge, int D, int nvec,
                   int16_t* ym, int8_t* ye) {
  __shared__ long long s_sq[4][96];
  __shared__ int s_inv[4], s_einv[4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v = blockIdx.x * 4 + warp;
  if (v >= nvec) return;
  const int NT = D / 16;
  const int16_t* x = xm + (size_t)v * D;
  const int8_t* x_e = xe + (size_t)v * NT;
  for (int t = lane; t < NT; t += 32) {
    long long s = 0;
    #pragma unroll
    for (int k = 0; k < 16; ++k) s += (long long)x[t * 16 + k] * (long long)x[t * 16 + k];
    s_sq[warp][t] = s;
  }
  __syncwarp();
  if (lane == 0) {
    long long acc = s_sq[warp][0];
    int acc_e = 2 * (int)x_e[0];
    for (int t = 1; t < NT; ++t) {
      long long s = s_sq[warp][t];
      const int e = 2 * (int)x_e[t];
      const int d = e - acc_e;
      if (d > 0) {
        acc = d > RT_ACC_W - 1 ? 0 : (acc >> d);
        acc_e = e;
      } else if (d < 0) {
        s = -d > RT_ACC_W - 1 ? 0 : (s >> -d);
      }
      acc += s;
    }
    const unsigned __int128 prod = (unsigned __int128)(unsigned long long)acc * (unsigned long long)((1ull << 32) / D);
    const unsigned long long mean = (unsigned long long)(prod >> 32);
    int lead = mean ? 63 - __clzll((long long)mean) : 0;
    if ((acc_e + lead) & 1) lead -= 1;
    unsigned long long vq = lead >= 30 ? (mean >> (lead - 30)) : (mean << (30 - lead));
    vq += 10737;                                                    // 1e-5 in Q2.30
    const int msb = 63 - __clzll((long long)vq);
    long long y = (msb >= 6 && msb <= 31) ? RSQRT_SEED_Q12[msb - 6] : (1LL << 24) - 1;
    const long long C = (3LL << 30) / 2;
    for (int it = 0; it < 3; ++it) {
      const unsigned __int128 vy2 = (unsigned __int128)vq * (unsigned __int128)(unsigned long long)(y * y);
      const unsigned __int128 t24 = vy2 >> 24;
      long long corr;
      if (t24 >= ((unsigned __int128)1 << 32)) corr = 0;
      else {
        corr = C - (long long)(t24 >> 1);
        corr = corr > 0 ? corr : 0;
      }
      long long ny = (long long)(((__int128)y * corr + (1LL << 29)) >> 30);
      y = ny < (1LL << 24) - 1 ? ny : (1LL << 24) - 1;
    }
    s_inv[warp] = (int)y;
    s_einv[warp] = (30 - acc_e - lead) >> 1;                        // arithmetic shift: floor
  }
  __syncwarp();
  const long long inv = s_inv[warp];
  const int e_inv = s_einv[warp];
  const int16_t* g = gm + (size_t)v * D;
  const int8_t* g_e = ge + (size_t)v * NT;
  // per tile: a half warp, one element per lane
  const int half = lane >> 4, k = lane & 15;
  for (int t0 = 0; t0 < NT; t0 += 2) {
    const int t = t0 + half;
    long long p = 0;
    if (t < NT) p = (long long)x[t * 16 + k] * (long long)g[t * 16 + k] * inv;
    const int sh = half_max(p ? lead64(p) : 0) - 14;
    if (t < NT) {
      ym[(size_t)v * D + t * 16 + k] = norm_mant(p, sh);
      if (k == 0) ye[(size_t)v * NT + t] = clamp8((int)x_e[t] + (int)g_e[t] + e_inv + sh - 27);
    }
  }
}

// ---- RoPE: one thread per rotary pair
__device__ __constant__ int CORDIC_ATAN[16] = {105414357, 62229729, 32880480, 16690645, 8377711, 4192939, 2096981,
                                               1048555,   524285,   262144,   131072,   65536,   32768,   16384,
                                               8192,      4096};

__device__ __forceinline__ long long wrap31(long long v) {
  v &= (1LL << 31) - 1;
  return (v & (1LL << 30)) ? v - (1LL << 31) : v;
}

__global__ void rtl_rope_kernel(const int16_t* xm, const int8_t* xe, const int* pos, const unsigned* turns, int HD,
                                int nvec, int16_t* ym, int8_t* ye) {
  const int H2 = HD / 2;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long long)nvec * H2) return;
  const int v = (int)(gid / H2), j = (int)(gid % H2);
  // angle: pos * turns wrapped to 31 bits, times pi/8 (Q2.29), >> 29, wrapped
  const long long ang = wrap31((wrap31((long long)pos[v] * (long long)turns[j]) * 210828714LL) >> 29);
  long long z = ang;
  bool neg = false;
  if (z > 210828714LL) { z = 421657428LL - z; neg = true; }
  else if (z < -210828714LL) { z = -421657428LL - z; neg = true; }
  long long x = 81504109LL, y = 0;
  #pragma unroll
  for (int i = 0; i < 16; ++i) {
    const long long xs = x >> i, ys = y >> i;
    if (z >= 0) { x -= ys; y += xs; z -= CORDIC_ATAN[i]; }
    else { x += ys; y -= xs; z += CORDIC_ATAN[i]; }
  }
  const long long xr = (x + 2048) >> 12, yr = (y + 2048) >> 12;
  long long c, s;
  if (xr > 32767) c = neg ? -32767 : 32767;
  else if (xr < -32768) c = neg ? 32767 : -32768;
  else c = neg ? -xr : xr;
  s = yr > 32767 ? 32767 : (yr < -32768 ? -32768 : yr);
  const int16_t* xv = xm + (size_t)v * HD;
  const int8_t* ev = xe + (size_t)v * (HD / 16);
  const int ea = ev[j / 16], eb = ev[(j + H2) / 16];
  const int em = ea > eb ? ea : eb;
  const long long a = (em - ea) < 16 ? ((long long)xv[j] >> (em - ea)) : 0;
  const long long b = (em - eb) < 16 ? ((long long)xv[j + H2] >> (em - eb)) : 0;
  const long long p0 = a * c - b * s, p1 = b * c + a * s;
  const int s0 = lead64(p0) - 14, s1 = lead64(p1) - 14;
  ym[(size_t)v * HD + j] = norm_mant(p0, s0);
  ym[(size_t)v * HD + j + H2] = norm_mant(p1, s1);
  ye[(size_t)v * HD + j] = clamp8(em + s0 - 15);
  ye[(size_t)v * HD + j + H2] = clamp8(em + s1 - 15);
}

// ---- softmax: one warp per vector of n scores with one shared exponent.
// ROM index of a difference d <= 0 scaled by 2^shamt (exact: any nonzero d
// scaled by 2^11 or more is below the ROM's -1023 floor)
__device__ __forceinline__ int exp_rom_index(long long d, int shamt) {
  if (d >= 0) return 1023;
  long long ds;
  if (shamt >= 0) {
    if (shamt >= 11) return 0;
    ds = d * (1LL << shamt);
  } else {
    ds = d >> (-shamt > 63 ? 63 : -shamt);
  }
  return ds >= 0 ? 1023 : (ds <= -1023 ? 0 : (int)(ds + 1023));
}

__global__ void __launch_bounds__(128)
rtl_softmax_kernel(const int16_t* xm, const int* xe, int n, int nvec, const uint16_t* lut, int16_t* ym, int* ye) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v = blockIdx.x * 4 + warp;
  if (v >= nvec) return;
  const int16_t* x = xm + (size_t)v * n;
  int mx = -32768;
  for (int i = lane; i < n; i += 32) mx = max(mx, (int)x[i]);
  mx = warp_max_i(mx);
  const int shamt = xe[v] - 8;
  long long sum = 0;
  for (int i = lane; i < n; i += 32) {
    const int idx = exp_rom_index((long long)x[i] - mx, shamt);
    sum += lut[idx];
  }
  #pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  // 1/sum by Newton-Raphson in Q0.32: y <- y (2^33 - sum y) >> 32, 4 steps
  const int msb = sum ? 63 - __clzll(sum) : 0;
  long long y = 1LL << (31 - msb);
  for (int it = 0; it < 4; ++it) {
    const __int128 diff = ((__int128)1 << 33) - (__int128)sum * y;
    y = (long long)(((__int128)y * diff) >> 32);
  }
  int ml = 0;
  for (int i = lane; i < n; i += 32) {
    const int idx = exp_rom_index((long long)x[i] - mx, shamt);
    const long long p = (long long)lut[idx] * y;
    if (p) ml = max(ml, lead64(p));
  }
  const int sh = warp_max_i(ml) - 14;
  for (int i = lane; i < n; i += 32) {
    const int idx = exp_rom_index((long long)x[i] - mx, shamt);
    ym[(size_t)v * n + i] = norm_mant((long long)lut[idx] * y, sh);
  }
  if (lane == 0) {
    const int e = sh - 17;
    ye[v] = e < -128 ? -128 : (e > 127 ? 127 : e);
  }
}

// ---- SwiGLU and the residual add: a half warp per 16-element tile
__global__ void rtl_swiglu_kernel(const int16_t* gm, const int8_t* ge, const int16_t* um, const int8_t* ue,
                                  long long ntiles, const int16_t* lut, int16_t* ym, int8_t* ye) {
  const long long tile = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int k = threadIdx.x & 15;
  const bool ok = tile < ntiles;
  const long long tt = ok ? tile : 0;
  // gate mantissa at the ROM's scale: shifted by e_gate - 5, saturated to
  // 16 bits (a nonzero value shifted left by 16 or more saturates)
  const int sh0 = (int)ge[tt] - 5;
  long long i = gm[tt * 16 + k];
  if (sh0 >= 16) i = i > 0 ? 32767 : (i < 0 ? -32768 : 0);
  else if (sh0 >= 0) i = i * (1LL << sh0);
  else i = i >> (-sh0 > 63 ? 63 : -sh0);
  i = i > 32767 ? 32767 : (i < -32768 ? -32768 : i);
  const long long p = (long long)lut[(int)(i & 0xFFFF)] * (long long)um[tt * 16 + k];
  const int sh = half_max(p ? lead64(p) : 0) - 14;
  if (!ok) return;
  ym[tt * 16 + k] = norm_mant(p, sh);
  if (k == 0) ye[tt] = clamp8((int)ue[tt] + sh - 10);
}

__global__ void rtl_residual_kernel(const int16_t* am, const int8_t* ae, const int16_t* bm, const int8_t* be,
                                    long long ntiles, int16_t* ym, int8_t* ye) {
  const long long tile = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 4;
  const int k = threadIdx.x & 15;
  const bool ok = tile < ntiles;
  const long long tt = ok ? tile : 0;
  const int ea = ae[tt], eb = be[tt], em = ea > eb ? ea : eb;
  const long long a = (em - ea) < 16 ? ((long long)am[tt * 16 + k] >> (em - ea)) : 0;
  const long long b = (em - eb) < 16 ? ((long long)bm[tt * 16 + k] >> (em - eb)) : 0;
  const long long s = a + b;
  const int sh = half_max(s ? lead64(s) : 0) - 14;
  if (!ok) return;
  ym[tt * 16 + k] = norm_mant(s, sh);
  if (k == 0) ye[tt] = clamp8(em + sh);
}

}  // namespace

cudaError_t launch_rtl_matvec(const int16_t* xm, const int8_t* xe, const int16_t* wm, const int8_t* we, int R,
                              int NT, int batch, int16_t* ym, int8_t* ye, cudaStream_t s) {
  if (NT > 96) return cudaErrorInvalidValue;
  const long long items = (long long)R * batch;
  rtl_matvec_kernel<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(xm, xe, wm, we, R, NT, batch, ym, ye);
  return cudaGetLastError();
}

cudaError_t launch_rtl_rmsnorm(const int16_t* xm, const int8_t* xe, const int16_t* gm, const int8_t* ge, int D,
                               int nvec, int16_t* ym, int8_t* ye, cudaStream_t s) {
  if (D % 16 || D / 16 > 96) return cudaErrorInvalidValue;
  rtl_rmsnorm_kernel<<<(nvec + 3) / 4, 128, 0, s>>>(xm, xe, gm, ge, D, nvec, ym, ye);
  return cudaGetLastError();
}

cudaError_t launch_rtl_rope(const int16_t* xm, const int8_t* xe, const int* pos, const unsigned* turns, int HD,
                            int nvec, int16_t* ym, int8_t* ye, cudaStream_t s) {
  const long long n = (long long)nvec * (HD / 2);
  rtl_rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(xm, xe, pos, turns, HD, nvec, ym, ye);
  return cudaGetLastError();
}

cudaError_t launch_rtl_softmax(const int16_t* xm, const int* xe, int n, int nvec, const uint16_t* lut, int16_t* ym,
                               int* ye, cudaStream_t s) {
  rtl_softmax_kernel<<<(nvec + 3) / 4, 128, 0, s>>>(xm, xe, n, nvec, lut, ym, ye);
  return cudaGetLastError();
}

cudaError_t launch_rtl_swiglu(const int16_t* gm, const int8_t* ge, const int16_t* um, const int8_t* ue,
                              long long ntiles, const int16_t* lut, int16_t* ym, int8_t* ye, cudaStream_t s) {
  rtl_swiglu_kernel<<<(unsigned)((ntiles * 16 + 255) / 256), 256, 0, s>>>(gm, ge, um, ue, ntiles, lut, ym, ye);
  return cudaGetLastError();
}

cudaError_t launch_rtl_residual(const int16_t* am, const int8_t* ae, const int16_t* bm, const int8_t* be,
                                long long ntiles, int16_t* ym, int8_t* ye, cudaStream_t s) {
  rtl_residual_kernel<<<(unsigned)((ntiles * 16 + 255) / 256), 256, 0, s>>>(am, ae, bm, be, ntiles, ym, ye);
  return cudaGetLastError();
}

}  // namespace bfp
