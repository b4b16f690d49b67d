// stamps.cuh -- optional phase timestamps of the decode-path kernels, for
// measurement builds only: compiled in with -DBFP200_STAMPS, absent (no code,
// no storage) otherwise.  Thread 0 of a CTA records %clock64 (per-SM cycles)
// and %globaltimer (ns, comparable across SMs) at point `pt` of kernel kind
// `kind` on layer `layer`.
#pragma once
#ifdef BFP200_STAMPS
namespace bfp {
constexpr int STAMP_KINDS = 4, STAMP_CTAS = 128, STAMP_PTS = 16, STAMP_LAYERS = 30;
constexpr int STAMP_N = STAMP_LAYERS * STAMP_KINDS * STAMP_CTAS * STAMP_PTS;
static __device__ unsigned long long g_stamp_clk[STAMP_N];
static __device__ unsigned long long g_stamp_ns[STAMP_N];
}  // namespace bfp
#define BFP_STAMP(kind, layer, cta, pt)                                                              \
  do {                                                                                               \
    if (threadIdx.x == 0 && (layer) < STAMP_LAYERS && (cta) < STAMP_CTAS) {                          \
      unsigned long long c_, t_;                                                                     \
      asm volatile("mov.u64 %0, %%clock64;" : "=l"(c_) :: "memory");                                \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_) :: "memory");                             \
      const int i_ = ((((layer) * STAMP_KINDS + (kind)) * STAMP_CTAS + (cta)) * STAMP_PTS + (pt));   \
      g_stamp_clk[i_] = c_;                                                                          \
      g_stamp_ns[i_] = t_;                                                                           \
    }                                                                                                \
  } while (0)
// the same, recorded by thread `th` instead of thread 0
#define BFP_STAMP_T(th, kind, layer, cta, pt)                                                        \
  do {                                                                                               \
    if (threadIdx.x == (th) && (layer) < STAMP_LAYERS && (cta) < STAMP_CTAS) {                       \
      unsigned long long c_;                                                                         \
      asm volatile("mov.u64 %0, %%clock64;" : "=l"(c_) :: "memory");                                \
      g_stamp_clk[((((layer) * STAMP_KINDS + (kind)) * STAMP_CTAS + (cta)) * STAMP_PTS + (pt))] = c_; \
    }                                                                                                \
  } while (0)
#define BFP_STAMP_READER(name)                                                                       \
  extern "C" int name(unsigned long long* clk, unsigned long long* ns) {                             \
    if (cudaMemcpyFromSymbol(clk, bfp::g_stamp_clk, sizeof(bfp::g_stamp_clk)) != cudaSuccess) return -1; \
    if (cudaMemcpyFromSymbol(ns, bfp::g_stamp_ns, sizeof(bfp::g_stamp_ns)) != cudaSuccess) return -1; \
    return 0;                                                                                        \
  }
#else
#define BFP_STAMP(kind, layer, cta, pt) do {} while (0)
#define BFP_STAMP_T(th, kind, layer, cta, pt) do {} while (0)
#define BFP_STAMP_READER(name)
#endif
