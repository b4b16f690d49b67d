// tc.cu -- batched BFP matvec (>= 16 columns) on the tcgen05 tensor cores.
//
// matvec_hw_golden (gen_smollm_blockfp_full.py:214-233) needs, for every
// output row r, column c and 16-element K tile t, the exact tile sum
// S = sum_k W[r,k] x[c,k], floor-shifted by its own exponent gap before the
// int64 accumulation.  The tensor cores form the tile sums; the CUDA cores
// do the per-tile shift and accumulation.
//
// Limbs.  With W' = W - 128 = 256 Wh + Wl' (Wh = W >> 8, Wl' = (W & 255) - 128,
// both signed 8-bit) and x' likewise,
//   S = sum W'x' + 128 sum W + 128 sum x - 16 * 128^2
//   sum W'x' = 65536 (Wh.xh) + 256 (Wh.xl' + Wl'.xh) + (Wl'.xl')
// so every limb product is signed x signed.  One kind::i8 MMA per tile with
// K = 32 (A = [Wl' | Wh]) produces the three limb sums side by side in N:
// the B operand of all tiles is laid out once in shared memory as blocks of
// Nc rows x 16 bytes  [0, xh_0, xl'_0, 0, xh_1, xl'_1, 0, ...]; tile t's
// descriptor starts at block 3t with the K-chunk stride one block, so its
// chunk 0 is [0; xh; xl'] and chunk 1 [xh; xl'; 0], and the N-blocks of D are
// (Wh.xh, Wl'.xh + Wh.xl', Wl'.xl').  Every limb sum fits int32; they are
// recombined in int64.
//
// Weights are repacked once into per-(128-row block, K tile) records
//   [Wl' rows 128 x 16 B][Wh rows 128 x 16 B]
// followed by per-block tables of the rows' corrections cw = 128 sum_k W -
// 16 * 128^2 and tile exponents (rows padded to a multiple of 128 are zero
// weights).  Records stream through a shared-memory ring by TMA bulk copies;
// the tables are bulk-copied once per CTA before the dependency wait.  D
// cycles through four tensor-memory buffers so the MMAs of the next tiles
// overlap the epilogue of this one.
//
// Per (row, column, tile) the epilogue needs S >> sh with sh = (max exponent
// of the row and column) - (tile exponent).  The max exponents come first
// (two pairs per instruction on packed 16-bit lanes); then every tile costs
// two wide multiply-adds when its shifts are at most 16, a 32-bit shift of
// floor(S / 2^16) above.
#include "bfp_device.cuh"
#include "kernels.cuh"

namespace bfp {

namespace {

// CTA shape: NCB columns per CTA; warp 0 streams the records (TMA), warp 1
// issues the MMAs, then EW epilogue warps, four per group of columns (one
// per 32-lane quarter of tensor memory).  16 epilogue warps: the whole
// tensor memory, one CTA per SM, CPT = NCB / 4 columns per thread -- the
// shortest per-thread chains, for grids that leave SMs idle.  8 epilogue
// warps (16 columns only): 256 tensor-memory columns and registers for two
// CTAs per SM, 8 columns per thread, so that on grids larger than the GPU
// one CTA's latency-bound phases (B staging, exponent maxima, the final
// quantization) overlap the other's tile loop.
template <int NCB, int EW>
struct TcShape {
  static_assert((EW == 16 && (NCB == 16 || NCB == 32)) || (EW == 8 && NCB == 16), "shape");
  static constexpr int EPI_WARPS = EW;
  static constexpr int THREADS = (2 + EW) * 32;
  static constexpr int NQ = EW / 4;                        // column groups
  static constexpr int CPT = NCB / NQ;                     // columns per epilogue thread (4 or 8)
  static constexpr int CTAS_PER_SM = EW == 8 ? 2 : 1;
  static constexpr unsigned TMEM_COLS = EW == 8 ? 256u : 512u;
  static constexpr int D_STRIDE = (int)TMEM_COLS / 4;       // columns per D buffer (four buffers, >= 3 NCB)
  static_assert(D_STRIDE >= 3 * NCB, "a D buffer holds 3 NCB columns");
};
constexpr int TC_M = 128;
constexpr int TC_REC = 4096;            // bytes per (128-row block, K tile) record: Wl' and Wh rows
constexpr int TC_SA = 4;                // record ring stages
constexpr int TC_SPIN = 1 << 20;

__device__ __forceinline__ unsigned su32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void pdl_wait_tc() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_tc() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void mb_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(su32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mb_try(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(su32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// bounded wait; returns false (and raises the error flag) when it gives up
__device__ __forceinline__ bool mb_wait(unsigned long long* bar, unsigned parity, int* err) {
  int it = 0;
  while (!mb_try(bar, parity)) {
    if (++it > TC_SPIN) { atomicExch(err, 4); return false; }
  }
  return true;
}

__device__ __forceinline__ uint64_t smem_desc(const void* p, unsigned lbo, unsigned sbo) {
  // K-major, no swizzle; start >> 4 [0,14), LBO >> 4 [16,30), SBO >> 4 [32,46),
  // descriptor version 1 at [46,48), layout type 0 (none) at [61,64)
  const uint64_t a = (su32(p) >> 4) & 0x3FFFu;
  return a | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// kind::i8 instruction descriptor: D s32 [4,6)=2, A s8 [7,10)=1, B s8 [10,13)=1,
// both K-major, N >> 3 at [17,23), M >> 4 at [24,29)
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  const uint32_t z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n"
      :: "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(z), "r"(z) : "memory");
}
__device__ __forceinline__ void tc_commit(unsigned long long* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(su32(bar)) : "memory");
}
// d = a * b + c with a 64-bit product and sum (one wide integer multiply-add)
__device__ __forceinline__ long long mad_wide_s32(int a, int b, long long c) {
  long long d;
  asm("mad.wide.s32 %0, %1, %2, %3;" : "=l"(d) : "r"(a), "r"(b), "l"(c));
  return d;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// consecutive 32-bit TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(taddr) : "memory");
}

template <int CPT>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[CPT]) {
  if constexpr (CPT == 8) tmem_ld8(taddr, r);
  else tmem_ld4(taddr, r);
}


// Per 128-row block: NT records, the rows' limb corrections tile by tile
// ([NT][128] int32), their tile exponents tile by tile ([NT][128] int8) and
// row by row ([128 rows][NTP] bytes, NTP = NT rounded up to 16: the
// max-exponent pass).  The tables are copied into shared memory once per
// CTA; only the records stream through the ring.
__host__ __device__ inline int tc_ntp(int NT) { return (NT + 15) & ~15; }
__host__ __device__ inline size_t tc_cw_off(int NT) { return (size_t)NT * TC_REC; }
__host__ __device__ inline size_t tc_wt_off(int NT) { return (size_t)NT * (TC_REC + TC_M * 4); }
__host__ __device__ inline size_t tc_we_off(int NT) { return (size_t)NT * (TC_REC + TC_M * 5); }
__host__ __device__ inline size_t tc_block_bytes(int NT) { return tc_we_off(NT) + (size_t)TC_M * tc_ntp(NT); }

// ---------------------------------------------------------------------------
// repack: DevMat (planes [G][NT][2][16][16], exponents [G][NT][16]) -> records
// ---------------------------------------------------------------------------
__global__ void tc_pack_kernel(const uint8_t* wm, const int8_t* we, int rows, int NT, int gstride, int goff,
                               uint8_t* rec) {
  // block (b, t); thread = row within the 128-row block
  const int b = blockIdx.x, t = blockIdx.y, r = threadIdx.x;
  const int R = b * TC_M + r;
  uint8_t* blockp = rec + (size_t)b * tc_block_bytes(NT);
  uint8_t* dst = blockp + (size_t)t * TC_REC;
  uint4 hi = make_uint4(0, 0, 0, 0), lo = make_uint4(0, 0, 0, 0);
  int8_t e = 0;
  if (R < rows) {
    const int g = (R / 16) * gstride + goff, ri = R % 16;
    const uint4* src = reinterpret_cast<const uint4*>(wm + ((size_t)g * NT + t) * 512);
    hi = src[ri];
    lo = src[16 + ri];
    e = we[((size_t)g * NT + t) * 16 + ri];
  }
  // W = 256 hi + lo; Wl' = lo - 128 = lo ^ 0x80 as a signed byte
  int sw = 0;
  const unsigned hw[4] = {hi.x, hi.y, hi.z, hi.w}, lw[4] = {lo.x, lo.y, lo.z, lo.w};
  #pragma unroll
  for (int q = 0; q < 4; ++q)
    #pragma unroll
    for (int k = 0; k < 4; ++k) sw += 256 * (int)(int8_t)(hw[q] >> (8 * k)) + (int)((lw[q] >> (8 * k)) & 0xFF);
  const uint4 los = make_uint4(lo.x ^ 0x80808080u, lo.y ^ 0x80808080u, lo.z ^ 0x80808080u, lo.w ^ 0x80808080u);
  reinterpret_cast<uint4*>(dst)[r] = los;                       // Wl' rows
  reinterpret_cast<uint4*>(dst + 2048)[r] = hi;                 // Wh rows
  reinterpret_cast<int*>(blockp + tc_cw_off(NT))[(size_t)t * TC_M + r] = 128 * sw - 16 * 128 * 128;
  reinterpret_cast<int8_t*>(blockp + tc_wt_off(NT))[(size_t)t * TC_M + r] = e;
  reinterpret_cast<int8_t*>(blockp + tc_we_off(NT))[(size_t)r * tc_ntp(NT) + t] = e;
}

// ---------------------------------------------------------------------------
// the matmul
// ---------------------------------------------------------------------------
// Shared memory of one CTA that owns ntl of the NT K tiles (split K: the
// CTAs of a cluster share the tiles; every CTA keeps all NT column exponents
// for the max-exponent pass, and a 128 x NCB int64 block for the reduction).
struct TcLayout {
  size_t bar, tptr, ring, z, xe, xe16, cx, emin, wex, cwt, wet, red, total;
};
__host__ __device__ inline TcLayout tc_layout(int NT, int NCB, int ntl, bool split) {
  TcLayout L;
  L.bar = 0;                                           // mbarriers: ring full / empty, D full / empty, exponents
  L.tptr = 192;                                        // TMEM base address
  L.ring = 256;
  L.z = L.ring + (size_t)TC_SA * TC_REC;
  L.xe = L.z + (size_t)(3 * ntl + 1) * NCB * 16;
  L.xe16 = L.xe + (size_t)NT * NCB * 4;
  L.cx = L.xe16 + (size_t)NT * NCB * 2;
  L.emin = L.cx + (size_t)ntl * NCB * 4;
  L.wex = (L.emin + (size_t)NT * 4 * 4 + 15) & ~(size_t)15;
  L.cwt = L.wex + (size_t)TC_M * tc_ntp(NT);
  L.wet = L.cwt + (size_t)ntl * TC_M * 4;
  L.red = (L.wet + (size_t)ntl * TC_M + 15) & ~(size_t)15;
  L.total = L.red + (split ? (size_t)TC_M * NCB * 8 : 0);
  return L;
}

__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ long long ld_peer_s64(const long long* p, unsigned rank) {
  unsigned remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(su32(p)), "r"(rank));
  long long v;
  asm volatile("ld.shared::cluster.s64 %0, [%1];" : "=l"(v) : "r"(remote) : "memory");
  return v;
}

// Warp roles: warp 0 streams the weight records (TMA), warp 1 issues the
// MMAs, warps 2.. are the epilogue: warp w reads TMEM lanes 32 (w % 4) ..
// +31 (the rows) for column group (w - 2) / 4 (CPT columns per thread).
// Records pass through a ring of TC_SA stages (full: TMA bytes; empty: the
// MMA's commit), D through TC_NB tensor-memory buffers of D_STRIDE columns
// (full: MMA commit; empty: the epilogue warps).  The CTAs resident on an SM
// together allocate all of its tensor memory (512 columns), and the next
// kernel's CTAs allocate only after their dependency wait, when this grid's
// allocations are released.
// Split K: gridDim.z CTAs form a cluster over the K tiles of one output
// block; each computes the full max exponent, accumulates its own tiles,
// and the final phase is shared out by row quarter: rank (q mod ks) adds the
// other CTAs' int64 sums of rows 32q..32q+31 through distributed shared
// memory (integer addition: exact in any order) and runs their epilogue, so
// the clip / quantize / store work of a split runs on up to four SMs.
constexpr int TC_NB = 4;

template <int NCB, int EW, int MODE>
__global__ void __launch_bounds__(TcShape<NCB, EW>::THREADS, TcShape<NCB, EW>::CTAS_PER_SM)
tc_matmul_kernel(TcArgs a) {
  using Shape = TcShape<NCB, EW>;
  constexpr int CPT = Shape::CPT, NQ = Shape::NQ, EPIW = Shape::EPI_WARPS;
  constexpr int TC_THREADS = Shape::THREADS;
  constexpr int N = 3 * NCB;
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NT = a.NT;
  const int blk = blockIdx.x, c0 = blockIdx.y * NCB;
  const int ks = gridDim.z;
  const int kr = ks > 1 ? (int)cluster_rank() : 0;
  const int t_lo = kr * NT / ks, t_hi = (kr + 1) * NT / ks, ntl = t_hi - t_lo;
  const TcLayout L = tc_layout(NT, NCB, (NT + ks - 1) / ks, ks > 1);
  unsigned long long* rfull = reinterpret_cast<unsigned long long*>(smem + L.bar);   // [TC_SA]
  unsigned long long* rempty = rfull + TC_SA;                                         // [TC_SA]
  unsigned long long* dfull = rempty + TC_SA;                                         // [TC_NB]
  unsigned long long* dempty = dfull + TC_NB;                                         // [TC_NB]
  unsigned long long* wbar = dempty + TC_NB;                                          // the exponent table
  uint32_t* tptr = reinterpret_cast<uint32_t*>(smem + L.tptr);
  unsigned char* ring = smem + L.ring;
  unsigned char* Z = smem + L.z;
  int* xe_s = reinterpret_cast<int*>(smem + L.xe);           // [NT][NCB]
  int16_t* xe16_s = reinterpret_cast<int16_t*>(smem + L.xe16); // [NT][NCB], the same exponents as 16-bit lanes
  int* cx_s = reinterpret_cast<int*>(smem + L.cx);           // [ntl][NCB]
  int* emin_s = reinterpret_cast<int*>(smem + L.emin);       // [NT][NQ]: min column exponent per column group
  long long* red = reinterpret_cast<long long*>(smem + L.red); // [NCB][128] (split K)
  const unsigned char* wex_s = smem + L.wex;                  // [128][NTP] tile exponents of the block's rows
  const int* cw_s = reinterpret_cast<const int*>(smem + L.cwt); // [ntl][128] limb corrections of this CTA's tiles
  const int8_t* wt_s = reinterpret_cast<const int8_t*>(smem + L.wet); // [ntl][128] their tile exponents
  const uint8_t* rec = a.rec + (size_t)blk * tc_block_bytes(NT);
  const uint8_t* rec_k = rec + (size_t)t_lo * TC_REC;         // this CTA's first K tile
  pdl_trigger_tc();
  // ---- barriers and the first weight records: the weights do not depend on
  // the previous kernel, so they stream before the wait
  if (tid == 0) {
    for (int s = 0; s < TC_SA; ++s) { mb_init(&rfull[s], 1); mb_init(&rempty[s], 1); }
    for (int b = 0; b < TC_NB; ++b) { mb_init(&dfull[b], 1); mb_init(&dempty[b], EPIW); }
    mb_init(wbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    {
      const unsigned wbytes = (unsigned)(TC_M * tc_ntp(NT)), cbytes = (unsigned)(ntl * TC_M * 4),
                     tbytes = (unsigned)(ntl * TC_M);
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(su32(wbar)), "r"(wbytes + cbytes + tbytes)
                   : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   :: "r"(su32(wt_s)), "l"(rec + tc_wt_off(NT) + (size_t)t_lo * TC_M), "r"(tbytes), "r"(su32(wbar))
                   : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   :: "r"(su32(wex_s)), "l"(rec + tc_we_off(NT)), "r"(wbytes), "r"(su32(wbar)) : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   :: "r"(su32(cw_s)), "l"(rec + tc_cw_off(NT) + (size_t)t_lo * TC_M * 4), "r"(cbytes), "r"(su32(wbar))
                   : "memory");
    }
    for (int s = 0; s < TC_SA && s < ntl; ++s) {
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(su32(&rfull[s])), "r"(TC_REC) : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   :: "r"(su32(ring + (size_t)s * TC_REC)), "l"(rec_k + (size_t)s * TC_REC), "r"(TC_REC),
                      "r"(su32(&rfull[s])) : "memory");
    }
  }
  pdl_wait_tc();
  // tensor memory only after the wait: a CTA waiting on its predecessor holds
  // none, so the predecessor's CTAs can always allocate theirs
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(su32(tptr)), "r"(Shape::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // ---- B operand of every tile, column exponents and sums (columns c0 .. c0+NCB-1)
  for (int i = tid; i < NCB; i += TC_THREADS) {               // the leading zero block (NCB x 16 B)
    reinterpret_cast<uint4*>(Z)[i] = make_uint4(0, 0, 0, 0);
  }
  constexpr int ZB = 4;                                      // items in flight per thread
  for (int i0 = tid; i0 < NT * NCB; i0 += ZB * TC_THREADS) {
    uint4 v[ZB][2];
    int8_t ev[ZB];
    #pragma unroll
    for (int u = 0; u < ZB; ++u) {
      const int i = i0 + u * TC_THREADS, t = i / NCB, c = i - t * NCB, col = c0 + c;
      v[u][0] = v[u][1] = make_uint4(0, 0, 0, 0);
      ev[u] = -127;
      if (i < NT * NCB && col < a.ncols) {
        if (t >= t_lo && t < t_hi) {
          const uint4* xp = reinterpret_cast<const uint4*>(a.xm + (size_t)col * a.x_ld + t * 16);
          v[u][0] = xp[0];
          v[u][1] = xp[1];
        }
        ev[u] = a.xe[(size_t)col * a.x_lde + t];
      }
    }
    #pragma unroll
    for (int u = 0; u < ZB; ++u) {
      const int i = i0 + u * TC_THREADS, t = i / NCB, c = i - t * NCB;
      if (i >= NT * NCB) break;
      xe_s[i] = (int)ev[u];
      xe16_s[i] = (int16_t)ev[u];
      if (t < t_lo || t >= t_hi) continue;
      const int lt = t - t_lo;
      const uint4 v0 = v[u][0], v1 = v[u][1];
      // x = 256 xh + lo: xh = odd bytes, xl' = even bytes ^ 0x80
      const uint4 xh = make_uint4(__byte_perm(v0.x, v0.y, 0x7531), __byte_perm(v0.z, v0.w, 0x7531),
                                  __byte_perm(v1.x, v1.y, 0x7531), __byte_perm(v1.z, v1.w, 0x7531));
      const uint4 xl = make_uint4(__byte_perm(v0.x, v0.y, 0x6420) ^ 0x80808080u, __byte_perm(v0.z, v0.w, 0x6420) ^ 0x80808080u,
                                  __byte_perm(v1.x, v1.y, 0x6420) ^ 0x80808080u, __byte_perm(v1.z, v1.w, 0x6420) ^ 0x80808080u);
      uint4* zb = reinterpret_cast<uint4*>(Z + (size_t)(3 * lt + 1) * NCB * 16);
      zb[c] = xh;
      zb[NCB + c] = xl;
      zb[2 * NCB + c] = make_uint4(0, 0, 0, 0);
      int sx = 0;
      const unsigned w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      #pragma unroll
      for (int k = 0; k < 8; ++k) sx += (int)(int16_t)(w[k] & 0xFFFF) + (int)(int16_t)(w[k] >> 16);
      cx_s[lt * NCB + c] = 128 * sx;
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");     // B written by threads, read by the MMA
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tptr;
  const uint32_t idesc = idesc_i8(TC_M, N);
  // per epilogue thread: max exponent and int64 sum of (row, column cb + j)
  int Mx[CPT];
  long long acc[CPT];
  int resid[CPT];                 // EPI_RESIDUAL: h mantissa (low 16 bits) and tile exponent (above)
  #pragma unroll
  for (int j = 0; j < CPT; ++j) { Mx[j] = 0; acc[j] = 0; resid[j] = 0; }

  if (warp == 0) {
    // ---- producer: refill a ring stage once its MMA and epilogue reads are done
    if (lane == 0) {
      for (int t = TC_SA; t < ntl; ++t) {
        const int s = t % TC_SA;
        mb_wait(&rempty[s], (unsigned)(((t / TC_SA) - 1) & 1), a.err);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(su32(&rfull[s])), "r"(TC_REC) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                     :: "r"(su32(ring + (size_t)s * TC_REC)), "l"(rec_k + (size_t)t * TC_REC), "r"(TC_REC),
                        "r"(su32(&rfull[s])) : "memory");
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      for (int t = 0; t < ntl; ++t) {
        const int s = t % TC_SA, b = t % TC_NB;
        mb_wait(&rfull[s], (unsigned)((t / TC_SA) & 1), a.err);
        if (t >= TC_NB) mb_wait(&dempty[b], (unsigned)(((t / TC_NB) - 1) & 1), a.err);
        tc_fence_after();
        tc_mma(tbase + (uint32_t)(b * Shape::D_STRIDE), smem_desc(ring + (size_t)s * TC_REC, 2048, 128),
               smem_desc(Z + (size_t)3 * t * NCB * 16, NCB * 16, 128), idesc);
        tc_commit(&dfull[b]);
        tc_commit(&rempty[s]);
      }
    }
  } else {
    // ---- epilogue warps
    const int q = warp & 3, quarter = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const int cb = quarter * CPT;
    // max exponent per (row, column) over all tiles (:221-222); the row's tile
    // exponents come from the block's exponent table, 16 at a time
    #pragma unroll
    for (int j = 0; j < CPT; ++j) Mx[j] = -100000;
    if (q == 0) {                   // smallest column exponent of the quarter, per tile (one vector load each)
      for (int t = lane; t < NT; t += 32) {
        const int16_t* xr = xe16_s + t * NCB + cb;
        unsigned m;
        if constexpr (CPT == 8) {
          const uint4 x8 = *reinterpret_cast<const uint4*>(xr);
          m = __vmins2(__vmins2(x8.x, x8.y), __vmins2(x8.z, x8.w));
        } else {
          const uint2 x4 = *reinterpret_cast<const uint2*>(xr);
          m = __vmins2(x4.x, x4.y);
        }
        emin_s[t * NQ + quarter] = min((int)(int16_t)(m & 0xFFFFu), (int)(int16_t)(m >> 16));
      }
    }
    {
      // two (row, column) pairs per instruction: exponent sums fit 16 bits
      // (|we + ex| <= 254), so max(we + ex, M) runs on packed 16-bit lanes
      const int NTP = tc_ntp(NT);
      mb_wait(wbar, 0u, a.err);                              // the table, copied before the dependency wait
      const uint4* wrow = reinterpret_cast<const uint4*>(wex_s + (size_t)row * NTP);
      // four independent chains (tile t in chain t % 4), merged at the end
      unsigned m2[4][CPT / 2];
      #pragma unroll
      for (int c = 0; c < 4; ++c)
        #pragma unroll
        for (int k = 0; k < CPT / 2; ++k) m2[c][k] = 0x8AD08AD0u;       // -30000 in both lanes
      auto step = [&](int t, unsigned wbyte, unsigned (&m)[CPT / 2]) {
        const unsigned we2 = (unsigned)(uint16_t)(int16_t)(int8_t)wbyte * 0x10001u;
        const int16_t* xr = xe16_s + t * NCB + cb;
        if constexpr (CPT == 8) {
          const uint4 x8 = *reinterpret_cast<const uint4*>(xr);
          m[0] = __viaddmax_s16x2(we2, x8.x, m[0]);
          m[1] = __viaddmax_s16x2(we2, x8.y, m[1]);
          m[2] = __viaddmax_s16x2(we2, x8.z, m[2]);
          m[3] = __viaddmax_s16x2(we2, x8.w, m[3]);
        } else {
          const uint2 x4 = *reinterpret_cast<const uint2*>(xr);
          m[0] = __viaddmax_s16x2(we2, x4.x, m[0]);
          m[1] = __viaddmax_s16x2(we2, x4.y, m[1]);
        }
      };
      int t0 = 0;
      for (; t0 + 16 <= NT; t0 += 16) {                     // whole groups of 16 tiles: no guards
        const uint4 w16 = wrow[t0 / 16];
        const unsigned ww[4] = {w16.x, w16.y, w16.z, w16.w};
        #pragma unroll
        for (int k = 0; k < 16; ++k) step(t0 + k, ww[k >> 2] >> (8 * (k & 3)), m2[k & 3]);
      }
      if (t0 < NT) {
        const uint4 w16 = wrow[t0 / 16];
        const unsigned ww[4] = {w16.x, w16.y, w16.z, w16.w};
        #pragma unroll
        for (int k = 0; k < 16; ++k)
          if (t0 + k < NT) step(t0 + k, ww[k >> 2] >> (8 * (k & 3)), m2[k & 3]);
      }
      #pragma unroll
      for (int k = 0; k < CPT / 2; ++k)
        m2[0][k] = __vmaxs2(__vmaxs2(m2[0][k], m2[1][k]), __vmaxs2(m2[2][k], m2[3][k]));
      #pragma unroll
      for (int k = 0; k < CPT / 2; ++k) {
        Mx[2 * k] = (int)(int16_t)(m2[0][k] & 0xFFFFu);
        Mx[2 * k + 1] = (int)(int16_t)(m2[0][k] >> 16);
      }
    }
    int MxMax = Mx[0];
    #pragma unroll
    for (int j = 1; j < CPT; ++j) MxMax = max(MxMax, Mx[j]);
    if constexpr (MODE == EPI_RESIDUAL) {
      // the residual input, loaded now so its latency hides behind the tiles
      const int R = blk * TC_M + row;
      if (kr == q % ks && R < a.rows) {              // this CTA finalises row quarter q
        #pragma unroll
        for (int j = 0; j < CPT; ++j) {
          const int col = c0 + cb + j;
          if (col < a.ncols)
            resid[j] = (int)((unsigned)(uint16_t)a.rm[(size_t)col * a.o_ld + R] |
                             ((unsigned)(int)a.re[(size_t)col * a.o_lde + R / 16] << 16));
        }
      }
    }
    asm volatile("bar.sync 1, %0;" :: "r"(EPIW * 32) : "memory");     // emin_s complete
    #pragma unroll
    for (int j = 0; j < CPT; ++j) acc[j] = 0;
    // per-tile operands advance by pointer: the row's correction and tile
    // exponent ([t][128] tables), the group's smallest column exponent, the
    // columns' exponents and sums
    const uint32_t tq0 = tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)cb;
    const int* cw_p = cw_s + row;
    const int8_t* wt_p = wt_s + row;
    const int* em_p = emin_s + t_lo * NQ + quarter;
    const int* xe_p = xe_s + t_lo * NCB + cb;
    const int* cx_p = cx_s + cb;
    int b = 0;
    unsigned ph = 0;
    for (int t = 0; t < ntl; ++t) {
      // the three limb sums of tile t
      mb_wait(&dfull[b], ph, a.err);
      tc_fence_after();
      uint32_t hh[CPT], cr[CPT], ll[CPT];
      const uint32_t tq = tq0 + (uint32_t)(b * Shape::D_STRIDE);
      tmem_ld<CPT>(tq, hh);
      tmem_ld<CPT>(tq + NCB, cr);
      tmem_ld<CPT>(tq + 2 * NCB, ll);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(su32(&dempty[b])) : "memory");
      const int cw = *cw_p;
      const int wer = (int)*wt_p;
      const int emn = *em_p;
      int ev[CPT], cv[CPT];
      #pragma unroll
      for (int j = 0; j < CPT; j += 4) {
        const int4 e4 = *reinterpret_cast<const int4*>(xe_p + j);
        const int4 x4 = *reinterpret_cast<const int4*>(cx_p + j);
        ev[j] = e4.x; ev[j + 1] = e4.y; ev[j + 2] = e4.z; ev[j + 3] = e4.w;
        cv[j] = x4.x; cv[j + 1] = x4.y; cv[j + 2] = x4.z; cv[j + 3] = x4.w;
      }
      cw_p += TC_M; wt_p += TC_M; em_p += NQ; xe_p += NCB; cx_p += NCB;
      if (++b == TC_NB) { b = 0; ph ^= 1u; }
      // per-tile floor shift and int64 accumulation (:223-228).  S = 65536 hh + w
      // with w = 256 cr + ll + cw + cx = S - 65536 hh (|w| < 2^28).  For
      // sh <= 16, floor(S / 2^sh) = hh * 2^(16-sh) + (w >> sh): two 32 x 32 ->
      // 64-bit multiply-adds.  For sh >= 16, floor(S / 2^sh) =
      // floor(floor(S / 2^16) / 2^(sh-16)) = (hh + (w >> 16)) >> (sh - 16), in
      // 32 bits.  Shifts above ALIGN_MAX contribute nothing.  When every shift
      // of this warp is at most 16 (a bound from the row's largest max
      // exponent and the group's smallest column exponent) only the first form
      // runs.
      const int shb = MxMax - wer - emn;
      if (__all_sync(0xffffffffu, shb <= 16)) {
        #pragma unroll
        for (int j = 0; j < CPT; ++j) {
          const int sh = Mx[j] - wer - ev[j];
          const int w = (int)cr[j] * 256 + ((int)ll[j] + cw + cv[j]);
          acc[j] = mad_wide_s32(w >> sh, 1, mad_wide_s32((int)hh[j], 0x10000 >> sh, acc[j]));
        }
      } else {
        #pragma unroll
        for (int j = 0; j < CPT; ++j) {
          const int sh = Mx[j] - wer - ev[j];
          const int w = (int)cr[j] * 256 + ((int)ll[j] + cw + cv[j]);
          if (sh <= 16) acc[j] = mad_wide_s32(w >> sh, 1, mad_wide_s32((int)hh[j], 0x10000 >> sh, acc[j]));
          else if (sh <= ALIGN_MAX) acc[j] += ((int)hh[j] + (w >> 16)) >> (sh - 16);
        }
      }
    }
    if (ks > 1) {
      #pragma unroll
      for (int j = 0; j < CPT; ++j) red[(cb + j) * TC_M + row] = acc[j];
    }
  }
  // ---- split K: the rank that finalises a row quarter adds the other CTAs'
  // sums of those rows (DSMEM); the second barrier keeps every CTA's shared
  // memory alive until it is read
  const bool fin = warp >= 2 && kr == (warp & 3) % ks;
  if (ks > 1) {
    cluster_sync_all();
    if (fin) {
      const int q = warp & 3, quarter = (warp - 2) >> 2, row = q * 32 + lane, cb = quarter * CPT;
      for (int r = 0; r < ks; ++r) {
        if (r == kr) continue;
        #pragma unroll
        for (int j = 0; j < CPT; ++j) acc[j] += ld_peer_s64(red + (cb + j) * TC_M + row, (unsigned)r);
      }
    }
    cluster_sync_all();
  }
  if (fin) {
    const int q = warp & 3, quarter = (warp - 2) >> 2;
    const int row = q * 32 + lane, R = blk * TC_M + row;
    const int cb = quarter * CPT;
    // ---- epilogue: clip, scale (:229-232), quantize over 16-row output tiles
    // (:233); the CPT columns' quantizations are interleaved (independent
    // warp-wide reductions)
    const bool row_ok = R < a.rows;
    double v[CPT];
    int16_t qm[CPT];
    int qe[CPT];
    #pragma unroll
    for (int j = 0; j < CPT; ++j) {
      long long sacc = acc[j];
      sacc = sacc > SAT_HI ? SAT_HI : (sacc < SAT_LO ? SAT_LO : sacc);
      v[j] = (double)sacc * pow2(Mx[j] - 30);
    }
    tile_quantize_16lanes_n<CPT>(v, qm, qe);
    if constexpr (MODE == EPI_STORE) {
      #pragma unroll
      for (int j = 0; j < CPT; ++j) {
        const int col = c0 + cb + j;
        if (row_ok && col < a.ncols) {
          a.om[(size_t)col * a.o_ld + R] = qm[j];
          if ((R & 15) == 0) a.oe[(size_t)col * a.o_lde + R / 16] = (int8_t)qe[j];
        }
      }
    } else if constexpr (MODE == EPI_RESIDUAL) {
      #pragma unroll
      for (int j = 0; j < CPT; ++j) {                                                  // fpq(h + o)
        const int col = c0 + cb + j;
        const bool valid = row_ok && col < a.ncols;
        const double hv = valid ? bfp_decode((int16_t)(resid[j] & 0xFFFF), resid[j] >> 16) : 0.0;
        v[j] = __dadd_rn(hv, bfp_decode(qm[j], qe[j]));
      }
      tile_quantize_16lanes_n<CPT>(v, qm, qe);
      #pragma unroll
      for (int j = 0; j < CPT; ++j) {
        const int col = c0 + cb + j;
        if (row_ok && col < a.ncols) {
          a.om[(size_t)col * a.o_ld + R] = qm[j];
          if ((R & 15) == 0) a.oe[(size_t)col * a.o_lde + R / 16] = (int8_t)qe[j];
        }
      }
    } else {   // EPI_SWIGLU: lanes 0-15 hold a gate group, lanes 16-31 its up group (the same output rows)
      // Columns go in pairs (j, j+1): the low half-warp computes silu of
      // column j's gate values, the high half-warp that of column j+1's
      // (fetched from the low lanes), so every lane's exp, divide and
      // quantization is kept; each half then forms its column's products with
      // the up values and quantizes them as its own 16-row tile.  The same
      // operations on the same values as one column at a time.
      const bool lo = (lane & 16) == 0;
      constexpr int CP = CPT / 2;
      double sv[CP], up[CP];
      #pragma unroll
      for (int k = 0; k < CP; ++k) {
        const double a0 = bfp_decode(qm[2 * k], qe[2 * k]);            // low: g of column j, high: u of j
        const double a1 = bfp_decode(qm[2 * k + 1], qe[2 * k + 1]);    // low: g of j+1,      high: u of j+1
        const double x0 = __shfl_xor_sync(0xffffffffu, a0, 16);        // low: u of j,        high: g of j
        const double x1 = __shfl_xor_sync(0xffffffffu, a1, 16);        // low: u of j+1,      high: g of j+1
        const double g = lo ? a0 : x1;
        up[k] = lo ? x0 : a1;
        sv[k] = __ddiv_rn(g, __dadd_rn(1.0, exp(-g)));                  // silu_fp (:241-242)
      }
      int16_t sm[CP];
      int se[CP];
      tile_quantize_16lanes_n<CP>(sv, sm, se);
      #pragma unroll
      for (int k = 0; k < CP; ++k) sv[k] = __dmul_rn(bfp_decode(sm[k], se[k]), up[k]);   // (:290)
      tile_quantize_16lanes_n<CP>(sv, sm, se);
      const int ug = R / 32;                                                             // mlp group of the pair
      #pragma unroll
      for (int k = 0; k < CP; ++k) {
        const int col = c0 + cb + 2 * k + (lo ? 0 : 1);
        const bool valid = row_ok && col < a.ncols;
        int16_t pm = sm[k];
        int pe = se[k];
        const unsigned bal = __ballot_sync(0xffffffffu, valid && pm == (int16_t)-32768);
        const bool has_min = ((bal >> (lane & 16)) & 0xFFFFu) != 0;
        pm = requant_mant(pm, has_min && pe < 127);                                     // (:291)
        pe = requant_exp(pe, has_min);
        if (valid) {
          a.om[(size_t)col * a.o_ld + ug * 16 + (lane & 15)] = pm;
          if ((lane & 15) == 0) a.oe[(size_t)col * a.o_lde + ug] = (int8_t)pe;
        }
      }
    }
  }
  // ---- release tensor memory (every MMA waited for, every load completed)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tbase), "r"(Shape::TMEM_COLS) : "memory");
  }
}

template <int NCB, int EW, int MODE>
cudaError_t launch_tc_t(const TcArgs& a, int ks, int nsm, cudaStream_t s, bool pdl) {
  using Shape = TcShape<NCB, EW>;
  const dim3 grid((a.rows + TC_M - 1) / TC_M, (a.ncols + NCB - 1) / NCB, ks);
  const size_t smem = tc_layout(a.NT, NCB, (a.NT + ks - 1) / ks, ks > 1).total;
  // the two-CTAs-per-SM shape is for grids larger than the GPU; on fewer
  // CTAs the sixteen-warp shape's shorter per-thread chains are faster
  if (Shape::CTAS_PER_SM > 1 && (long)grid.x * grid.y * grid.z <= nsm) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(tc_matmul_kernel<NCB, EW, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  if (Shape::CTAS_PER_SM > 1) {      // all of the SM's unified memory as shared memory: room for both CTAs
    e = cudaFuncSetAttribute(tc_matmul_kernel<NCB, EW, MODE>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
  }
  if (ks > 1) {
    e = cudaFuncSetAttribute(tc_matmul_kernel<NCB, EW, MODE>, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(Shape::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (ks > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = ks;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, tc_matmul_kernel<NCB, EW, MODE>, a);
}

bool tc_config_fits(int NT, int ncb, int ks) {
  return (ncb == 16 || ncb == 32) && ks >= 1 && ks <= 8 && ks <= NT &&
         tc_layout(NT, ncb, (NT + ks - 1) / ks, ks > 1).total <= 227 * 1024;
}

// Without a tuned configuration: no K split; 32 columns per CTA when that
// grid still covers the SMs, else 16.
void tc_default_config(int rows, int NT, int ncols, int nsm, int* ncb, int* ks) {
  const int nblk = (rows + TC_M - 1) / TC_M;
  *ks = 1;
  *ncb = (nblk * ((ncols + 31) / 32) >= nsm && tc_config_fits(NT, 32, 1)) ? 32 : 16;
}

}  // namespace

size_t tc_records_bytes(int rows, int NT) { return (size_t)((rows + TC_M - 1) / TC_M) * tc_block_bytes(NT); }

cudaError_t launch_tc_pack(const uint8_t* wm, const int8_t* we, int rows, int NT, uint8_t* rec, cudaStream_t s) {
  dim3 grid((rows + TC_M - 1) / TC_M, NT);
  tc_pack_kernel<<<grid, TC_M, 0, s>>>(wm, we, rows, NT, 1, 0, rec);
  return cudaGetLastError();
}

bool tc_supported(int NT, int ncols) {
  if (ncols < 1 || NT < 1) return false;
  return tc_config_fits(NT, 16, 1) || tc_config_fits(NT, 16, 8);
}

bool tc_config_valid(int NT, int ncb, int ks) { return tc_config_fits(NT, ncb, ks); }

cudaError_t launch_tc_matmul(const TcArgs& a, cudaStream_t s, bool pdl) {
  int ncb = a.ncb, ks = a.ks;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (ncb == 0 || ks == 0) tc_default_config(a.rows, a.NT, a.ncols, nsm, &ncb, &ks);
  if (!tc_config_fits(a.NT, ncb, ks)) return cudaErrorInvalidValue;
  if (a.mode == EPI_SWIGLU && (a.rows % 32)) return cudaErrorInvalidValue;
  const int ew = a.ew ? a.ew : 16;
  if (ew != 16 && !(ew == 8 && ncb == 16)) return cudaErrorInvalidValue;
  auto go = [&](auto mode_tag) -> cudaError_t {
    constexpr int M = decltype(mode_tag)::value;
    if (ncb == 32) return launch_tc_t<32, 16, M>(a, ks, nsm, s, pdl);
    if (ew == 8) return launch_tc_t<16, 8, M>(a, ks, nsm, s, pdl);
    return launch_tc_t<16, 16, M>(a, ks, nsm, s, pdl);
  };
  switch (a.mode) {
    case EPI_STORE: return go(std::integral_constant<int, EPI_STORE>{});
    case EPI_RESIDUAL: return go(std::integral_constant<int, EPI_RESIDUAL>{});
    case EPI_SWIGLU: return go(std::integral_constant<int, EPI_SWIGLU>{});
  }
  return cudaErrorInvalidValue;
}

}  // namespace bfp
