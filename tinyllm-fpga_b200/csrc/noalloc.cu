// noalloc.cu -- bfp200_matvec_noalloc: the BFP matvec for callers that
// cannot allocate device memory.
//
// Some callers manage every byte of device memory themselves: a framework
// with its own caching allocator or fixed memory pool, or a latency-critical
// loop that cannot afford the implicit device synchronisation of
// cudaMalloc/cudaFree.  This entry point takes device pointers for all
// inputs and outputs and allocates nothing.  The one piece of memory the
// kernel needs beyond them -- the K-split accumulators and arrival counters
// of the matmul -- lives in the file-scope array below, which every GPU that
// loads libbfp200 holds until the process exits.
#include "../../include/bfp200.h"
#include "kernels.cuh"

#include <mutex>
#include <string>

using namespace bfp;

// Set the calling thread's bfp200_last_error text (engine.cu).
int bfp200_set_error(int code, const std::string& msg);

namespace {

// int64 accumulators: D_out * batch entries at most (2 MiB) ...
constexpr size_t NOALLOC_ACC_MAX = 262144;
// ... followed by 16384 uint32 arrival counters (64 KiB).
constexpr size_t NOALLOC_CNT_MAX = 16384;

static __device__ __align__(256) long long g_noalloc_scratch[NOALLOC_ACC_MAX + NOALLOC_CNT_MAX / 2];

struct DevState {
  bool ready = false;
  long long* scratch = nullptr;   // device address of g_noalloc_scratch on this device
  int nsm = 0;
};

std::mutex g_mu;
DevState g_dev[128];

// Once per device, with that device current: the device address of the
// scratch array (the host-side symbol is only a stand-in) and the kernels'
// shared-memory limits.
int setup(int dev, DevState** out) {
  if (dev < 0 || dev >= 128) return bfp200_set_error(BFP200_ENODEV, "matvec_noalloc: device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  DevState& d = g_dev[dev];
  if (!d.ready) {
    int major = 0;
    cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return bfp200_set_error(BFP200_ECUDA, std::string("matvec_noalloc: ") + cudaGetErrorString(e));
    if (major != 10) return bfp200_set_error(BFP200_ENODEV, "matvec_noalloc: needs an sm_100 (B200) device");
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.scratch), g_noalloc_scratch);
    if (e != cudaSuccess)
      return bfp200_set_error(BFP200_ECUDA, std::string("matvec_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    e = init_kernel_attributes();
    if (e != cudaSuccess) return bfp200_set_error(BFP200_ECUDA, std::string("matvec_noalloc: ") + cudaGetErrorString(e));
    e = cudaDeviceGetAttribute(&d.nsm, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return bfp200_set_error(BFP200_ECUDA, std::string("matvec_noalloc: ") + cudaGetErrorString(e));
    d.ready = true;
  }
  *out = &d;
  return BFP200_OK;
}

}  // namespace

extern "C" int bfp200_matvec_noalloc(const int16_t* x_m, const int8_t* x_e, const int16_t* W_m, const int8_t* W_e,
                                     int D_out, int D_in, int batch, int16_t* out_m, int8_t* out_e, void* stream) {
  if (!x_m || !x_e || !W_m || !W_e || !out_m || !out_e || D_out <= 0 || D_in <= 0 || D_out % 16 || D_in % 16 ||
      batch <= 0)
    return bfp200_set_error(BFP200_EINVAL,
                            "matvec_noalloc: bad arguments (device pointers, D_out and D_in multiples of 16, batch >= 1)");
  // x_m rows are read 16 bytes at a time and W_m rows by bulk copies, which
  // need 16-byte-aligned addresses; out_m takes 2-byte stores.  A caller that
  // sub-allocates from its own pool can hand in offset pointers: reject them
  // here, before any kernel could fault on them.
  if (((reinterpret_cast<uintptr_t>(x_m) | reinterpret_cast<uintptr_t>(W_m)) & 15u) ||
      (reinterpret_cast<uintptr_t>(out_m) & 1u))
    return bfp200_set_error(BFP200_EINVAL,
                            "matvec_noalloc: x_m and W_m must be 16-byte aligned and out_m 2-byte aligned");
  if ((size_t)D_out * (size_t)batch > NOALLOC_ACC_MAX)
    return bfp200_set_error(BFP200_EINVAL, "matvec_noalloc: D_out * batch = " +
                                               std::to_string((long long)D_out * batch) +
                                               " exceeds the fixed scratch of " + std::to_string(NOALLOC_ACC_MAX) +
                                               " accumulators");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return bfp200_set_error(BFP200_ECUDA, cudaGetErrorString(e));
  DevState* ds = nullptr;
  int rc = setup(dev, &ds);
  if (rc != BFP200_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  const int NT = D_in / 16, G = D_out / 16;
  MatmulArgs a;
  a.W.wm = reinterpret_cast<const uint8_t*>(W_m);
  a.W.we = W_e;
  a.W.G = G;
  a.W.NT = NT;
  a.xm = x_m; a.xe = x_e; a.x_ld = D_in; a.x_lde = NT;
  a.ncols = batch;
  a.epi = EPI_STORE;
  a.om = out_m; a.oe = out_e; a.o_ld = D_out; a.o_lde = G;
  a.rg = 1;
  a.bn = batch <= 32 ? batch : 32;
  // K split: smallest that fits shared memory, grown while the grid stays
  // under two CTAs per SM and the arrival counters fit the scratch.
  const long tiles = (long)G * ((batch + a.bn - 1) / a.bn);
  int best = -1;
  for (int ks = 1; ks <= NT; ++ks) {
    if (NT % ks) continue;
    if (matmul_refw_smem_bytes(a.rg, a.bn, NT / ks, NT) > 200 * 1024) continue;
    if (ks > 1 && tiles > (long)NOALLOC_CNT_MAX) break;
    if (best < 0) best = ks;
    else if (tiles * ks <= 2L * ds->nsm && NT / ks >= 4) best = ks;
  }
  if (best < 0) return bfp200_set_error(BFP200_EINVAL, "matvec_noalloc: no K split fits shared memory");
  a.ksplit = best;
  a.acc = ds->scratch;
  a.counters = reinterpret_cast<unsigned*>(ds->scratch + NOALLOC_ACC_MAX);
  a.acc_ld = batch;
  if (a.ksplit > 1) {
    // the kernel leaves the accumulators and counters at zero, but a call
    // that failed part-way could not: clear what this call uses
    e = cudaMemsetAsync(a.acc, 0, (size_t)D_out * batch * sizeof(long long), s);
    if (e == cudaSuccess) e = cudaMemsetAsync(a.counters, 0, (size_t)tiles * sizeof(unsigned), s);
    if (e != cudaSuccess) return bfp200_set_error(BFP200_ECUDA, std::string("matvec_noalloc: ") + cudaGetErrorString(e));
  }
  e = launch_matmul_refw(a, s);
  if (e != cudaSuccess) return bfp200_set_error(BFP200_ECUDA, std::string("matvec_noalloc: ") + cudaGetErrorString(e));
  return BFP200_OK;
}
