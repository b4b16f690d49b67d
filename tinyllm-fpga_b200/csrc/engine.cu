// engine.cu -- host runtime and C ABI (include/bfp200.h) of libbfp200.so.
//
// A handle owns one device: the repacked weight image, a per-sequence BFP KV
// arena, activation buffers and a captured CUDA graph of one decode step.
// generate() = causal prefill of every prompt position (chunked, position
// ordered, so each chunk only reads KV written by earlier chunks or earlier
// in the same layer), then n_gen decode steps replayed from the graph with
// the token feedback kept on the device.
#include "../../include/bfp200.h"
#include "bfp_device.cuh"
#include "kernels.cuh"

#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <map>
#include <tuple>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

using namespace bfp;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define CK(x)                                                                                  \
  do {                                                                                         \
    cudaError_t _e = (x);                                                                      \
    if (_e != cudaSuccess) return fail(BFP200_ECUDA, std::string(#x) + ": " + cudaGetErrorString(_e)); \
  } while (0)

#define CKR(x)                       \
  do {                               \
    int _r = (x);                    \
    if (_r != BFP200_OK) return _r;  \
  } while (0)

template <typename T>
struct DBuf {
  T* p = nullptr;
  size_t n = 0;
  DBuf() = default;
  DBuf(const DBuf&) = delete;
  DBuf& operator=(const DBuf&) = delete;
  ~DBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  // (Re)allocates to at least `count` elements, zero-filled.  The fill runs on
  // the legacy default stream, which does not order against the handle's
  // non-blocking stream: wait for it before the buffer is used.
  cudaError_t ensure(size_t count) {
    if (count <= n && p) return cudaSuccess;
    release();
    cudaError_t e = cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T));
    if (e != cudaSuccess) { p = nullptr; return e; }
    n = count;
    e = cudaMemset(p, 0, std::max<size_t>(count, 1) * sizeof(T));
    if (e != cudaSuccess) return e;
    return cudaStreamSynchronize(0);
  }
};

struct MMPlan {
  int rg = 1, bn = 1, ks = 1;
};

constexpr size_t MM_SMEM_LIMIT = 200 * 1024;

MMPlan plan_matmul(int G, int NT, int ncols, bool swiglu, int nsm, int max_ks = 1 << 30) {
  MMPlan p;
  p.rg = swiglu ? 2 : 1;
  p.bn = ncols <= 32 ? ncols : 32;
  const long rows_t = G / p.rg, cols_t = (ncols + p.bn - 1) / p.bn;
  const long target = 2L * nsm;
  int best = -1;
  for (int ks = 1; ks <= NT; ++ks) {
    if (NT % ks) continue;
    const int ntc = NT / ks;
    if (matmul_smem_bytes(p.rg, p.bn, ntc, NT) > MM_SMEM_LIMIT) continue;
    if (best < 0) best = ks;
    else if (rows_t * cols_t * ks <= target && ntc >= 4 && ks <= max_ks) best = ks;
  }
  p.ks = best < 0 ? NT : best;
  return p;
}

// Layout of the packed DDR3 image (gen_smollm_blockfp_ddr.py:155-221,
// lbfp_ddr3.svh:45-86): each region padded to 4 KiB, in this order.
struct Region {
  std::string name;
  size_t off = 0, size = 0;
};

size_t align4k(size_t n) { return (n + 4095) & ~size_t(4095); }

std::vector<Region> image_regions(const bfp200_cfg& c) {
  std::vector<Region> r;
  size_t off = 0;
  auto add = [&](const std::string& name, size_t size) {
    r.push_back({name, off, size});
    off += align4k(size);
  };
  const int KVD = c.H_KV * c.HD;
  const struct { const char* tag; int dout, din; } mats[] = {
      {"WQ", c.D, c.D}, {"WK", KVD, c.D}, {"WV", KVD, c.D}, {"WO", c.D, c.D},
      {"WG", c.FFN, c.D}, {"WU", c.FFN, c.D}, {"WDN", c.D, c.FFN}};
  for (auto& m : mats) {
    add(std::string(m.tag) + "_m", (size_t)c.NL * (m.dout / 16) * m.din * 32);
    add(std::string(m.tag) + "_e", (size_t)c.NL * (m.dout / 16) * (m.din / 16) * 16);
  }
  const int NTD = c.D / 16;
  add("G1_m", (size_t)c.NL * c.D * 2);
  add("G1_e", (size_t)c.NL * NTD);
  add("G2_m", (size_t)c.NL * c.D * 2);
  add("G2_e", (size_t)c.NL * NTD);
  add("EMBED_m", (size_t)c.VOCAB / 16 * c.D * 32);
  add("EMBED_e", (size_t)c.VOCAB / 16 * NTD * 16);
  add("EMBED_LU_m", (size_t)c.VOCAB * c.D * 2);
  add("EMBED_LU_e", (size_t)c.VOCAB * 64);
  add("NORM_W_m", (size_t)c.D * 2);
  add("NORM_W_e", (size_t)NTD);
  r.push_back({"END", off, 0});
  return r;
}

const Region* find_region(const std::vector<Region>& rs, const std::string& name) {
  for (auto& r : rs)
    if (r.name == name) return &r;
  return nullptr;
}

// numpy pairwise-summation plan of a length n (see np_sum_warp_plan): the
// recursive tree of pairwise_sum (leaves <= 128, split at n/2 rounded down to
// a multiple of 8), flattened to leaf starts and internal nodes by height.
void build_pw_plan_one(int n, std::vector<unsigned short>& out) {
  struct Node { int lo, len, left, right, height; };
  std::vector<Node> nodes;
  std::vector<int> leaves;
  auto build = [&](auto&& self, int lo, int len) -> int {
    if (len <= 128) {
      nodes.push_back({lo, len, -1, -1, 0});
      leaves.push_back((int)nodes.size() - 1);
      return (int)nodes.size() - 1;
    }
    int n2 = len / 2;
    n2 -= n2 % 8;
    const int l = self(self, lo, n2);
    const int r = self(self, lo + n2, len - n2);
    nodes.push_back({lo, len, l, r, std::max(nodes[l].height, nodes[r].height) + 1});
    return (int)nodes.size() - 1;
  };
  build(build, 0, n);
  std::vector<int> internal;
  for (int i = 0; i < (int)nodes.size(); ++i)
    if (nodes[i].left >= 0) internal.push_back(i);
  std::stable_sort(internal.begin(), internal.end(),
                   [&](int a, int b) { return nodes[a].height < nodes[b].height; });
  std::vector<int> slot(nodes.size(), -1);
  const int L = (int)leaves.size();
  for (int k = 0; k < L; ++k) slot[leaves[k]] = k;
  for (int j = 0; j < (int)internal.size(); ++j) slot[internal[j]] = L + j;
  const int H = internal.empty() ? 0 : nodes[internal.back()].height;
  out.push_back((unsigned short)L);
  out.push_back((unsigned short)H);
  for (int k = 0; k < L; ++k) out.push_back((unsigned short)nodes[leaves[k]].lo);
  for (int hgt = 1; hgt <= H; ++hgt) {
    int cnt = 0;
    for (int i : internal) cnt += nodes[i].height == hgt;
    out.push_back((unsigned short)cnt);
  }
  for (int i : internal) {
    out.push_back((unsigned short)slot[nodes[i].left]);
    out.push_back((unsigned short)slot[nodes[i].right]);
  }
}

// Exact (m, e) form of a tile of BFP grid values (lossless; a tile whose
// minimum is -2^e keeps exponent e and mantissa -32768).  Returns false if
// the values are not on a 16-bit BFP grid.
bool grid_encode_tile(const double* v, int16_t* m, int8_t* e) {
  double mx = 0.0;
  for (int i = 0; i < 16; ++i) mx = std::max(mx, std::fabs(v[i]));
  const int e1 = tile_exponent(mx);
  for (int ee : {e1, e1 - 1}) {
    if (ee < -127) continue;
    bool ok = true;
    int16_t mm[16];
    for (int i = 0; i < 16 && ok; ++i) {
      const double x = v[i] * pow2(15 - ee);
      if (x != std::rint(x) || x < -32768.0 || x > 32767.0) ok = false;
      else mm[i] = (int16_t)(int)x;
    }
    if (ok) {
      std::memcpy(m, mm, sizeof(mm));
      *e = (int8_t)ee;
      return true;
    }
  }
  return false;
}

__global__ void advance_kernel(const int* tok, const int* cert, int ncols, int n_gen, int* gen_out, int* col_tok,
                               int* col_pos, int* dec_step, long long* uncert) {
  __shared__ int s_step;
  if (threadIdx.x == 0) s_step = *dec_step;
  __syncthreads();
  const int step = s_step;
  int bad = 0;
  for (int c = threadIdx.x; c < ncols; c += blockDim.x) {
    const int t = tok[c];
    if (step < n_gen) gen_out[(size_t)c * n_gen + step] = t;
    col_tok[c] = t;
    col_pos[c] += 1;
    bad += cert[c] ? 0 : 1;
  }
  if (bad) atomicAdd(reinterpret_cast<unsigned long long*>(uncert), (unsigned long long)bad);
  __syncthreads();
  if (threadIdx.x == 0) *dec_step = step + 1;
}

__global__ void scatter_tokens_kernel(const int* tok, const int* cert, const int* slot, const int* pos, int ncols,
                                      int stride, int* out, long long* uncert) {
  int bad = 0;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < ncols; c += gridDim.x * blockDim.x) {
    out[(size_t)slot[c] * stride + pos[c]] = tok[c];
    bad += cert[c] ? 0 : 1;
  }
  if (bad) atomicAdd(reinterpret_cast<unsigned long long*>(uncert), (unsigned long long)bad);
}

}  // namespace

int bfp200_set_error(int code, const std::string& msg) { return fail(code, msg); }

// Makes a handle's device current for one entry point and restores the
// caller's device afterwards (callers such as torch keep their own notion of
// the current device).
struct DeviceGuard {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    err = cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// ---------------------------------------------------------------------------
// NCCL, loaded at run time: only the vocabulary-sharded head uses it, so the
// library itself does not depend on libnccl.  The types are NCCL's C ABI
// (ncclUniqueId: 128 bytes by value; results and data types: C enums).
// ---------------------------------------------------------------------------
// a tuned tensor-core matmul configuration; all zero: the built-in choice
struct TcChoice { int ncb = 0, ks = 0, ew = 0; };

struct NcclUid { char internal[BFP200_NCCL_ID_BYTES]; };
typedef struct ncclComm* NcclComm;
constexpr int NCCL_OK = 0, NCCL_IN_PROGRESS = 7, NCCL_F64 = 8;

struct NcclApi {
  int (*get_unique_id)(NcclUid*) = nullptr;
  int (*comm_init_rank)(NcclComm*, int, NcclUid, int) = nullptr;
  int (*comm_init_all)(NcclComm*, int, const int*) = nullptr;
  int (*all_gather)(const void*, void*, size_t, int, NcclComm, cudaStream_t) = nullptr;
  int (*comm_destroy)(NcclComm) = nullptr;
  int (*comm_abort)(NcclComm) = nullptr;
  int (*async_error)(NcclComm, int*) = nullptr;
  const char* (*error_string)(int) = nullptr;
  int (*group_start)() = nullptr;
  int (*group_end)() = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    // the copy already in the process (e.g. torch's), else $BFP200_NCCL_LIB,
    // else whatever the loader finds
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib)
      if (const char* p = std::getenv("BFP200_NCCL_LIB")) lib = dlopen(p, RTLD_NOW | RTLD_GLOBAL);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return;
    auto sym = [&](const char* n) { return dlsym(lib, n); };
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
    api.comm_init_all = reinterpret_cast<decltype(api.comm_init_all)>(sym("ncclCommInitAll"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(sym("ncclCommAbort"));
    api.async_error = reinterpret_cast<decltype(api.async_error)>(sym("ncclCommGetAsyncError"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(sym("ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(sym("ncclGroupEnd"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_init_all && api.all_gather && api.comm_destroy &&
             api.comm_abort && api.async_error && api.error_string && api.group_start && api.group_end;
  });
  return api;
}

std::string nccl_err(int r) {
  const NcclApi& a = nccl();
  return a.error_string ? std::string(a.error_string(r)) : "NCCL error " + std::to_string(r);
}

// Small exchanges gain nothing from NVLink SHARP: keep the multicast objects
// unbound.  Connect every peer at communicator creation (NCCL otherwise
// connects on the first collective, a host-side exchange that would block an
// exchange captured in a graph, or wait forever for a rank that never comes).
// Caller settings win.
void nccl_env_defaults() {
  setenv("NCCL_NVLS_ENABLE", "0", /*overwrite=*/0);
  setenv("NCCL_RUNTIME_CONNECT", "0", /*overwrite=*/0);
}

struct bfp200_handle {
  bfp200_cfg cfg{};
  int device = 0;
  int nsm = 148;
  cudaStream_t stream = nullptr;
  int D = 0, HQ = 0, HKV = 0, HD = 0, FFN = 0, NL = 0, V = 0, MAXC = 0, NTD = 0, NTF = 0, KVD = 0, QD = 0;
  int RQKV = 0, GQKV = 0, GO = 0, GGU = 0, GD = 0;
  bool pdl = true;
  bool use_clusters = true;   // K-split reduction through distributed shared memory
  bool use_small = true;      // 1..4 columns: the fused small-batch kernels (gemv.cu)
  bool use_tc = true;         // >= tc_min_cols columns: matmuls on the tcgen05 tensor cores (tc.cu)
  int tc_min_cols = 16;       // below: the dp2a matmul (one 16-column tile is the MMA's smallest N)
  bool use_block = true;      // 1 column: the attention half of a layer in one cluster launch (layer1.cu)
  bool block_ok = false;      // ... and its plan fits this configuration
  L1Args block{};             // plan fields of that launch (og_*, ch)
  // stage dump of the decode-path kernels (bfp200_fwd_layer_decode): device
  // buffer [column][stage values] in bfp200_fwd_layer's stage layout, or null
  DBuf<double> stage_buf;
  double* stage_dbg = nullptr;
  int stage_ld = 0;
  int smem_optin = 0;
  // weights
  DBuf<uint8_t> wm_qkv, wm_o, wm_gu, wm_d;
  DBuf<int8_t> we_qkv, we_o, we_gu, we_d;
  DBuf<double> g1, g2, nw;
  DBuf<int16_t> emb_m;
  DBuf<int8_t> emb_e;
  DBuf<double> emb_norm;
  double emb_norm_max = 0.0;
  DBuf<double> rope_cs;
  DBuf<int> pw_off;                 // numpy pairwise-sum plans for lengths 0..MAX_CTX
  DBuf<unsigned short> pw_data;
  std::vector<int16_t> g1m, g2m, nwm;
  std::vector<int8_t> g1e, g2e, nwe;
  std::vector<int32_t> rom_prompt;
  bool have_image = false;
  // KV arena
  DBuf<int16_t> km, vm;
  DBuf<int8_t> ke, ve;
  // activations (column capacity cap)
  int cap = 0;
  DBuf<int16_t> h_m, h1_m, n_m, qkv_m, qr_m, a_m, mlp_m, dbg_m;
  DBuf<int8_t> h_e, h1_e, n_e, qkv_e, qr_e, a_e, mlp_e, dbg_e;
  DBuf<long long> acc;
  DBuf<unsigned> counters;
  DBuf<double> hn, hn_norm, part_val, part_sec;
  DBuf<int> part_idx, tok, cert;
  DBuf<int> col_slot, col_pos, col_kvpos, col_tok;
  DBuf<int> gen_out, dec_step, rtl_out;
  DBuf<long long> uncert_dev;
  // tensor-core records of the QKV, O, gate/up and down matrices, all layers
  DBuf<uint8_t> tc_rec[4];
  size_t tc_stride[4] = {0, 0, 0, 0};
  DBuf<unsigned> head_ctr;     // arrival counter of the single-launch head (left zeroed)
  HeadAdvance head_adv;        // set while a decode graph is captured: the head does the token feedback
  // tensor-core matmul configuration (columns per CTA, K split, epilogue
  // warps) per (rows, K tiles, columns, epilogue), chosen by timing the candidates
  std::map<std::tuple<int, int, int, int>, TcChoice> tc_cfg;
  // vocabulary-sharded head: this rank scans rows [v_lo, v_hi) and exchanges
  // one record per column with the other ranks (xsend -> xrecv, all-gather)
  NcclComm comm = nullptr;
  int shard_n = 1, shard_rank = 0, v_lo = 0, v_hi = 0;
  // set when work of an aborted exchange never left the stream: the handle
  // can no longer be used (every call fails; the process should exit)
  bool broken = false;
  DBuf<double> xsend, xrecv, xwarm;
  // sampling (bfp200_generate_sampled): full logits, scratch, uniforms, and
  // numpy's pairwise-sum plan for the vocabulary length
  DBuf<double> s_logits, s_work, s_cdf, s_uni;
  DBuf<int> s_incl;
  DBuf<unsigned short> v_plan;
  int v_plan_leaves = 0;
  cudaGraphExec_t graph = nullptr;
  int graph_cols = -1, graph_ngen = -1;
  double graph_temp = 0.0;        // sampling parameters the cached graph was captured with (0: greedy)
  int graph_topk = 0;
  long long uncert = 0;
  double t_prefill = 0.0, t_decode = 0.0;
  long long launch_count = 0;       // kernel launches issued (mark); see bfp200_last_launches
  long long graph_launches = 0;     // launches in one replay of the cached decode graph
  long long last_launches = 0;      // kernel launches of the last generate call
  // per-kernel profiling (bfp200_profile_forward): an event before every launch
  std::vector<std::pair<int, cudaEvent_t>>* prof = nullptr;

  ~bfp200_handle() {
    if (graph) cudaGraphExecDestroy(graph);       // before the communicator its NCCL node uses
    if (comm) nccl().comm_abort(comm);            // local teardown: never waits on other ranks
    if (stream) cudaStreamDestroy(stream);
  }

  size_t layer_stride_m(int G, int NT) const { return (size_t)G * NT * 512; }
  size_t layer_stride_e(int G, int NT) const { return (size_t)G * NT * 16; }
  DevMat mat(const DBuf<uint8_t>& wm, const DBuf<int8_t>& we, int G, int NT, int l) const {
    DevMat m;
    m.wm = wm.p + layer_stride_m(G, NT) * l;
    m.we = we.p + layer_stride_e(G, NT) * l;
    m.G = G;
    m.NT = NT;
    return m;
  }
  Dims dims() const { return Dims{D, HQ, HKV, HD, FFN, NL, V, MAXC}; }
  KvArena kv() const {
    KvArena k;
    k.km = km.p; k.ke = ke.p; k.vm = vm.p; k.ve = ve.p;
    k.NL = NL; k.HKV = HKV; k.HD = HD; k.MAX_CTX = MAXC;
    return k;
  }
  ColDesc cols() const {
    ColDesc c;
    c.slot = col_slot.p;
    c.pos = col_pos.p;
    return c;
  }
};

namespace {

int ensure_cols(bfp200_handle* h, int ncols) {
  if (ncols <= h->cap) return BFP200_OK;
  const int cap = std::max(ncols, 64);
  const int R_MAX = std::max({h->RQKV, 2 * h->FFN, h->D});
  CK(h->h_m.ensure((size_t)cap * h->D)); CK(h->h_e.ensure((size_t)cap * h->NTD));
  CK(h->h1_m.ensure((size_t)cap * h->D)); CK(h->h1_e.ensure((size_t)cap * h->NTD));
  CK(h->n_m.ensure((size_t)cap * h->D)); CK(h->n_e.ensure((size_t)cap * h->NTD));
  CK(h->qkv_m.ensure((size_t)cap * h->RQKV)); CK(h->qkv_e.ensure((size_t)cap * h->RQKV / 16));
  CK(h->qr_m.ensure((size_t)cap * h->QD)); CK(h->qr_e.ensure((size_t)cap * h->QD / 16));
  CK(h->a_m.ensure((size_t)cap * h->QD)); CK(h->a_e.ensure((size_t)cap * h->QD / 16));
  CK(h->mlp_m.ensure((size_t)cap * h->FFN)); CK(h->mlp_e.ensure((size_t)cap * h->NTF));
  CK(h->dbg_m.ensure((size_t)cap * R_MAX)); CK(h->dbg_e.ensure((size_t)cap * R_MAX / 16));
  CK(h->acc.ensure((size_t)R_MAX * cap));
  CK(h->counters.ensure((size_t)(R_MAX / 16) * (cap + 1)));
  const int nrb_max = std::max((h->V + 63) / 64, 2 * h->nsm);
  CK(h->hn.ensure((size_t)cap * h->D)); CK(h->hn_norm.ensure(cap));
  CK(h->part_val.ensure((size_t)cap * nrb_max)); CK(h->part_sec.ensure((size_t)cap * nrb_max));
  CK(h->part_idx.ensure((size_t)cap * nrb_max));
  CK(h->tok.ensure(cap)); CK(h->cert.ensure(cap));
  CK(h->col_slot.ensure(cap)); CK(h->col_pos.ensure(cap)); CK(h->col_kvpos.ensure(cap)); CK(h->col_tok.ensure(cap));
  CK(h->head_ctr.ensure(1));
  if (h->comm) { CK(h->xsend.ensure((size_t)cap * 4)); CK(h->xrecv.ensure((size_t)h->shard_n * cap * 4)); }
  h->cap = cap;
  if (h->graph) { cudaGraphExecDestroy(h->graph); h->graph = nullptr; h->graph_cols = -1; }
  return BFP200_OK;
}

int ensure_kv(bfp200_handle* h, int nslots) {
  const size_t per = (size_t)nslots * h->NL * h->HKV * h->MAXC;
  if (h->km.n >= per * h->HD) return BFP200_OK;
  CK(h->km.ensure(per * h->HD)); CK(h->vm.ensure(per * h->HD));
  CK(h->ke.ensure(per * (h->HD / 16))); CK(h->ve.ensure(per * (h->HD / 16)));
  if (h->graph) { cudaGraphExecDestroy(h->graph); h->graph = nullptr; h->graph_cols = -1; }
  return BFP200_OK;
}

// Kernel kinds of the per-kernel profile (bfp200_profile_forward).
enum ProfKind { PK_EMBED, PK_RMSNORM, PK_MM_QKV, PK_ROPE_KV, PK_ATTENTION, PK_MM_O, PK_MM_GU, PK_MM_D, PK_HEAD_PREP,
                PK_HEAD_LOGITS, PK_HEAD_REDUCE, PK_COUNT };

// Called before every kernel launch an enqueue_* function issues: counts the
// launch, and with profiling on, records an event in front of it.
void mark(bfp200_handle* h, int kind) {
  ++h->launch_count;
  if (!h->prof) return;
  cudaEvent_t ev;
  cudaEventCreate(&ev);
  cudaEventRecord(ev, h->stream);
  h->prof->push_back({kind, ev});
}

// The tensor-core records of a handle matrix (one layer), found from its
// DevMat pointer; nullptr for matrices the handle does not own.
const uint8_t* tc_records_of(bfp200_handle* h, const DevMat& W) {
  const DBuf<uint8_t>* wm[4] = {&h->wm_qkv, &h->wm_o, &h->wm_gu, &h->wm_d};
  const int G[4] = {h->GQKV, h->GO, h->GGU, h->GD};
  const int NT[4] = {h->NTD, h->QD / 16, h->NTD, h->NTF};
  for (int m = 0; m < 4; ++m) {
    if (!h->tc_rec[m].p || !wm[m]->p || W.G != G[m] || W.NT != NT[m]) continue;
    const size_t stride = h->layer_stride_m(G[m], NT[m]);
    if (W.wm >= wm[m]->p && W.wm < wm[m]->p + stride * h->NL) {
      const size_t off = (size_t)(W.wm - wm[m]->p);
      if (off % stride) return nullptr;
      return h->tc_rec[m].p + h->tc_stride[m] * (off / stride);
    }
  }
  return nullptr;
}

// >= tc_min_cols columns: the tcgen05 matmul (tc.cu)
bool tc_path(bfp200_handle* h, const DevMat& W, int ncols, int epi) {
  return h->use_tc && ncols >= h->tc_min_cols && tc_supported(W.NT, ncols) && !(epi == EPI_SWIGLU && W.G % 2);
}

// Times every valid (columns per CTA, epilogue warps, K split) candidate of
// one matmul call on its own arguments (the call only reads its inputs and
// writes its outputs, so repeating it is harmless) and keeps the fastest.
// The timed calls are chained the way a decode step chains its kernels
// (programmatic dependent launch when the handle uses it): what counts is
// the time from one kernel's dependency wait to the next's, not a lone
// kernel's duration.
int tc_tune(bfp200_handle* h, TcArgs t, const std::tuple<int, int, int, int>& key) {
  static const int KS[] = {1, 2, 3, 4, 6, 8};
  static const int SHAPES[][2] = {{16, 16}, {16, 8}, {32, 16}};     // (columns per CTA, epilogue warps)
  constexpr int REPS = 4;
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  float best = -1.f;
  TcChoice pick;
  for (const auto& sh : SHAPES)
    for (int ks : KS) {
      if (!tc_config_valid(t.NT, sh[0], ks)) continue;
      t.ncb = sh[0];
      t.ew = sh[1];
      t.ks = ks;
      if (launch_tc_matmul(t, h->stream, h->pdl) != cudaSuccess) { cudaGetLastError(); continue; }
      cudaEventRecord(e0, h->stream);
      bool ok = true;
      for (int r = 0; r < REPS && ok; ++r) ok = launch_tc_matmul(t, h->stream, h->pdl) == cudaSuccess;
      cudaEventRecord(e1, h->stream);
      h->launch_count += 1 + REPS;
      if (!ok) { cudaGetLastError(); continue; }
      if (cudaEventSynchronize(e1) != cudaSuccess) { cudaGetLastError(); continue; }
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      if (best < 0.f || ms < best) { best = ms; pick = {sh[0], ks, sh[1]}; }
    }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  h->tc_cfg[key] = pick;                 // {0, 0, 0}: the built-in choice
  if (const char* lg = std::getenv("BFP200_TC_LOG"); lg && *lg && *lg != '0')
    std::fprintf(stderr, "bfp200: tensor-core matmul %d x %d at %d columns (epilogue %d): %d columns per CTA, "
                 "%d epilogue warps, K split %d, %.1f us\n", t.rows, t.NT * 16, t.ncols, t.mode, pick.ncb, pick.ew,
                 pick.ks, best * 1e3f / REPS);
  return BFP200_OK;
}

int enqueue_tc(bfp200_handle* h, const uint8_t* rec, DevMat W, const int16_t* xm, const int8_t* xe, int x_ld,
               int x_lde, int ncols, int epi, int16_t* om, int8_t* oe, int o_ld, int o_lde, const int16_t* rm,
               const int8_t* re) {
  TcArgs t;
  t.rec = rec; t.we = W.we; t.rows = W.G * 16; t.NT = W.NT;
  t.xm = xm; t.xe = xe; t.x_ld = x_ld; t.x_lde = x_lde; t.ncols = ncols;
  t.mode = epi;
  t.om = om; t.oe = oe; t.o_ld = o_ld; t.o_lde = o_lde; t.rm = rm; t.re = re;
  t.err = error_flag_device_ptr();
  const auto key = std::make_tuple(t.rows, t.NT, ncols, epi);
  auto it = h->tc_cfg.find(key);
  if (it == h->tc_cfg.end()) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(h->stream, &st);
    if (st == cudaStreamCaptureStatusNone) {        // (inside a capture: the built-in choice)
      CKR(tc_tune(h, t, key));
      it = h->tc_cfg.find(key);
    }
  }
  if (it != h->tc_cfg.end()) { t.ncb = it->second.ncb; t.ks = it->second.ks; t.ew = it->second.ew; }
  CK(launch_tc_matmul(t, h->stream, h->pdl));
  return BFP200_OK;
}

int enqueue_matmul(bfp200_handle* h, DevMat W, const int16_t* xm, const int8_t* xe, int x_ld, int x_lde,
                   int ncols, int epi, int16_t* om, int8_t* oe, int o_ld, int o_lde, const int16_t* rm,
                   const int8_t* re, long long* acc, unsigned* counters, int acc_ld) {
  if (tc_path(h, W, ncols, epi)) {
    if (const uint8_t* rec = tc_records_of(h, W))
      return enqueue_tc(h, rec, W, xm, xe, x_ld, x_lde, ncols, epi, om, oe, o_ld, o_lde, rm, re);
  }
  MatmulArgs a;
  a.W = W;
  a.xm = xm; a.xe = xe; a.x_ld = x_ld; a.x_lde = x_lde;
  a.ncols = ncols;
  a.epi = epi;
  a.om = om; a.oe = oe; a.o_ld = o_ld; a.o_lde = o_lde;
  a.rm = rm; a.re = re;
  const MMPlan p = plan_matmul(W.G, W.NT, ncols, epi == EPI_SWIGLU, h->nsm, h->use_clusters ? 8 : (1 << 30));
  a.rg = p.rg; a.bn = p.bn; a.ksplit = p.ks;
  a.cluster = (p.ks > 1 && p.ks <= 8 && h->use_clusters) ? 1 : 0;
  a.acc = acc; a.counters = counters; a.acc_ld = acc_ld;
  if (p.ks > 1 && !a.cluster && (acc == nullptr || counters == nullptr))
    return fail(BFP200_EINVAL, "matmul needs K-split scratch");
  CK(launch_matmul(a, h->stream, h->pdl));
  return BFP200_OK;
}

// Stage capture for bfp200_fwd_layer (nullptr in the fast path).
struct StageSink {
  std::vector<std::vector<double>> st;  // [stage][ncols * dim]
};

int download_decoded(bfp200_handle* h, const int16_t* m, const int8_t* e, int ld, int n_per_col, int off,
                     int ncols, std::vector<double>& out) {
  // copies columns [0, ncols) elements [off, off + n_per_col) of a (m, e) buffer
  std::vector<int16_t> hm((size_t)ncols * ld);
  std::vector<int8_t> he((size_t)ncols * ld / 16);
  CK(cudaMemcpyAsync(hm.data(), m, hm.size() * 2, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaMemcpyAsync(he.data(), e, he.size(), cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  out.assign((size_t)ncols * n_per_col, 0.0);
  for (int c = 0; c < ncols; ++c)
    for (int i = 0; i < n_per_col; ++i) {
      const size_t src = (size_t)c * ld + off + i;
      out[(size_t)c * n_per_col + i] = bfp_decode(hm[src], he[src / 16]);
    }
  return BFP200_OK;
}

// first_pdl: the layer's first kernel follows one of this library's kernels
// in the stream (never a host copy), so it may use programmatic dependent
// launch.  The stage-dump path copies to the host between kernels and runs
// without PDL.
int enqueue_layer(bfp200_handle* h, int l, int ncols, StageSink* sink, bool first_pdl = true, bool early_kv = false) {
  const Dims d = h->dims();
  const bool saved_pdl = h->pdl;
  if (sink) h->pdl = false;
  struct Restore { bfp200_handle* h; bool v; ~Restore() { h->pdl = v; } } restore{h, saved_pdl};
  const bool pdl = h->pdl;
  cudaStream_t s = h->stream;
  long long* acc = h->acc.p;
  unsigned* cnt = h->counters.p;
  const int accld = h->cap;
  // n1 = tile_quantize(rmsnorm_fp(h, g1))               (:263-264)
  mark(h, PK_RMSNORM);
  CK(launch_rmsnorm(h->h_m.p, h->h_e.p, h->g1.p + (size_t)l * h->D, h->cfg.eps, h->D, ncols, h->n_m.p, h->n_e.p, s,
                    pdl && first_pdl));
  if (sink) CKR(download_decoded(h, h->n_m.p, h->n_e.p, h->D, h->D, 0, ncols, sink->st[0]));
  // q, k, v = matvec(n1, Wq|Wk|Wv)                         (:265-267)
  mark(h, PK_MM_QKV);
  CKR(enqueue_matmul(h, h->mat(h->wm_qkv, h->we_qkv, h->GQKV, h->NTD, l), h->n_m.p, h->n_e.p, h->D, h->NTD, ncols,
                     EPI_STORE, h->qkv_m.p, h->qkv_e.p, h->RQKV, h->RQKV / 16, nullptr, nullptr, acc, cnt, accld));
  if (sink) CKR(download_decoded(h, h->qkv_m.p, h->qkv_e.p, h->RQKV, h->KVD, h->QD + h->KVD, ncols, sink->st[3]));
  // rope on q, k; KV write                                (:268-272): folded into
  // the batched group attention kernel in decode steps, where every column is
  // its own sequence (a prefill's columns are positions of one sequence: their
  // attention reads K / V rows other columns write, so those rows are written
  // by a kernel of their own first) and no stage dump asks for the rotated q
  const bool rope_in_attention = early_kv && !sink && attention_group_path(d, ncols);
  if (!rope_in_attention) {
    mark(h, PK_ROPE_KV);
    CK(launch_rope_kv(h->qkv_m.p, h->qkv_e.p, h->qr_m.p, h->qr_e.p, h->kv(), l, h->cols(), h->rope_cs.p, d, ncols, s,
                      pdl));
  }
  // attention -> tile_quantize(fpq(attn))                 (:273-283)
  mark(h, PK_ATTENTION);
  CK(launch_attention(h->qr_m.p, h->qr_e.p, h->kv(), l, h->cols(), d, ncols, h->a_m.p, h->a_e.p, s, pdl,
                      h->pw_off.p, h->pw_data.p, early_kv, rope_in_attention ? h->qkv_m.p : nullptr,
                      rope_in_attention ? h->qkv_e.p : nullptr, h->rope_cs.p));
  if (sink) {
    CKR(download_decoded(h, h->qr_m.p, h->qr_e.p, h->QD, h->QD, 0, ncols, sink->st[1]));
    CKR(download_decoded(h, h->a_m.p, h->a_e.p, h->QD, h->QD, 0, ncols, sink->st[4]));
    CKR(enqueue_matmul(h, h->mat(h->wm_o, h->we_o, h->GO, h->QD / 16, l), h->a_m.p, h->a_e.p, h->QD, h->QD / 16,
                       ncols, EPI_STORE, h->dbg_m.p, h->dbg_e.p, h->D, h->NTD, nullptr, nullptr, acc, cnt, accld));
    CKR(download_decoded(h, h->dbg_m.p, h->dbg_e.p, h->D, h->D, 0, ncols, sink->st[5]));
  }
  // h1 = fpq(h + matvec(attn, Wo))                          (:284-285)
  mark(h, PK_MM_O);
  CKR(enqueue_matmul(h, h->mat(h->wm_o, h->we_o, h->GO, h->QD / 16, l), h->a_m.p, h->a_e.p, h->QD, h->QD / 16, ncols,
                     EPI_RESIDUAL, h->h1_m.p, h->h1_e.p, h->D, h->NTD, h->h_m.p, h->h_e.p, acc, cnt, accld));
  if (sink) CKR(download_decoded(h, h->h1_m.p, h->h1_e.p, h->D, h->D, 0, ncols, sink->st[6]));
  // n2 = tile_quantize(rmsnorm_fp(h1, g2))                 (:286-287)
  mark(h, PK_RMSNORM);
  CK(launch_rmsnorm(h->h1_m.p, h->h1_e.p, h->g2.p + (size_t)l * h->D, h->cfg.eps, h->D, ncols, h->n_m.p, h->n_e.p, s, pdl));
  if (sink) {
    CKR(download_decoded(h, h->n_m.p, h->n_e.p, h->D, h->D, 0, ncols, sink->st[7]));
    CKR(enqueue_matmul(h, h->mat(h->wm_gu, h->we_gu, h->GGU, h->NTD, l), h->n_m.p, h->n_e.p, h->D, h->NTD, ncols,
                       EPI_STORE, h->dbg_m.p, h->dbg_e.p, 2 * h->FFN, 2 * h->FFN / 16, nullptr, nullptr, acc, cnt,
                       accld));
    std::vector<double> gu;
    CKR(download_decoded(h, h->dbg_m.p, h->dbg_e.p, 2 * h->FFN, 2 * h->FFN, 0, ncols, gu));
    sink->st[8].assign((size_t)ncols * h->FFN, 0.0);
    sink->st[9].assign((size_t)ncols * h->FFN, 0.0);
    for (int c = 0; c < ncols; ++c)
      for (int i = 0; i < h->FFN; ++i) {
        const int grp = i / 16, r = i % 16;
        sink->st[8][(size_t)c * h->FFN + i] = gu[(size_t)c * 2 * h->FFN + (2 * grp) * 16 + r];
        sink->st[9][(size_t)c * h->FFN + i] = gu[(size_t)c * 2 * h->FFN + (2 * grp + 1) * 16 + r];
      }
  }
  // mlp = tile_quantize(fpq(silu_fp(g) * u))                (:288-291)
  mark(h, PK_MM_GU);
  CKR(enqueue_matmul(h, h->mat(h->wm_gu, h->we_gu, h->GGU, h->NTD, l), h->n_m.p, h->n_e.p, h->D, h->NTD, ncols,
                     EPI_SWIGLU, h->mlp_m.p, h->mlp_e.p, h->FFN, h->NTF, nullptr, nullptr, acc, cnt, accld));
  if (sink) {
    CKR(download_decoded(h, h->mlp_m.p, h->mlp_e.p, h->FFN, h->FFN, 0, ncols, sink->st[10]));
    CKR(enqueue_matmul(h, h->mat(h->wm_d, h->we_d, h->GD, h->NTF, l), h->mlp_m.p, h->mlp_e.p, h->FFN, h->NTF, ncols,
                       EPI_STORE, h->dbg_m.p, h->dbg_e.p, h->D, h->NTD, nullptr, nullptr, acc, cnt, accld));
    CKR(download_decoded(h, h->dbg_m.p, h->dbg_e.p, h->D, h->D, 0, ncols, sink->st[11]));
  }
  // h = fpq(h1 + matvec(mlp, Wd))                           (:292-293)
  mark(h, PK_MM_D);
  CKR(enqueue_matmul(h, h->mat(h->wm_d, h->we_d, h->GD, h->NTF, l), h->mlp_m.p, h->mlp_e.p, h->FFN, h->NTF, ncols,
                     EPI_RESIDUAL, h->h_m.p, h->h_e.p, h->D, h->NTD, h->h1_m.p, h->h1_e.p, acc, cnt, accld));
  return BFP200_OK;
}

// Small-batch layer (1..4 columns): 5 kernels -- fused RMSNorm+QKV+RoPE+KV
// write, attention, O+residual, RMSNorm+gate/up+SwiGLU, down+residual.
bool small_path_ok(bfp200_handle* h, int ncols) {
  return h->use_small && ncols >= 1 && ncols <= 4 && gemv_supported(GV_QKV_ROPE, true, h->NTD, ncols) &&
         gemv_supported(GV_RESIDUAL, false, h->QD / 16, ncols) && gemv_supported(GV_SWIGLU, true, h->NTD, ncols) &&
         gemv_supported(GV_RESIDUAL, false, h->NTF, ncols);
}

GemvArgs gemv_args(bfp200_handle* h, DevMat W, int ncols, int mode) {
  GemvArgs a;
  a.W = W;
  a.ncols = ncols;
  a.mode = mode;
  a.eps = h->cfg.eps;
  return a;
}

// Offset of stage s (n1 q k v attn o h1 n2 g u mlp d) within one column of
// the stage dump.
int stage_off(const bfp200_handle* h, int s) {
  const int len[BFP200_NSTAGES] = {h->D, h->QD, h->KVD, h->KVD, h->QD, h->D, h->D, h->D, h->FFN, h->FFN, h->FFN, h->D};
  int o = 0;
  for (int i = 0; i < s; ++i) o += len[i];
  return o;
}
int stage_stride(const bfp200_handle* h) { return stage_off(h, BFP200_NSTAGES); }

int enqueue_gemv_qkv(bfp200_handle* h, int l, int ncols, bool pdl) {
  GemvArgs a = gemv_args(h, h->mat(h->wm_qkv, h->we_qkv, h->GQKV, h->NTD, l), ncols, GV_QKV_ROPE);
  a.xm = h->h_m.p; a.xe = h->h_e.p; a.x_ld = h->D; a.x_lde = h->NTD;
  a.norm = 1; a.gamma = h->g1.p + (size_t)l * h->D;
  a.rope_cs = h->rope_cs.p; a.col_slot = h->col_slot.p; a.col_pos = h->col_pos.p;
  a.kv = h->kv(); a.layer = l; a.HQ = h->HQ; a.HKV = h->HKV;
  a.qr_m = h->qr_m.p; a.qr_e = h->qr_e.p;
  if (h->stage_dbg) {
    a.dbg_in = h->stage_dbg + stage_off(h, 0);
    a.dbg_mid = h->stage_dbg + stage_off(h, 1);     // q | k | v rows are consecutive stages
    a.dbg_ld = h->stage_ld;
  }
  CK(launch_gemv(a, h->stream, pdl));
  return BFP200_OK;
}

int enqueue_gemv_o(bfp200_handle* h, int l, int ncols, bool pdl, int16_t* om, int8_t* oe) {
  GemvArgs a = gemv_args(h, h->mat(h->wm_o, h->we_o, h->GO, h->QD / 16, l), ncols, GV_RESIDUAL);
  a.layer = l;
  a.xm = h->a_m.p; a.xe = h->a_e.p; a.x_ld = h->QD; a.x_lde = h->QD / 16;
  a.rm = h->h_m.p; a.re = h->h_e.p;
  a.om = om; a.oe = oe; a.o_ld = h->D; a.o_lde = h->NTD;
  if (h->stage_dbg) { a.dbg_mid = h->stage_dbg + stage_off(h, 5); a.dbg_ld = h->stage_ld; }
  CK(launch_gemv(a, h->stream, pdl));
  return BFP200_OK;
}

int enqueue_gemv_gu(bfp200_handle* h, int l, int ncols, bool pdl) {
  GemvArgs a = gemv_args(h, h->mat(h->wm_gu, h->we_gu, h->GGU, h->NTD, l), ncols, GV_SWIGLU);
  a.layer = l;
  a.xm = h->h1_m.p; a.xe = h->h1_e.p; a.x_ld = h->D; a.x_lde = h->NTD;
  a.norm = 1; a.gamma = h->g2.p + (size_t)l * h->D;
  a.om = h->mlp_m.p; a.oe = h->mlp_e.p; a.o_ld = h->FFN; a.o_lde = h->NTF;
  if (h->stage_dbg) {
    a.dbg_in = h->stage_dbg + stage_off(h, 7);
    a.dbg_mid = h->stage_dbg + stage_off(h, 8);
    a.dbg_mid2 = h->stage_dbg + stage_off(h, 9);
    a.dbg_ld = h->stage_ld;
  }
  CK(launch_gemv(a, h->stream, pdl));
  return BFP200_OK;
}

int enqueue_gemv_d(bfp200_handle* h, int l, int ncols, bool pdl, int16_t* om, int8_t* oe) {
  GemvArgs a = gemv_args(h, h->mat(h->wm_d, h->we_d, h->GD, h->NTF, l), ncols, GV_RESIDUAL);
  a.layer = l;
  a.xm = h->mlp_m.p; a.xe = h->mlp_e.p; a.x_ld = h->FFN; a.x_lde = h->NTF;
  a.rm = h->h1_m.p; a.re = h->h1_e.p;
  a.om = om; a.oe = oe; a.o_ld = h->D; a.o_lde = h->NTD;
  if (h->stage_dbg) { a.dbg_mid = h->stage_dbg + stage_off(h, 11); a.dbg_ld = h->stage_ld; }
  CK(launch_gemv(a, h->stream, pdl));
  return BFP200_OK;
}

// One column: RMSNorm + Q/K/V + RoPE + KV write + attention + O + residual
// in one cluster launch (h -> h1).
int enqueue_attn_block(bfp200_handle* h, int l, bool pdl) {
  L1Args a = h->block;
  a.Wqkv = h->mat(h->wm_qkv, h->we_qkv, h->GQKV, h->NTD, l);
  a.Wo = h->mat(h->wm_o, h->we_o, h->GO, h->QD / 16, l);
  a.gamma = h->g1.p + (size_t)l * h->D;
  a.eps = h->cfg.eps;
  a.hm = h->h_m.p; a.he = h->h_e.p;
  a.h1m = h->h1_m.p; a.h1e = h->h1_e.p;
  a.rope_cs = h->rope_cs.p;
  a.col_slot = h->col_slot.p; a.col_pos = h->col_pos.p;
  a.kv = h->kv();
  a.layer = l;
  a.pw_off = h->pw_off.p; a.pw_data = h->pw_data.p;
  a.err = error_flag_device_ptr();
  a.sqrt_hd = std::sqrt((double)h->HD);
  int ex = 0;
  a.inv_hd = std::frexp(a.sqrt_hd, &ex) == 0.5 ? std::ldexp(1.0, 1 - ex) : 0.0;
  a.dbg = h->stage_dbg;                               // column 0: stages n1 .. h1
  CK(launch_attn_block(a, h->stream, pdl));
  return BFP200_OK;
}

bool attn_block_ok(bfp200_handle* h, int ncols) { return ncols == 1 && h->use_block && h->block_ok; }

int enqueue_layer_small(bfp200_handle* h, int l, int ncols, bool first_pdl, bool early_kv) {
  const bool pdl = h->pdl;
  if (attn_block_ok(h, ncols)) {
    mark(h, PK_ATTENTION);
    CKR(enqueue_attn_block(h, l, pdl && first_pdl));
#ifdef BFP200_DOUBLE_BLOCK
    CKR(enqueue_attn_block(h, l, pdl));   // measurement builds: the same launch again, with warm code
#endif
    mark(h, PK_MM_GU);
    CKR(enqueue_gemv_gu(h, l, ncols, pdl));
    mark(h, PK_MM_D);
    CKR(enqueue_gemv_d(h, l, ncols, pdl, h->h_m.p, h->h_e.p));
    return BFP200_OK;
  }
  mark(h, PK_MM_QKV);
  CKR(enqueue_gemv_qkv(h, l, ncols, pdl && first_pdl));
  mark(h, PK_ATTENTION);
  CK(launch_attention(h->qr_m.p, h->qr_e.p, h->kv(), l, h->cols(), h->dims(), ncols, h->a_m.p, h->a_e.p, h->stream,
                      pdl, h->pw_off.p, h->pw_data.p, early_kv));
  mark(h, PK_MM_O);
  CKR(enqueue_gemv_o(h, l, ncols, pdl, h->h1_m.p, h->h1_e.p));
  mark(h, PK_MM_GU);
  CKR(enqueue_gemv_gu(h, l, ncols, pdl));
  mark(h, PK_MM_D);
  CKR(enqueue_gemv_d(h, l, ncols, pdl, h->h_m.p, h->h_e.p));
  return BFP200_OK;
}

// Vocabulary-sharded head: this rank's rows give one (best, index,
// runner-up, ||hn||) record per column, the ranks all-gather the records and
// every rank combines them into the token (lowest index on ties).
int enqueue_head_sharded(bfp200_handle* h, int ncols) {
  cudaStream_t s = h->stream;
  const int NT = h->D / 16, nv = h->v_hi - h->v_lo;
  const int16_t* em = h->emb_m.p + (size_t)h->v_lo * h->D;
  const int8_t* ee = h->emb_e.p + (size_t)h->v_lo * NT;
  mark(h, PK_HEAD_LOGITS);
  if (h->use_small && head_small_supported(ncols, h->D)) {
    CK(launch_head_small(h->h_m.p, h->h_e.p, h->nw.p, h->cfg.eps, em, ee, nv, h->D, ncols, h->emb_norm_max,
                         h->part_val.p, h->part_idx.p, h->part_sec.p, h->head_ctr.p, h->tok.p, h->cert.p, s, h->pdl,
                         h->v_lo, h->xsend.p));
  } else {
    CK(launch_head_prep(h->h_m.p, h->h_e.p, h->nw.p, h->cfg.eps, h->D, ncols, h->hn.p, h->hn_norm.p, s, h->pdl));
    ++h->launch_count;
    int nrb = 0;
    CK(launch_head_logits(em, ee, nv, h->D, h->hn.p, ncols, h->part_val.p, h->part_idx.p, h->part_sec.p, &nrb, s,
                          h->pdl));
    ++h->launch_count;
    CK(launch_head_reduce(h->part_val.p, h->part_idx.p, h->part_sec.p, nrb, h->hn_norm.p, h->emb_norm_max, h->D,
                          ncols, h->tok.p, h->cert.p, s, h->pdl, h->v_lo, h->xsend.p));
  }
  const int r = nccl().all_gather(h->xsend.p, h->xrecv.p, (size_t)ncols * 4, NCCL_F64, h->comm, s);
  if (r != NCCL_OK && r != NCCL_IN_PROGRESS) return fail(BFP200_ECUDA, "ncclAllGather: " + nccl_err(r));
  mark(h, PK_HEAD_REDUCE);
  CK(launch_head_combine(h->xrecv.p, h->shard_n, ncols, h->emb_norm_max, h->D, h->V, h->tok.p, h->cert.p, s));
  return BFP200_OK;
}

int enqueue_head(bfp200_handle* h, int ncols) {
  cudaStream_t s = h->stream;
  if (h->comm) return enqueue_head_sharded(h, ncols);
  if (h->use_small && head_small_supported(ncols, h->D)) {
    // one launch: hn, logits, certified argmax (last CTA); head_ctr is
    // allocated by ensure_cols, outside any stream capture
    mark(h, PK_HEAD_LOGITS);
    CK(launch_head_small(h->h_m.p, h->h_e.p, h->nw.p, h->cfg.eps, h->emb_m.p, h->emb_e.p, h->V, h->D, ncols,
                         h->emb_norm_max, h->part_val.p, h->part_idx.p, h->part_sec.p, h->head_ctr.p, h->tok.p,
                         h->cert.p, s, h->pdl, 0, nullptr, h->head_adv));
    return BFP200_OK;
  }
  mark(h, PK_HEAD_PREP);
  CK(launch_head_prep(h->h_m.p, h->h_e.p, h->nw.p, h->cfg.eps, h->D, ncols, h->hn.p, h->hn_norm.p, s, h->pdl));
  int nrb = 0;
  mark(h, PK_HEAD_LOGITS);
  CK(launch_head_logits(h->emb_m.p, h->emb_e.p, h->V, h->D, h->hn.p, ncols, h->part_val.p, h->part_idx.p,
                        h->part_sec.p, &nrb, s, h->pdl));
  mark(h, PK_HEAD_REDUCE);
  CK(launch_head_reduce(h->part_val.p, h->part_idx.p, h->part_sec.p, nrb, h->hn_norm.p, h->emb_norm_max, h->D, ncols,
                        h->tok.p, h->cert.p, s, h->pdl));
  return BFP200_OK;
}

// The four matmuls of layer l at ncols columns on the handle's scratch
// activations (measurement, and choosing tensor-core configurations before
// a graph capture): their outputs are overwritten by any later forward.
int enqueue_layer_matmuls(bfp200_handle* h, int l, int ncols) {
  long long* acc = h->acc.p;
  unsigned* cnt = h->counters.p;
  const int accld = h->cap;
  CKR(enqueue_matmul(h, h->mat(h->wm_qkv, h->we_qkv, h->GQKV, h->NTD, l), h->n_m.p, h->n_e.p, h->D, h->NTD, ncols,
                     EPI_STORE, h->qkv_m.p, h->qkv_e.p, h->RQKV, h->RQKV / 16, nullptr, nullptr, acc, cnt, accld));
  CKR(enqueue_matmul(h, h->mat(h->wm_o, h->we_o, h->GO, h->QD / 16, l), h->a_m.p, h->a_e.p, h->QD, h->QD / 16,
                     ncols, EPI_RESIDUAL, h->h1_m.p, h->h1_e.p, h->D, h->NTD, h->h_m.p, h->h_e.p, acc, cnt, accld));
  CKR(enqueue_matmul(h, h->mat(h->wm_gu, h->we_gu, h->GGU, h->NTD, l), h->n_m.p, h->n_e.p, h->D, h->NTD, ncols,
                     EPI_SWIGLU, h->mlp_m.p, h->mlp_e.p, h->FFN, h->NTF, nullptr, nullptr, acc, cnt, accld));
  CKR(enqueue_matmul(h, h->mat(h->wm_d, h->we_d, h->GD, h->NTF, l), h->mlp_m.p, h->mlp_e.p, h->FFN, h->NTF, ncols,
                     EPI_RESIDUAL, h->dbg_m.p, h->dbg_e.p, h->D, h->NTD, h->h1_m.p, h->h1_e.p, acc, cnt, accld));
  return BFP200_OK;
}

struct Sampling {
  double temperature = 0.0;
  int top_k = 0;
  uint32_t seed = 0;
};

// Sampled head: hn, the full fp64 logits of every column, then one sampling
// CTA per column (uniforms indexed by the device step counter).
int enqueue_sample_head(bfp200_handle* h, int ncols, const Sampling& smp, int u_ld) {
  cudaStream_t s = h->stream;
  mark(h, PK_HEAD_PREP);
  CK(launch_head_prep(h->h_m.p, h->h_e.p, h->nw.p, h->cfg.eps, h->D, ncols, h->hn.p, h->hn_norm.p, s, h->pdl));
  int nrb = 0;
  mark(h, PK_HEAD_LOGITS);
  CK(launch_head_logits(h->emb_m.p, h->emb_e.p, h->V, h->D, h->hn.p, ncols, h->part_val.p, h->part_idx.p,
                        h->part_sec.p, &nrb, s, h->pdl, h->s_logits.p));
  SampleArgs a;
  a.logits = h->s_logits.p; a.ld = h->V; a.V = h->V; a.D = h->D;
  a.temperature = smp.temperature; a.top_k = smp.top_k;
  a.work = h->s_work.p; a.cdf = h->s_cdf.p; a.incl = h->s_incl.p;
  a.plan = h->v_plan.p;
  a.uniforms = h->s_uni.p; a.u_ld = u_ld; a.step = h->dec_step.p;
  a.hn_norm = h->hn_norm.p; a.emb_norm_max = h->emb_norm_max;
  a.tok = h->tok.p; a.cert = h->cert.p;
  mark(h, PK_HEAD_REDUCE);
  CK(launch_sample(a, ncols, h->v_plan_leaves, s));
  return BFP200_OK;
}

// The embedding kernel is the first kernel after host copies of the column
// descriptors (prefill) or after the non-PDL advance kernel (decode graph):
// it is launched without programmatic dependent launch.
int enqueue_forward(bfp200_handle* h, int ncols, bool head, bool decode = false) {
  mark(h, PK_EMBED);
  CK(launch_embed(h->emb_m.p, h->emb_e.p, h->col_tok.p, h->D, ncols, h->h_m.p, h->h_e.p, h->stream, false));
  const bool small = small_path_ok(h, ncols);
  for (int l = 0; l < h->NL; ++l) {
    if (small) CKR(enqueue_layer_small(h, l, ncols, /*first_pdl=*/true, decode));
    else CKR(enqueue_layer(h, l, ncols, nullptr, true, decode));
  }
  if (head) CKR(enqueue_head(h, ncols));
  return BFP200_OK;
}

// Leaves any sharding (destroys the decode graph first: it holds the
// communicator's all-gather) and joins `comm` as rank `rank` of `n`.
// Polls the handle's stream until it is idle or `limit_s` seconds passed;
// false on timeout (never blocks longer).
bool bounded_drain(bfp200_handle* h, double limit_s) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(h->stream);
    if (e != cudaErrorNotReady) return e == cudaSuccess;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > limit_s) return false;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int set_shard(bfp200_handle* h, NcclComm comm, int n, int rank) {
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  if (h->broken) return fail(BFP200_ESTATE, "handle unusable: an aborted exchange never left its stream");
  if (!bounded_drain(h, 30.0)) {
    h->broken = true;
    return fail(BFP200_ETIMEOUT, "head_shard: the handle's stream did not drain (an exchange is stuck)");
  }
  if (h->graph) { cudaGraphExecDestroy(h->graph); h->graph = nullptr; h->graph_cols = -1; }
  // local teardown (ncclCommAbort frees the communicator without waiting on
  // the other ranks; every exchange of this handle has completed or timed out)
  if (h->comm) { nccl().comm_abort(h->comm); h->comm = nullptr; }
  h->comm = comm;
  h->shard_n = comm ? n : 1;
  h->shard_rank = comm ? rank : 0;
  h->v_lo = (int)((long long)h->shard_rank * h->V / h->shard_n);
  h->v_hi = (int)((long long)(h->shard_rank + 1) * h->V / h->shard_n);
  if (comm && h->cap > 0) {
    CK(h->xsend.ensure((size_t)h->cap * 4));
    CK(h->xrecv.ensure((size_t)h->shard_n * h->cap * 4));
  }
  if (comm) CK(h->xwarm.ensure((size_t)(h->shard_n + 1) * 4));
  return BFP200_OK;
}

// One all-gather on a freshly joined communicator (every rank makes it at
// the same point), outside any graph capture, waited for with the bounded
// poll: the exchange path is exercised once before decode graphs hold it.
int enqueue_warm_exchange(bfp200_handle* h) {
  const int r = nccl().all_gather(h->xwarm.p, h->xwarm.p + 4, 4, NCCL_F64, h->comm, h->stream);
  if (r != NCCL_OK && r != NCCL_IN_PROGRESS) return fail(BFP200_ECUDA, "ncclAllGather: " + nccl_err(r));
  return BFP200_OK;
}

// Waits for the handle's stream.  With a sharded head the wait is bounded:
// a rank that never joins the exchange (or an NCCL error) aborts the
// communicator, which ends the waiting NCCL kernel, and the handle leaves
// sharding.
int sync_stream(bfp200_handle* h) {
  if (!h->comm) { CK(cudaStreamSynchronize(h->stream)); return BFP200_OK; }
  double limit_s = 120.0;
  if (const char* e = std::getenv("BFP200_NCCL_TIMEOUT_S")) limit_s = std::max(0.1, std::atof(e));
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(h->stream);
    if (e == cudaSuccess) return BFP200_OK;
    if (e != cudaErrorNotReady) return fail(BFP200_ECUDA, std::string("CUDA: ") + cudaGetErrorString(e));
    int ae = NCCL_OK;
    nccl().async_error(h->comm, &ae);
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if ((ae != NCCL_OK && ae != NCCL_IN_PROGRESS) || el > limit_s) {
      const std::string why = ae != NCCL_OK && ae != NCCL_IN_PROGRESS
                                  ? "sharded head: NCCL error " + nccl_err(ae)
                                  : "sharded head: the exchange did not complete (a rank is missing)";
      // the abort ends the waiting NCCL kernel; at most one decode step is
      // ever queued behind it while sharded, so nothing else on the stream
      // uses the freed communicator.  The drain is bounded as well: if the
      // stream still does not empty, the handle is marked unusable instead
      // of blocking the caller.
      nccl().comm_abort(h->comm);
      h->comm = nullptr;
      if (!bounded_drain(h, 30.0)) {
        h->broken = true;
        return fail(BFP200_ETIMEOUT, why + "; the stream did not drain after the abort (handle unusable)");
      }
      set_shard(h, nullptr, 1, 0);
      return fail(BFP200_ETIMEOUT, why);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// host <-> device staging of the op-level entry points
template <typename T>
int upload(DBuf<T>& d, const T* host, size_t n, cudaStream_t s) {
  CK(d.ensure(n ? n : 1));
  if (n) CK(cudaMemcpyAsync(d.p, host, n * sizeof(T), cudaMemcpyHostToDevice, s));
  return BFP200_OK;
}
template <typename T>
int download(T* host, const DBuf<T>& d, size_t n, cudaStream_t s) {
  if (n) CK(cudaMemcpyAsync(host, d.p, n * sizeof(T), cudaMemcpyDeviceToHost, s));
  return BFP200_OK;
}

int check_cfg(const bfp200_cfg& c) {
  if (c.D <= 0 || c.D % 16 || c.FFN <= 0 || c.FFN % 16 || c.H_Q <= 0 || c.H_KV <= 0 || c.H_Q % c.H_KV ||
      c.HD != 64 || c.H_Q * c.HD != c.D || c.NL <= 0 || c.VOCAB <= 0 || c.VOCAB % 16 || c.MAX_CTX <= 0 ||
      c.MAX_CTX > 3072 || c.NPROMPT_MAX <= 0 || c.max_seqs <= 0 || c.D > 8192)
    return fail(BFP200_EINVAL,
                "unsupported config (need HD=64, H_Q*HD=D, D/FFN/VOCAB multiples of 16, H_Q % H_KV == 0, "
                "MAX_CTX <= 3072)");
  return BFP200_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

void bfp200_default_cfg(bfp200_cfg* c) {
  c->D = 576; c->H_Q = 9; c->H_KV = 3; c->HD = 64; c->FFN = 1536; c->NL = 30; c->VOCAB = 49152;
  c->MAX_CTX = 64; c->NPROMPT_MAX = 48; c->max_seqs = 1;
  c->rope_base = 10000.0;
  c->eps = 1e-5;
}

int bfp200_last_error(char* buf, size_t len) {
  if (buf && len) {
    std::strncpy(buf, g_err.c_str(), len - 1);
    buf[len - 1] = 0;
  }
  return BFP200_OK;
}

int bfp200_rope_table(double* out, int n_pos, int HD, double base) {
  if (!out || n_pos < 0 || HD <= 0 || HD % 2) return fail(BFP200_EINVAL, "rope_table: bad arguments");
  const int H2 = HD / 2;
  for (int p = 0; p < n_pos; ++p)
    for (int j = 0; j < H2; ++j) {
      // theta = 1.0 / (base ** (2*j/HD)) * pos   (gen_smollm_blockfp_full.py:253)
      const double expo = (double)(2 * j) / (double)HD;
      const double pw = (expo == 0.0) ? 1.0 : std::pow(base, expo);
      const double theta = 1.0 / pw * (double)p;
      out[((size_t)p * H2 + j) * 2 + 0] = std::cos(theta);
      out[((size_t)p * H2 + j) * 2 + 1] = std::sin(theta);
    }
  return BFP200_OK;
}

int bfp200_open(const bfp200_cfg* cfg, int device, bfp200_handle** out) {
  if (!cfg || !out) return fail(BFP200_EINVAL, "open: null argument");
  CKR(check_cfg(*cfg));
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) return fail(BFP200_ENODEV, "no CUDA device");
  if (device < 0 || device >= ndev) return fail(BFP200_ENODEV, "device index out of range");
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return fail(BFP200_ENODEV, "libbfp200 is built for sm_100a (B200); device is sm_" +
                                                       std::to_string(prop.major) + std::to_string(prop.minor));
  DeviceGuard dguard(device);
  CK(dguard.err);
  CK(init_kernel_attributes());
  auto* h = new bfp200_handle();
  h->cfg = *cfg;
  h->device = device;
  h->nsm = prop.multiProcessorCount;
  h->D = cfg->D; h->HQ = cfg->H_Q; h->HKV = cfg->H_KV; h->HD = cfg->HD; h->FFN = cfg->FFN; h->NL = cfg->NL;
  h->V = cfg->VOCAB; h->MAXC = cfg->MAX_CTX;
  h->v_lo = 0; h->v_hi = h->V;
  h->NTD = h->D / 16; h->NTF = h->FFN / 16; h->KVD = h->HKV * h->HD; h->QD = h->HQ * h->HD;
  h->RQKV = h->QD + 2 * h->KVD;
  h->GQKV = h->RQKV / 16; h->GO = h->D / 16; h->GGU = 2 * h->FFN / 16; h->GD = h->D / 16;
  if (const char* e = std::getenv("BFP200_NO_PDL")) h->pdl = !(e[0] == '1');
  if (const char* e = std::getenv("BFP200_NO_CLUSTER")) h->use_clusters = !(e[0] == '1');
  if (const char* e = std::getenv("BFP200_NO_SMALL")) h->use_small = !(e[0] == '1');
  if (const char* e = std::getenv("BFP200_NO_TC")) h->use_tc = !(e[0] == '1');
  if (const char* e = std::getenv("BFP200_TC_MIN_COLS")) h->tc_min_cols = std::max(1, std::atoi(e));
  if (const char* e = std::getenv("BFP200_NO_BLOCK")) h->use_block = !(e[0] == '1');
  h->smem_optin = (int)prop.sharedMemPerBlockOptin;
  {
    int budget = 0;
    const cudaError_t be = init_attn_block_attributes(h->smem_optin, &budget);
    if (be != cudaSuccess) { delete h; return fail(BFP200_ECUDA, std::string("open: ") + cudaGetErrorString(be)); }
    L1Args& b = h->block;
    b.D = h->D; b.HQ = h->HQ; b.HKV = h->HKV;
    b.kv.MAX_CTX = h->MAXC;
    h->block_ok = h->HD == 64 && attn_block_plan(b, budget);
  }
  cudaError_t ce = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking);
  if (ce != cudaSuccess) { delete h; return fail(BFP200_ECUDA, cudaGetErrorString(ce)); }
  std::vector<double> cs((size_t)h->MAXC * h->HD);
  bfp200_rope_table(cs.data(), h->MAXC, h->HD, cfg->rope_base);
  if (h->rope_cs.ensure(cs.size()) != cudaSuccess ||
      cudaMemcpyAsync(h->rope_cs.p, cs.data(), cs.size() * 8, cudaMemcpyHostToDevice, h->stream) != cudaSuccess ||
      cudaStreamSynchronize(h->stream) != cudaSuccess) {
    delete h;
    return fail(BFP200_ENOMEM, "open: rope table allocation failed");
  }
  {
    std::vector<int> offs(h->MAXC + 1, 0);
    std::vector<unsigned short> data;
    for (int n = 1; n <= h->MAXC; ++n) {
      offs[n] = (int)data.size();
      build_pw_plan_one(n, data);
    }
    if (h->pw_off.ensure(offs.size()) != cudaSuccess || h->pw_data.ensure(data.size()) != cudaSuccess ||
        cudaMemcpyAsync(h->pw_off.p, offs.data(), offs.size() * 4, cudaMemcpyHostToDevice, h->stream) != cudaSuccess ||
        cudaMemcpyAsync(h->pw_data.p, data.data(), data.size() * 2, cudaMemcpyHostToDevice, h->stream) != cudaSuccess ||
        cudaStreamSynchronize(h->stream) != cudaSuccess) {
      delete h;
      return fail(BFP200_ENOMEM, "open: pairwise-sum plan allocation failed");
    }
  }
  *out = h;
  return BFP200_OK;
}

int bfp200_close(bfp200_handle* h) {
  if (!h) return BFP200_OK;
  DeviceGuard dguard(h->device);
  cudaStreamSynchronize(h->stream);
  delete h;
  return BFP200_OK;
}

static void decode_vec(const int16_t* m, const int8_t* e, size_t n, double* out) {
  for (size_t i = 0; i < n; ++i) out[i] = bfp_decode(m[i], e[i / 16]);
}

static int upload_gammas(bfp200_handle* h) {
  std::vector<double> g1(h->g1m.size()), g2(h->g2m.size()), nw(h->nwm.size());
  decode_vec(h->g1m.data(), h->g1e.data(), g1.size(), g1.data());
  decode_vec(h->g2m.data(), h->g2e.data(), g2.size(), g2.data());
  decode_vec(h->nwm.data(), h->nwe.data(), nw.size(), nw.data());
  CK(h->g1.ensure(g1.size())); CK(h->g2.ensure(g2.size())); CK(h->nw.ensure(nw.size()));
  CK(cudaMemcpyAsync(h->g1.p, g1.data(), g1.size() * 8, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(h->g2.p, g2.data(), g2.size() * 8, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(h->nw.p, nw.data(), nw.size() * 8, cudaMemcpyHostToDevice, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_load_image(bfp200_handle* h, const void* img, size_t len) {
  if (!h || !img) return fail(BFP200_EINVAL, "load_image: null argument");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  const auto rs = image_regions(h->cfg);
  const size_t total = find_region(rs, "END")->off;
  if (len != total)
    return fail(BFP200_EIMAGE, "image is " + std::to_string(len) + " bytes; this config needs " + std::to_string(total));
  const uint8_t* b = static_cast<const uint8_t*>(img);
  // weights: raw image to the device, then repacked per matrix
  DBuf<uint8_t> staging;
  const size_t wbytes = find_region(rs, "G1_m")->off;
  CK(staging.ensure(wbytes));
  CK(cudaMemcpyAsync(staging.p, b, wbytes, cudaMemcpyHostToDevice, h->stream));
  CK(h->wm_qkv.ensure((size_t)h->NL * h->GQKV * h->NTD * 512)); CK(h->we_qkv.ensure((size_t)h->NL * h->GQKV * h->NTD * 16));
  CK(h->wm_o.ensure((size_t)h->NL * h->GO * (h->QD / 16) * 512)); CK(h->we_o.ensure((size_t)h->NL * h->GO * (h->QD / 16) * 16));
  CK(h->wm_gu.ensure((size_t)h->NL * h->GGU * h->NTD * 512)); CK(h->we_gu.ensure((size_t)h->NL * h->GGU * h->NTD * 16));
  CK(h->wm_d.ensure((size_t)h->NL * h->GD * h->NTF * 512)); CK(h->we_d.ensure((size_t)h->NL * h->GD * h->NTF * 16));
  struct Spec { const char* tag; int dout, din; DBuf<uint8_t>* wm; DBuf<int8_t>* we; int Gtot, gstride, goff; };
  const Spec specs[] = {
      {"WQ", h->QD, h->D, &h->wm_qkv, &h->we_qkv, h->GQKV, 1, 0},
      {"WK", h->KVD, h->D, &h->wm_qkv, &h->we_qkv, h->GQKV, 1, h->QD / 16},
      {"WV", h->KVD, h->D, &h->wm_qkv, &h->we_qkv, h->GQKV, 1, (h->QD + h->KVD) / 16},
      {"WO", h->D, h->QD, &h->wm_o, &h->we_o, h->GO, 1, 0},
      {"WG", h->FFN, h->D, &h->wm_gu, &h->we_gu, h->GGU, 2, 0},
      {"WU", h->FFN, h->D, &h->wm_gu, &h->we_gu, h->GGU, 2, 1},
      {"WDN", h->D, h->FFN, &h->wm_d, &h->we_d, h->GD, 1, 0}};
  for (const auto& sp : specs) {
    const Region* rm = find_region(rs, std::string(sp.tag) + "_m");
    const Region* re = find_region(rs, std::string(sp.tag) + "_e");
    const int G = sp.dout / 16, NT = sp.din / 16;
    const size_t lm = (size_t)G * sp.din * 32, le = (size_t)G * NT * 16;
    for (int l = 0; l < h->NL; ++l) {
      CK(launch_pack_from_ddr(reinterpret_cast<const int16_t*>(staging.p + rm->off + l * lm),
                              reinterpret_cast<const int8_t*>(staging.p + re->off + l * le), sp.dout, NT,
                              sp.wm->p + (size_t)l * sp.Gtot * NT * 512, sp.we->p + (size_t)l * sp.Gtot * NT * 16,
                              sp.gstride, sp.goff, h->stream));
    }
  }
  // gammas and final norm (host copies kept for load_rom)
  auto take16 = [&](const char* nm, size_t n, std::vector<int16_t>& v) {
    v.resize(n);
    std::memcpy(v.data(), b + find_region(rs, nm)->off, n * 2);
  };
  auto take8 = [&](const char* nm, size_t n, std::vector<int8_t>& v) {
    v.resize(n);
    std::memcpy(v.data(), b + find_region(rs, nm)->off, n);
  };
  take16("G1_m", (size_t)h->NL * h->D, h->g1m); take8("G1_e", (size_t)h->NL * h->NTD, h->g1e);
  take16("G2_m", (size_t)h->NL * h->D, h->g2m); take8("G2_e", (size_t)h->NL * h->NTD, h->g2e);
  take16("NORM_W_m", h->D, h->nwm); take8("NORM_W_e", h->NTD, h->nwe);
  CKR(upload_gammas(h));
  // embedding table: row-major mantissas (EMBED_LU_m) and per-row exponents
  // (EMBED_LU_e, rows padded to 64 B); the head reads the same rows.
  CK(h->emb_m.ensure((size_t)h->V * h->D));
  CK(cudaMemcpyAsync(h->emb_m.p, b + find_region(rs, "EMBED_LU_m")->off, (size_t)h->V * h->D * 2,
                     cudaMemcpyHostToDevice, h->stream));
  std::vector<int8_t> ee((size_t)h->V * h->NTD);
  const uint8_t* lue = b + find_region(rs, "EMBED_LU_e")->off;
  for (int r = 0; r < h->V; ++r) std::memcpy(ee.data() + (size_t)r * h->NTD, lue + (size_t)r * 64, h->NTD);
  CK(h->emb_e.ensure(ee.size()));
  CK(cudaMemcpyAsync(h->emb_e.p, ee.data(), ee.size(), cudaMemcpyHostToDevice, h->stream));
  CK(h->emb_norm.ensure(h->V));
  CK(launch_row_norms(h->emb_m.p, h->emb_e.p, h->V, h->D, h->emb_norm.p, h->stream));
  std::vector<double> norms(h->V);
  CK(cudaMemcpyAsync(norms.data(), h->emb_norm.p, h->V * 8, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  h->emb_norm_max = *std::max_element(norms.begin(), norms.end());
  // tensor-core records for the batched path
  {
    const DBuf<uint8_t>* wm[4] = {&h->wm_qkv, &h->wm_o, &h->wm_gu, &h->wm_d};
    const DBuf<int8_t>* we[4] = {&h->we_qkv, &h->we_o, &h->we_gu, &h->we_d};
    const int G[4] = {h->GQKV, h->GO, h->GGU, h->GD};
    const int NT[4] = {h->NTD, h->QD / 16, h->NTD, h->NTF};
    for (int m = 0; m < 4; ++m) {
      h->tc_stride[m] = tc_records_bytes(G[m] * 16, NT[m]);
      CK(h->tc_rec[m].ensure(h->tc_stride[m] * h->NL));
      for (int l = 0; l < h->NL; ++l) {
        const DevMat W = h->mat(*wm[m], *we[m], G[m], NT[m], l);
        CK(launch_tc_pack(W.wm, W.we, G[m] * 16, NT[m], h->tc_rec[m].p + h->tc_stride[m] * l, h->stream));
      }
    }
    CK(cudaStreamSynchronize(h->stream));
  }
  h->have_image = true;
  return BFP200_OK;
}

int bfp200_load_rom(bfp200_handle* h, int kind, const uint16_t* entries, size_t n) {
  if (!h || (!entries && n)) return fail(BFP200_EINVAL, "load_rom: null argument");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  const size_t nld = (size_t)h->NL * h->D, nlt = (size_t)h->NL * h->NTD;
  auto put16 = [&](std::vector<int16_t>& v, size_t want) -> int {
    if (n != want) return fail(BFP200_EIMAGE, "load_rom kind " + std::to_string(kind) + ": " + std::to_string(n) +
                                                  " entries, expected " + std::to_string(want));
    v.resize(n);
    for (size_t i = 0; i < n; ++i) v[i] = (int16_t)entries[i];
    return BFP200_OK;
  };
  auto put8 = [&](std::vector<int8_t>& v, size_t want) -> int {
    if (n != want) return fail(BFP200_EIMAGE, "load_rom kind " + std::to_string(kind) + ": " + std::to_string(n) +
                                                  " entries, expected " + std::to_string(want));
    v.resize(n);
    for (size_t i = 0; i < n; ++i) v[i] = (int8_t)(entries[i] & 0xFF);
    return BFP200_OK;
  };
  switch (kind) {
    case 0: CKR(put16(h->g1m, nld)); break;
    case 1: CKR(put8(h->g1e, nlt)); break;
    case 2: CKR(put16(h->g2m, nld)); break;
    case 3: CKR(put8(h->g2e, nlt)); break;
    case 4: CKR(put16(h->nwm, h->D)); break;
    case 5: CKR(put8(h->nwe, h->NTD)); break;
    case 6:
      if (n == 0 || n > (size_t)h->cfg.NPROMPT_MAX)
        return fail(BFP200_EINVAL, "prompt ROM length must be 1..NPROMPT_MAX");
      h->rom_prompt.assign(entries, entries + n);
      return BFP200_OK;
    default: return fail(BFP200_EINVAL, "load_rom: kind must be 0..6");
  }
  if (h->g1m.size() == nld && h->g1e.size() == nlt && h->g2m.size() == nld && h->g2e.size() == nlt &&
      h->nwm.size() == (size_t)h->D && h->nwe.size() == (size_t)h->NTD)
    CKR(upload_gammas(h));
  return BFP200_OK;
}

static int generate_impl(bfp200_handle* h, const int32_t* prompt_ids, const int32_t* prompt_lens, int n_seq,
                         int n_gen, int feed_mode, int32_t* out_tokens, const Sampling* smp);

int bfp200_generate(bfp200_handle* h, const int32_t* prompt_ids, const int32_t* prompt_lens, int n_seq, int n_gen,
                    int feed_mode, int32_t* out_tokens) {
  return generate_impl(h, prompt_ids, prompt_lens, n_seq, n_gen, feed_mode, out_tokens, nullptr);
}

int bfp200_sample_uniforms(uint32_t seed, int n, double* out) {
  if (n < 0 || (n > 0 && !out)) return fail(BFP200_EINVAL, "sample_uniforms: bad arguments");
  mt19937_uniforms(seed, n, out);
  return BFP200_OK;
}

int bfp200_generate_sampled(bfp200_handle* h, const int32_t* prompt_ids, const int32_t* prompt_lens, int n_seq,
                            int n_gen, double temperature, int top_k, uint32_t seed, int32_t* out_tokens) {
  if (!(temperature > 0.0)) return generate_impl(h, prompt_ids, prompt_lens, n_seq, n_gen, 0, out_tokens, nullptr);
  if (!std::isfinite(temperature) || top_k < 0) return fail(BFP200_EINVAL, "generate_sampled: bad temperature / top_k");
  Sampling smp;
  smp.temperature = temperature;
  smp.top_k = top_k;
  smp.seed = seed;
  return generate_impl(h, prompt_ids, prompt_lens, n_seq, n_gen, 0, out_tokens, &smp);
}

static int generate_impl(bfp200_handle* h, const int32_t* prompt_ids, const int32_t* prompt_lens, int n_seq,
                         int n_gen, int feed_mode, int32_t* out_tokens, const Sampling* smp) {
  if (!h || !out_tokens) return fail(BFP200_EINVAL, "generate: null argument");
  if (h->broken) return fail(BFP200_ESTATE, "handle unusable: an aborted exchange never left its stream");
  if (smp && h->comm) return fail(BFP200_EINVAL, "sampling is not available with a sharded head");
  if (!h->have_image) return fail(BFP200_ESTATE, "generate before load_image");
  if (feed_mode != 0 && feed_mode != 1) return fail(BFP200_EINVAL, "feed_mode must be 0 (sim) or 1 (rtl)");
  if (n_gen < 0) return fail(BFP200_EINVAL, "n_gen < 0");
  std::vector<int32_t> ids, lens;
  if (!prompt_ids) {
    if (h->rom_prompt.empty() || n_seq != 1) return fail(BFP200_EINVAL, "no prompt given and no prompt ROM loaded");
    ids = h->rom_prompt;
    lens = {(int32_t)ids.size()};
  } else {
    if (!prompt_lens || n_seq <= 0) return fail(BFP200_EINVAL, "generate: bad prompt arguments");
    lens.assign(prompt_lens, prompt_lens + n_seq);
    const size_t tot = std::accumulate(lens.begin(), lens.end(), (size_t)0);
    ids.assign(prompt_ids, prompt_ids + tot);
  }
  if (n_seq > h->cfg.max_seqs) return fail(BFP200_EINVAL, "n_seq > max_seqs");
  for (int s = 0; s < n_seq; ++s) {
    if (lens[s] <= 0 || lens[s] > h->cfg.NPROMPT_MAX) return fail(BFP200_EINVAL, "prompt length outside 1..NPROMPT_MAX");
    if (lens[s] + n_gen > h->MAXC) return fail(BFP200_EINVAL, "prompt length + n_gen exceeds MAX_CTX");
  }
  for (int32_t t : ids)
    if (t < 0 || t >= h->V) return fail(BFP200_EINVAL, "token id outside the vocabulary");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  CKR(ensure_kv(h, n_seq));
  // ---- prefill: every prompt position, position-major
  const int PREFILL_CHUNK = 1024;
  std::vector<int32_t> off(n_seq + 1, 0);
  for (int s = 0; s < n_seq; ++s) off[s + 1] = off[s] + lens[s];
  std::vector<int> cs, cp, ct;
  const int maxlen = *std::max_element(lens.begin(), lens.end());
  for (int p = 0; p < maxlen; ++p)
    for (int s = 0; s < n_seq; ++s)
      if (p < lens[s]) { cs.push_back(s); cp.push_back(p); ct.push_back(ids[off[s] + p]); }
  const int ncp = (int)cs.size();
  CKR(ensure_cols(h, std::max(std::min(ncp, PREFILL_CHUNK), n_seq)));
  const bool rtl = feed_mode == 1;
  if (rtl) CK(h->rtl_out.ensure((size_t)n_seq * h->cfg.NPROMPT_MAX));
  CK(h->uncert_dev.ensure(1));
  CK(cudaMemsetAsync(h->uncert_dev.p, 0, 8, h->stream));
  cudaEvent_t ev0, ev1, ev2;
  cudaEventCreate(&ev0); cudaEventCreate(&ev1); cudaEventCreate(&ev2);
  CK(cudaEventRecord(ev0, h->stream));
  h->launch_count = 0;
  for (int c0 = 0; c0 < ncp; c0 += h->cap) {
    const int nc = std::min(h->cap, ncp - c0);
    CK(cudaMemcpyAsync(h->col_slot.p, cs.data() + c0, nc * 4, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(h->col_pos.p, cp.data() + c0, nc * 4, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(h->col_tok.p, ct.data() + c0, nc * 4, cudaMemcpyHostToDevice, h->stream));
    CKR(enqueue_forward(h, nc, rtl));
    if (rtl) {
      scatter_tokens_kernel<<<(nc + 255) / 256, 256, 0, h->stream>>>(h->tok.p, h->cert.p, h->col_slot.p,
                                                                     h->col_pos.p, nc, h->cfg.NPROMPT_MAX,
                                                                     h->rtl_out.p, h->uncert_dev.p);
      ++h->launch_count;
    }
    CKR(sync_stream(h));   // host column arrays are reused by the next chunk
  }
  CK(cudaEventRecord(ev1, h->stream));
  std::vector<int32_t> rtl_host;
  if (rtl) {
    rtl_host.resize((size_t)n_seq * h->cfg.NPROMPT_MAX);
    CK(cudaMemcpyAsync(rtl_host.data(), h->rtl_out.p, rtl_host.size() * 4, cudaMemcpyDeviceToHost, h->stream));
    CKR(sync_stream(h));
  }
  // ---- decode: column s = sequence s at position len_s, fed its last token
  std::vector<int> dslot(n_seq), dpos(n_seq), dtok(n_seq);
  for (int s = 0; s < n_seq; ++s) {
    dslot[s] = s;
    dpos[s] = lens[s];
    dtok[s] = rtl ? rtl_host[(size_t)s * h->cfg.NPROMPT_MAX + lens[s] - 1] : ids[off[s] + lens[s] - 1];
  }
  const int u_ld = n_gen + 1;
  if (n_gen > 0 && smp) {
    // one uniform per sampled step; index 0 is the draw the reference makes
    // (and discards) at the last prompt position
    const size_t nv = (size_t)n_seq * h->V;
    CK(h->s_logits.ensure(nv)); CK(h->s_work.ensure(nv)); CK(h->s_cdf.ensure(nv)); CK(h->s_incl.ensure(nv));
    CK(h->s_uni.ensure((size_t)n_seq * u_ld));
    if (!h->v_plan_leaves) {
      std::vector<unsigned short> plan;
      build_pw_plan_one(h->V, plan);
      CK(h->v_plan.ensure(plan.size()));
      CK(cudaMemcpyAsync(h->v_plan.p, plan.data(), plan.size() * 2, cudaMemcpyHostToDevice, h->stream));
      h->v_plan_leaves = plan[0];
    }
    std::vector<double> uni((size_t)n_seq * u_ld);
    for (int s = 0; s < n_seq; ++s) mt19937_uniforms(smp->seed + (uint32_t)s, u_ld, uni.data() + (size_t)s * u_ld);
    CK(cudaMemcpyAsync(h->s_uni.p, uni.data(), uni.size() * 8, cudaMemcpyHostToDevice, h->stream));
    CKR(sync_stream(h));
  }
  if (n_gen > 0) {
    CK(h->gen_out.ensure((size_t)n_seq * n_gen));
    CK(h->dec_step.ensure(1));
    CK(cudaMemcpyAsync(h->col_slot.p, dslot.data(), n_seq * 4, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(h->col_pos.p, dpos.data(), n_seq * 4, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemcpyAsync(h->col_tok.p, dtok.data(), n_seq * 4, cudaMemcpyHostToDevice, h->stream));
    CK(cudaMemsetAsync(h->dec_step.p, 0, 4, h->stream));
    {
      // one decode step captured once as a CUDA graph, replayed n_gen times
      const double temp = smp ? smp->temperature : 0.0;
      const int topk = smp ? smp->top_k : 0;
      if (!h->graph || h->graph_cols != n_seq || h->graph_ngen != n_gen || h->graph_temp != temp ||
          h->graph_topk != topk) {
        if (h->graph) { cudaGraphExecDestroy(h->graph); h->graph = nullptr; }
        if (!small_path_ok(h, n_seq) && h->use_tc && n_seq >= h->tc_min_cols) {
          // tensor-core configurations are chosen by timing, which a capture
          // cannot do: run the layer shapes once first (scratch outputs only)
          CKR(enqueue_layer_matmuls(h, 0, n_seq));
        }
        CKR(sync_stream(h));
        cudaGraph_t g;
        CK(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
        const long long before = h->launch_count;
        // 1..4 columns, greedy, unsharded: the single-launch head also feeds
        // the token back (no separate advance kernel)
        const bool fused_adv = !smp && !h->comm && h->use_small && head_small_supported(n_seq, h->D);
        if (fused_adv) {
          h->head_adv.gen_out = h->gen_out.p; h->head_adv.col_tok = h->col_tok.p; h->head_adv.col_pos = h->col_pos.p;
          h->head_adv.step = h->dec_step.p; h->head_adv.uncert = h->uncert_dev.p; h->head_adv.n_gen = n_gen;
        }
        int r = enqueue_forward(h, n_seq, smp == nullptr, /*decode=*/true);
        h->head_adv = HeadAdvance();
        if (r == BFP200_OK && smp) r = enqueue_sample_head(h, n_seq, *smp, u_ld);
        h->graph_launches = h->launch_count - before + (fused_adv ? 0 : 1);   // + the advance kernel
        h->launch_count = before;
        if (!fused_adv)
          advance_kernel<<<1, 256, 0, h->stream>>>(h->tok.p, h->cert.p, n_seq, n_gen, h->gen_out.p, h->col_tok.p,
                                                   h->col_pos.p, h->dec_step.p, h->uncert_dev.p);
        cudaError_t ce = cudaStreamEndCapture(h->stream, &g);
        if (r != BFP200_OK) { if (ce == cudaSuccess) cudaGraphDestroy(g); return r; }
        CK(ce);
        ce = cudaGraphInstantiate(&h->graph, g, 0);
        cudaGraphDestroy(g);
        CK(ce);
        h->graph_cols = n_seq;
        h->graph_ngen = n_gen;
        h->graph_temp = temp;
        h->graph_topk = topk;
      }
      if (h->comm) {
        // sharded: one step at a time, each waited for with the bounded poll,
        // so a missing rank can never leave later steps queued behind an
        // exchange that gets aborted
        for (int i = 0; i < n_gen; ++i) {
          CK(cudaGraphLaunch(h->graph, h->stream));
          CKR(sync_stream(h));
        }
      } else {
        for (int i = 0; i < n_gen; ++i) CK(cudaGraphLaunch(h->graph, h->stream));
      }
      h->launch_count += h->graph_launches * n_gen;
    }
  }
  CK(cudaEventRecord(ev2, h->stream));
  std::vector<int32_t> gen((size_t)n_seq * n_gen);
  if (n_gen > 0) CK(cudaMemcpyAsync(gen.data(), h->gen_out.p, gen.size() * 4, cudaMemcpyDeviceToHost, h->stream));
  long long unc = 0;
  CK(cudaMemcpyAsync(&unc, h->uncert_dev.p, 8, cudaMemcpyDeviceToHost, h->stream));
  CKR(sync_stream(h));
  float ms1 = 0, ms2 = 0;
  cudaEventElapsedTime(&ms1, ev0, ev1);
  cudaEventElapsedTime(&ms2, ev1, ev2);
  cudaEventDestroy(ev0); cudaEventDestroy(ev1); cudaEventDestroy(ev2);
  h->t_prefill = ms1;
  h->t_decode = ms2;
  h->last_launches = h->launch_count;
  h->uncert = unc;
  if (read_and_clear_error_flag(h->stream)) return fail(BFP200_ETIMEOUT, "a bounded device wait timed out");
  // ---- assemble: sim = prompt + generated; rtl = one argmax per step
  size_t o = 0;
  for (int s = 0; s < n_seq; ++s) {
    for (int p = 0; p < lens[s]; ++p)
      out_tokens[o++] = rtl ? rtl_host[(size_t)s * h->cfg.NPROMPT_MAX + p] : ids[off[s] + p];
    for (int i = 0; i < n_gen; ++i) out_tokens[o++] = gen[(size_t)s * n_gen + i];
  }
  return BFP200_OK;
}

int bfp200_generate_multi(bfp200_handle* const* hs, int n_dev, const int32_t* prompt_ids, const int32_t* prompt_lens,
                          int n_seq, int n_gen, int feed_mode, int32_t* out_tokens) {
  if (!hs || n_dev <= 0 || !prompt_ids || !prompt_lens || n_seq <= 0)
    return fail(BFP200_EINVAL, "generate_multi: bad arguments");
  // contiguous blocks balanced by total steps
  std::vector<long long> cum(n_seq + 1, 0);
  for (int s = 0; s < n_seq; ++s) cum[s + 1] = cum[s] + prompt_lens[s] + n_gen;
  std::vector<int> b(n_dev + 1, 0);
  b[n_dev] = n_seq;
  for (int d = 1; d < n_dev; ++d) {
    const long long target = cum[n_seq] * d / n_dev;
    b[d] = (int)(std::lower_bound(cum.begin(), cum.end(), target) - cum.begin());
    b[d] = std::max(b[d], b[d - 1]);
  }
  std::vector<size_t> id_off(n_seq + 1, 0), out_off(n_seq + 1, 0);
  for (int s = 0; s < n_seq; ++s) {
    id_off[s + 1] = id_off[s] + prompt_lens[s];
    out_off[s + 1] = out_off[s] + prompt_lens[s] + n_gen;
  }
  std::vector<int> rc(n_dev, BFP200_OK);
  std::vector<std::string> errs(n_dev);
  std::vector<std::thread> th;
  for (int d = 0; d < n_dev; ++d) {
    if (b[d + 1] == b[d]) continue;
    th.emplace_back([&, d] {
      rc[d] = bfp200_generate(hs[d], prompt_ids + id_off[b[d]], prompt_lens + b[d], b[d + 1] - b[d], n_gen,
                              feed_mode, out_tokens + out_off[b[d]]);
      if (rc[d] != BFP200_OK) errs[d] = g_err;
    });
  }
  for (auto& t : th) t.join();
  for (int d = 0; d < n_dev; ++d)
    if (rc[d] != BFP200_OK) return fail(rc[d], "device " + std::to_string(d) + ": " + errs[d]);
  return BFP200_OK;
}

int bfp200_nccl_unique_id(uint8_t* id) {
  if (!id) return fail(BFP200_EINVAL, "nccl_unique_id: null argument");
  const NcclApi& a = nccl();
  if (!a.ok) return fail(BFP200_ENODEV, "NCCL (libnccl.so.2) could not be loaded");
  NcclUid u;
  const int r = a.get_unique_id(&u);
  if (r != NCCL_OK) return fail(BFP200_ECUDA, "ncclGetUniqueId: " + nccl_err(r));
  std::memcpy(id, u.internal, BFP200_NCCL_ID_BYTES);
  return BFP200_OK;
}

int bfp200_head_shard(bfp200_handle* h, const uint8_t* id, int nranks, int rank) {
  if (!h || nranks < 1 || rank < 0 || rank >= nranks) return fail(BFP200_EINVAL, "head_shard: bad arguments");
  if (!id) {
    if (nranks == 1) return set_shard(h, nullptr, 1, 0);
    return fail(BFP200_EINVAL, "head_shard: null id");
  }
  if (nranks > h->V) return fail(BFP200_EINVAL, "head_shard: more ranks than vocabulary rows");
  const NcclApi& a = nccl();
  if (!a.ok) return fail(BFP200_ENODEV, "NCCL (libnccl.so.2) could not be loaded");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  nccl_env_defaults();
  NcclUid u;
  std::memcpy(u.internal, id, BFP200_NCCL_ID_BYTES);
  NcclComm c = nullptr;
  const int r = a.comm_init_rank(&c, nranks, u, rank);
  if (r != NCCL_OK) return fail(BFP200_ECUDA, "ncclCommInitRank: " + nccl_err(r));
  CKR(set_shard(h, c, nranks, rank));
  CKR(enqueue_warm_exchange(h));
  return sync_stream(h);
}

int bfp200_head_shard_group(bfp200_handle* const* hs, int n_dev) {
  if (!hs || n_dev < 1) return fail(BFP200_EINVAL, "head_shard_group: bad arguments");
  std::vector<int> devs(n_dev);
  for (int d = 0; d < n_dev; ++d) {
    if (!hs[d]) return fail(BFP200_EINVAL, "head_shard_group: null handle");
    devs[d] = hs[d]->device;
    for (int e = 0; e < d; ++e)
      if (devs[e] == devs[d]) return fail(BFP200_EINVAL, "head_shard_group: two handles on one device");
  }
  if (n_dev == 1) return set_shard(hs[0], nullptr, 1, 0);
  const NcclApi& a = nccl();
  if (!a.ok) return fail(BFP200_ENODEV, "NCCL (libnccl.so.2) could not be loaded");
  DeviceGuard dguard(hs[0]->device);
  for (int d = 0; d < n_dev; ++d) CKR(set_shard(hs[d], nullptr, 1, 0));
  nccl_env_defaults();
  std::vector<NcclComm> comms(n_dev, nullptr);
  const int r = a.comm_init_all(comms.data(), n_dev, devs.data());
  if (r != NCCL_OK) return fail(BFP200_ECUDA, "ncclCommInitAll: " + nccl_err(r));
  for (int d = 0; d < n_dev; ++d) CKR(set_shard(hs[d], comms[d], n_dev, d));
  // one thread drives every device here: the warm exchange is one NCCL group
  int rg = a.group_start();
  for (int d = 0; d < n_dev && rg == NCCL_OK; ++d) {
    cudaSetDevice(hs[d]->device);
    if (enqueue_warm_exchange(hs[d]) != BFP200_OK) rg = -1;
  }
  const int re = a.group_end();
  if (rg != NCCL_OK || (re != NCCL_OK && re != NCCL_IN_PROGRESS))
    return fail(BFP200_ECUDA, "warm exchange of the sharded head failed");
  for (int d = 0; d < n_dev; ++d) {
    DeviceGuard g(hs[d]->device);
    CKR(sync_stream(hs[d]));
  }
  return BFP200_OK;
}

int bfp200_generate_sharded(bfp200_handle* const* hs, int n_dev, const int32_t* prompt_ids,
                            const int32_t* prompt_lens, int n_seq, int n_gen, int feed_mode, int32_t* out_tokens) {
  if (!hs || n_dev < 1 || !out_tokens || n_gen < 0) return fail(BFP200_EINVAL, "generate_sharded: bad arguments");
  for (int d = 0; d < n_dev; ++d) {
    if (!hs[d]) return fail(BFP200_EINVAL, "generate_sharded: null handle");
    if (n_dev > 1 && (!hs[d]->comm || hs[d]->shard_n != n_dev || hs[d]->shard_rank != d))
      return fail(BFP200_ESTATE, "generate_sharded: handles are not one sharded group in rank order");
  }
  size_t n_out = 0;
  if (prompt_ids) {
    if (!prompt_lens || n_seq <= 0) return fail(BFP200_EINVAL, "generate_sharded: bad prompt arguments");
    for (int i = 0; i < n_seq; ++i) n_out += (size_t)std::max(0, prompt_lens[i]) + n_gen;
  } else {
    n_out = hs[0]->rom_prompt.size() + n_gen;
  }
  std::vector<std::vector<int32_t>> outs(n_dev, std::vector<int32_t>(n_out, 0));
  std::vector<int> rc(n_dev, BFP200_OK);
  std::vector<std::string> errs(n_dev);
  std::vector<std::thread> th;
  for (int d = 0; d < n_dev; ++d)
    th.emplace_back([&, d] {
      rc[d] = bfp200_generate(hs[d], prompt_ids, prompt_lens, n_seq, n_gen, feed_mode, outs[d].data());
      if (rc[d] != BFP200_OK) errs[d] = g_err;
    });
  for (auto& t : th) t.join();
  for (int d = 0; d < n_dev; ++d)
    if (rc[d] != BFP200_OK) return fail(rc[d], "rank " + std::to_string(d) + ": " + errs[d]);
  for (int d = 1; d < n_dev; ++d)
    if (outs[d] != outs[0]) return fail(BFP200_ESTATE, "generate_sharded: ranks disagree on the tokens");
  std::copy(outs[0].begin(), outs[0].end(), out_tokens);
  return BFP200_OK;
}

int bfp200_wait_probe(bfp200_handle* h, int limit_ms) {
  if (!h || limit_ms < 1 || limit_ms > 2000) return fail(BFP200_EINVAL, "wait_probe: limit_ms must be 1..2000");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<int> flag;
  CK(flag.ensure(1));
  CK(cudaMemsetAsync(flag.p, 0, sizeof(int), h->stream));
  CK(launch_wait_probe(flag.p, (unsigned long long)limit_ms * 1000000ull, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  if (read_and_clear_error_flag(h->stream)) return fail(BFP200_ETIMEOUT, "a bounded device wait timed out");
  return BFP200_OK;
}

int bfp200_uncertified_steps(bfp200_handle* h, long long* count) {
  if (!h || !count) return fail(BFP200_EINVAL, "null argument");
  *count = h->uncert;
  return BFP200_OK;
}

int bfp200_last_launches(bfp200_handle* h, long long* launches) {
  if (!h || !launches) return fail(BFP200_EINVAL, "last_launches: null argument");
  *launches = h->last_launches;
  return BFP200_OK;
}

int bfp200_last_timing(bfp200_handle* h, double* prefill_ms, double* decode_ms) {
  if (!h) return fail(BFP200_EINVAL, "null handle");
  if (prefill_ms) *prefill_ms = h->t_prefill;
  if (decode_ms) *decode_ms = h->t_decode;
  return BFP200_OK;
}

int bfp200_profile_forward(bfp200_handle* h, int ncols, int pos, double* ms_by_kind, int* launches_by_kind) {
  if (!h || ncols <= 0 || !ms_by_kind) return fail(BFP200_EINVAL, "profile_forward: bad arguments");
  if (!h->have_image) return fail(BFP200_ESTATE, "profile_forward before load_image");
  if (ncols > h->cfg.max_seqs || pos < 0 || pos >= h->MAXC) return fail(BFP200_EINVAL, "profile_forward: ncols/pos");
  if (h->comm) return fail(BFP200_ESTATE, "profile_forward: not on a handle with a sharded head");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  CKR(ensure_kv(h, ncols));
  CKR(ensure_cols(h, ncols));
  std::vector<int> slots(ncols), poss(ncols, pos), toks(ncols, 0);
  std::iota(slots.begin(), slots.end(), 0);
  CK(cudaMemcpyAsync(h->col_slot.p, slots.data(), ncols * 4, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(h->col_pos.p, poss.data(), ncols * 4, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(h->col_tok.p, toks.data(), ncols * 4, cudaMemcpyHostToDevice, h->stream));
  const bool saved = h->pdl;
  h->pdl = false;   // serialised launches: each kernel's time stands alone
  std::vector<std::pair<int, cudaEvent_t>> evs;
  int r = BFP200_OK;
  for (int pass = 0; pass < 2 && r == BFP200_OK; ++pass) {   // pass 0 warms caches and code
    for (auto& pe : evs) cudaEventDestroy(pe.second);
    evs.clear();
    h->prof = &evs;
    r = enqueue_forward(h, ncols, true);
    mark(h, PK_COUNT);
    h->prof = nullptr;
    cudaStreamSynchronize(h->stream);
  }
  h->pdl = saved;
  if (r != BFP200_OK) { for (auto& pe : evs) cudaEventDestroy(pe.second); return r; }
  for (int k = 0; k < PK_COUNT; ++k) { ms_by_kind[k] = 0.0; if (launches_by_kind) launches_by_kind[k] = 0; }
  for (size_t i = 0; i + 1 < evs.size(); ++i) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, evs[i].second, evs[i + 1].second);
    ms_by_kind[evs[i].first] += ms;
    if (launches_by_kind) launches_by_kind[evs[i].first] += 1;
  }
  for (auto& pe : evs) cudaEventDestroy(pe.second);
  CK(cudaGetLastError());
  return BFP200_OK;
}

int bfp200_time_matmuls(bfp200_handle* h, int ncols, int reps, double* ms_per_token, int* launches_per_token) {
  if (!h || ncols <= 0 || reps <= 0 || !ms_per_token) return fail(BFP200_EINVAL, "time_matmuls: bad arguments");
  if (!h->have_image) return fail(BFP200_ESTATE, "time_matmuls before load_image");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  CKR(ensure_cols(h, ncols));
  const bool small = small_path_ok(h, ncols);
  auto body = [&]() -> int {
    for (int l = 0; l < h->NL && small; ++l) {
      CKR(enqueue_gemv_qkv(h, l, ncols, h->pdl));
      CKR(enqueue_gemv_o(h, l, ncols, h->pdl, h->dbg_m.p, h->dbg_e.p));
      CKR(enqueue_gemv_gu(h, l, ncols, h->pdl));
      CKR(enqueue_gemv_d(h, l, ncols, h->pdl, h->dbg_m.p, h->dbg_e.p));
    }
    for (int l = 0; l < h->NL && !small; ++l) CKR(enqueue_layer_matmuls(h, l, ncols));
    return BFP200_OK;
  };
  if (!small) {                       // choose the tensor-core configurations outside the capture
    CKR(enqueue_layer_matmuls(h, 0, ncols));
    CK(cudaStreamSynchronize(h->stream));
  }
  CK(cudaStreamSynchronize(h->stream));
  cudaGraph_t g;
  CK(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
  const int r = body();
  cudaError_t ce = cudaStreamEndCapture(h->stream, &g);
  if (r != BFP200_OK) { if (ce == cudaSuccess) cudaGraphDestroy(g); return r; }
  CK(ce);
  cudaGraphExec_t ge;
  ce = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  CK(ce);
  for (int i = 0; i < 3; ++i) CK(cudaGraphLaunch(ge, h->stream));
  cudaEvent_t a, b;
  cudaEventCreate(&a); cudaEventCreate(&b);
  CK(cudaEventRecord(a, h->stream));
  for (int i = 0; i < reps; ++i) CK(cudaGraphLaunch(ge, h->stream));
  CK(cudaEventRecord(b, h->stream));
  CK(cudaEventSynchronize(b));
  float ms = 0;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a); cudaEventDestroy(b);
  cudaGraphExecDestroy(ge);
  *ms_per_token = ms / reps;
  if (launches_per_token) *launches_per_token = 4 * h->NL;
  if (read_and_clear_error_flag(h->stream)) return fail(BFP200_ETIMEOUT, "a bounded device wait timed out");
  return BFP200_OK;
}

// ---------------------------------------------------------------------------
// op-level entry points
// ---------------------------------------------------------------------------
int bfp200_tile_quantize(bfp200_handle* h, const double* v, size_t n, int16_t* m, int8_t* e) {
  if (!h || (n && (!v || !m || !e)) || n % 16) return fail(BFP200_EINVAL, "tile_quantize: bad arguments");
  if (!n) return BFP200_OK;
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<double> dv; DBuf<int16_t> dm; DBuf<int8_t> de;
  CK(dv.ensure(n)); CK(dm.ensure(n)); CK(de.ensure(n / 16));
  CK(cudaMemcpyAsync(dv.p, v, n * 8, cudaMemcpyHostToDevice, h->stream));
  CK(launch_tile_quantize(dv.p, (long long)(n / 16), dm.p, de.p, h->stream));
  CK(cudaMemcpyAsync(m, dm.p, n * 2, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaMemcpyAsync(e, de.p, n / 16, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_tile_decode(bfp200_handle* h, const int16_t* m, const int8_t* e, size_t n, double* v) {
  if (!h || (n && (!v || !m || !e)) || n % 16) return fail(BFP200_EINVAL, "tile_decode: bad arguments");
  if (!n) return BFP200_OK;
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<double> dv; DBuf<int16_t> dm; DBuf<int8_t> de;
  CK(dv.ensure(n)); CK(dm.ensure(n)); CK(de.ensure(n / 16));
  CK(cudaMemcpyAsync(dm.p, m, n * 2, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(de.p, e, n / 16, cudaMemcpyHostToDevice, h->stream));
  CK(launch_tile_decode(dm.p, de.p, (long long)(n / 16), dv.p, h->stream));
  CK(cudaMemcpyAsync(v, dv.p, n * 8, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

static int matvec_impl(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* W_m,
                       const int8_t* W_e, int D_out, int D_in, int batch, int16_t* out_m, int8_t* out_e, int reps,
                       double* ms_per_call);

int bfp200_matvec(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* W_m, const int8_t* W_e,
                  int D_out, int D_in, int batch, int16_t* out_m, int8_t* out_e) {
  return matvec_impl(h, x_m, x_e, W_m, W_e, D_out, D_in, batch, out_m, out_e, 0, nullptr);
}

int bfp200_matvec_timed(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* W_m,
                        const int8_t* W_e, int D_out, int D_in, int batch, int reps, int16_t* out_m, int8_t* out_e,
                        double* ms_per_call) {
  if (reps <= 0 || !ms_per_call) return fail(BFP200_EINVAL, "matvec_timed: reps >= 1 and an output required");
  return matvec_impl(h, x_m, x_e, W_m, W_e, D_out, D_in, batch, out_m, out_e, reps, ms_per_call);
}

static int matvec_impl(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* W_m,
                       const int8_t* W_e, int D_out, int D_in, int batch, int16_t* out_m, int8_t* out_e, int reps,
                       double* ms_per_call) {
  if (!h || !x_m || !x_e || !W_m || !W_e || !out_m || !out_e || D_out <= 0 || D_in <= 0 || D_out % 16 ||
      D_in % 16 || batch <= 0)
    return fail(BFP200_EINVAL, "matvec: bad arguments (D_out, D_in multiples of 16, batch >= 1)");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  const int NT = D_in / 16, G = D_out / 16;
  DBuf<int16_t> dWm, dxm, dom; DBuf<int8_t> dWe, dxe, doe; DBuf<uint8_t> wm; DBuf<int8_t> we;
  CK(dWm.ensure((size_t)D_out * D_in)); CK(dWe.ensure((size_t)D_out * NT));
  CK(dxm.ensure((size_t)batch * D_in)); CK(dxe.ensure((size_t)batch * NT));
  CK(dom.ensure((size_t)batch * D_out)); CK(doe.ensure((size_t)batch * G));
  CK(wm.ensure((size_t)G * NT * 512)); CK(we.ensure((size_t)G * NT * 16));
  CK(cudaMemcpyAsync(dWm.p, W_m, (size_t)D_out * D_in * 2, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(dWe.p, W_e, (size_t)D_out * NT, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(dxm.p, x_m, (size_t)batch * D_in * 2, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(dxe.p, x_e, (size_t)batch * NT, cudaMemcpyHostToDevice, h->stream));
  CK(launch_pack_weights(dWm.p, dWe.p, D_out, NT, wm.p, we.p, 1, 0, h->stream));
  DevMat W;
  W.wm = wm.p; W.we = we.p; W.G = G; W.NT = NT;
  DBuf<uint8_t> rec;
  DBuf<long long> acc; DBuf<unsigned> cnt;
  // 1..4 columns: the decode path's small-batch GEMV; 16+: tensor cores;
  // otherwise the dp2a matmul -- the kernels a decode step would run
  const bool small = h->use_small && batch <= 4 && gemv_supported(GV_STORE, false, NT, batch);
  const bool tc = !small && tc_path(h, W, batch, EPI_STORE);
  if (small) {
  } else if (tc) {
    CK(rec.ensure(tc_records_bytes(D_out, NT)));
    CK(launch_tc_pack(wm.p, we.p, D_out, NT, rec.p, h->stream));
  } else {
    const MMPlan p = plan_matmul(G, NT, batch, false, h->nsm);
    if (p.ks > 1) {
      CK(acc.ensure((size_t)D_out * batch));
      CK(cnt.ensure((size_t)G * ((batch + p.bn - 1) / p.bn)));
    }
  }
  // the matvec only reads its inputs and writes its outputs: repeating it
  // (timing) leaves the same result
  auto run = [&]() -> int {
    if (small) {
      GemvArgs g;
      g.W = W;
      g.xm = dxm.p; g.xe = dxe.p; g.x_ld = D_in; g.x_lde = NT;
      g.ncols = batch;
      g.mode = GV_STORE;
      g.om = dom.p; g.oe = doe.p; g.o_ld = D_out; g.o_lde = G;
      CK(launch_gemv(g, h->stream, false));
      return BFP200_OK;
    }
    if (tc) return enqueue_tc(h, rec.p, W, dxm.p, dxe.p, D_in, NT, batch, EPI_STORE, dom.p, doe.p, D_out, G, nullptr,
                              nullptr);
    return enqueue_matmul(h, W, dxm.p, dxe.p, D_in, NT, batch, EPI_STORE, dom.p, doe.p, D_out, G, nullptr, nullptr,
                          acc.p, cnt.p, batch);
  };
  CKR(run());
  if (reps > 0) {
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0)); CK(cudaEventCreate(&e1));
    int r = BFP200_OK;
    CK(cudaEventRecord(e0, h->stream));
    for (int i = 0; i < reps && r == BFP200_OK; ++i) r = run();
    CK(cudaEventRecord(e1, h->stream));
    CK(cudaEventSynchronize(e1));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0); cudaEventDestroy(e1);
    if (r != BFP200_OK) return r;
    *ms_per_call = ms / reps;
  }
  CK(cudaMemcpyAsync(out_m, dom.p, (size_t)batch * D_out * 2, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaMemcpyAsync(out_e, doe.p, (size_t)batch * G, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  if (read_and_clear_error_flag(h->stream)) return fail(BFP200_ETIMEOUT, "a bounded device wait timed out");
  return BFP200_OK;
}

int bfp200_rmsnorm_fp(bfp200_handle* h, const double* x, const double* gamma, int n, int ncols, double eps,
                      double* out) {
  if (!h || !x || !gamma || !out || n <= 0 || n % 16 || ncols <= 0 || n > 8192)
    return fail(BFP200_EINVAL, "rmsnorm_fp: bad arguments");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<double> dx, dg, dout;
  CK(dx.ensure((size_t)n * ncols)); CK(dg.ensure(n)); CK(dout.ensure((size_t)n * ncols));
  CK(cudaMemcpyAsync(dx.p, x, (size_t)n * ncols * 8, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(dg.p, gamma, (size_t)n * 8, cudaMemcpyHostToDevice, h->stream));
  CK(launch_rmsnorm_fp(dx.p, dg.p, eps, n, ncols, dout.p, h->stream));
  CK(cudaMemcpyAsync(out, dout.p, (size_t)n * ncols * 8, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_silu_fp(bfp200_handle* h, const double* x, size_t n, double* out) {
  if (!h || (n && (!x || !out)) || n % 16) return fail(BFP200_EINVAL, "silu_fp: bad arguments");
  if (!n) return BFP200_OK;
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<double> dx, dout;
  CK(dx.ensure(n)); CK(dout.ensure(n));
  CK(cudaMemcpyAsync(dx.p, x, n * 8, cudaMemcpyHostToDevice, h->stream));
  CK(launch_silu_fp(dx.p, (long long)n, dout.p, h->stream));
  CK(cudaMemcpyAsync(out, dout.p, n * 8, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_softmax_fp(bfp200_handle* h, const double* x, int n, int ncols, double* out) {
  if (!h || !x || !out || n <= 0 || ncols <= 0 || n > 4096) return fail(BFP200_EINVAL, "softmax_fp: bad arguments");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<double> dx, dout;
  CK(dx.ensure((size_t)n * ncols)); CK(dout.ensure((size_t)n * ncols));
  CK(cudaMemcpyAsync(dx.p, x, (size_t)n * ncols * 8, cudaMemcpyHostToDevice, h->stream));
  CK(launch_softmax_fp(dx.p, n, ncols, dout.p, h->stream));
  CK(cudaMemcpyAsync(out, dout.p, (size_t)n * ncols * 8, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_pairwise_sum(bfp200_handle* h, const double* x, int n, int ncols, double* out) {
  if (!h || !x || !out || n <= 0 || ncols <= 0 || n > 3072) return fail(BFP200_EINVAL, "pairwise_sum: bad arguments");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<double> dx, dout;
  CK(dx.ensure((size_t)n * ncols)); CK(dout.ensure(ncols));
  CK(cudaMemcpyAsync(dx.p, x, (size_t)n * ncols * 8, cudaMemcpyHostToDevice, h->stream));
  // the plan-driven reduction the attention kernel uses; the generic
  // single-lane tree walk is exercised by softmax_fp
  std::vector<unsigned short> plan;
  build_pw_plan_one(n, plan);
  DBuf<unsigned short> dplan;
  CK(dplan.ensure(plan.size()));
  CK(cudaMemcpyAsync(dplan.p, plan.data(), plan.size() * 2, cudaMemcpyHostToDevice, h->stream));
  CK(launch_np_sum_plan(dx.p, n, ncols, dplan.p, dout.p, h->stream));
  CK(cudaMemcpyAsync(out, dout.p, (size_t)ncols * 8, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_rope_fp(bfp200_handle* h, const double* x, const int32_t* pos, int nvec, int HD, double base, double* out) {
  if (!h || !x || !pos || !out || nvec <= 0 || HD <= 0 || HD % 32) return fail(BFP200_EINVAL, "rope_fp: bad arguments");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  std::vector<double> cs((size_t)nvec * HD);
  for (int i = 0; i < nvec; ++i) {
    if (pos[i] < 0) return fail(BFP200_EINVAL, "rope_fp: negative position");
    // one row of the table for this position
    const int H2 = HD / 2;
    for (int j = 0; j < H2; ++j) {
      const double expo = (double)(2 * j) / (double)HD;
      const double pw = (expo == 0.0) ? 1.0 : std::pow(base, expo);
      const double theta = 1.0 / pw * (double)pos[i];
      cs[(size_t)i * HD + 2 * j] = std::cos(theta);
      cs[(size_t)i * HD + 2 * j + 1] = std::sin(theta);
    }
  }
  DBuf<double> dx, dcs, dout;
  CK(dx.ensure((size_t)nvec * HD)); CK(dcs.ensure(cs.size())); CK(dout.ensure((size_t)nvec * HD));
  CK(cudaMemcpyAsync(dx.p, x, (size_t)nvec * HD * 8, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(dcs.p, cs.data(), cs.size() * 8, cudaMemcpyHostToDevice, h->stream));
  CK(launch_rope_fp(dx.p, dcs.p, HD, nvec, dout.p, h->stream));
  CK(cudaMemcpyAsync(out, dout.p, (size_t)nvec * HD * 8, cudaMemcpyDeviceToHost, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

// ---------------------------------------------------------------------------
// fixed-point ("rtl-exact") leaf ops: host buffers in and out
// ---------------------------------------------------------------------------

int bfp200_rtl_matvec(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* W_m, const int8_t* W_e,
                      int D_out, int D_in, int batch, int16_t* y_m, int8_t* y_e) {
  if (!h || !x_m || !x_e || !W_m || !W_e || !y_m || !y_e || D_out <= 0 || D_in <= 0 || D_in % 16 ||
      D_in / 16 > 96 || batch <= 0)
    return fail(BFP200_EINVAL, "rtl_matvec: bad arguments (D_in a multiple of 16, at most 1536)");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  const int NT = D_in / 16;
  DBuf<int16_t> xm, wm, ym;
  DBuf<int8_t> xe, we, ye;
  CKR(upload(xm, x_m, (size_t)batch * D_in, h->stream)); CKR(upload(xe, x_e, (size_t)batch * NT, h->stream));
  CKR(upload(wm, W_m, (size_t)D_out * D_in, h->stream)); CKR(upload(we, W_e, (size_t)D_out * NT, h->stream));
  CK(ym.ensure((size_t)batch * D_out)); CK(ye.ensure((size_t)batch * D_out));
  CK(launch_rtl_matvec(xm.p, xe.p, wm.p, we.p, D_out, NT, batch, ym.p, ye.p, h->stream));
  CKR(download(y_m, ym, (size_t)batch * D_out, h->stream)); CKR(download(y_e, ye, (size_t)batch * D_out, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_rtl_rmsnorm(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* g_m, const int8_t* g_e,
                       int D, int nvec, int16_t* y_m, int8_t* y_e) {
  if (!h || !x_m || !x_e || !g_m || !g_e || !y_m || !y_e || D <= 0 || D % 16 || D / 16 > 96 || nvec <= 0)
    return fail(BFP200_EINVAL, "rtl_rmsnorm: bad arguments (D a multiple of 16, at most 1536)");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  const size_t n = (size_t)nvec * D, nt = n / 16;
  DBuf<int16_t> xm, gm, ym;
  DBuf<int8_t> xe, ge, ye;
  CKR(upload(xm, x_m, n, h->stream)); CKR(upload(xe, x_e, nt, h->stream));
  CKR(upload(gm, g_m, n, h->stream)); CKR(upload(ge, g_e, nt, h->stream));
  CK(ym.ensure(n)); CK(ye.ensure(nt));
  CK(launch_rtl_rmsnorm(xm.p, xe.p, gm.p, ge.p, D, nvec, ym.p, ye.p, h->stream));
  CKR(download(y_m, ym, n, h->stream)); CKR(download(y_e, ye, nt, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_rtl_rope(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int32_t* pos, int nvec, int HD,
                    const uint32_t* turns_q31, int16_t* y_m, int8_t* y_e) {
  if (!h || !x_m || !x_e || !pos || !turns_q31 || !y_m || !y_e || nvec <= 0 || HD <= 0 || HD % 32)
    return fail(BFP200_EINVAL, "rtl_rope: bad arguments (HD a multiple of 32)");
  for (int i = 0; i < nvec; ++i)
    if (pos[i] < 0 || pos[i] >= (1 << 20)) return fail(BFP200_EINVAL, "rtl_rope: position outside 0 .. 2^20-1");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  const size_t n = (size_t)nvec * HD;
  DBuf<int16_t> xm, ym;
  DBuf<int8_t> xe, ye;
  DBuf<int> dp;
  DBuf<unsigned> dt;
  CKR(upload(xm, x_m, n, h->stream)); CKR(upload(xe, x_e, n / 16, h->stream));
  CKR(upload(dp, (const int*)pos, (size_t)nvec, h->stream));
  CKR(upload(dt, (const unsigned*)turns_q31, (size_t)HD / 2, h->stream));
  CK(ym.ensure(n)); CK(ye.ensure(n));
  CK(launch_rtl_rope(xm.p, xe.p, dp.p, dt.p, HD, nvec, ym.p, ye.p, h->stream));
  CKR(download(y_m, ym, n, h->stream)); CKR(download(y_e, ye, n, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_rtl_softmax(bfp200_handle* h, const int16_t* x_m, const int32_t* x_e, int n, int nvec,
                       const uint16_t* exp_lut, int16_t* y_m, int32_t* y_e) {
  if (!h || !x_m || !x_e || !exp_lut || !y_m || !y_e || n <= 0 || n > 65536 || nvec <= 0)
    return fail(BFP200_EINVAL, "rtl_softmax: bad arguments (1 <= n <= 65536)");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  const size_t nn = (size_t)nvec * n;
  DBuf<int16_t> xm, ym;
  DBuf<int> xe, ye;
  DBuf<uint16_t> lut;
  CKR(upload(xm, x_m, nn, h->stream)); CKR(upload(xe, (const int*)x_e, (size_t)nvec, h->stream));
  CKR(upload(lut, exp_lut, 1024, h->stream));
  CK(ym.ensure(nn)); CK(ye.ensure((size_t)nvec));
  CK(launch_rtl_softmax(xm.p, xe.p, n, nvec, lut.p, ym.p, ye.p, h->stream));
  CKR(download(y_m, ym, nn, h->stream)); CKR(download((int*)y_e, ye, (size_t)nvec, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_rtl_swiglu(bfp200_handle* h, const int16_t* gate_m, const int8_t* gate_e, const int16_t* up_m,
                      const int8_t* up_e, size_t n, const int16_t* silu_lut, int16_t* y_m, int8_t* y_e) {
  if (!h || !gate_m || !gate_e || !up_m || !up_e || !silu_lut || !y_m || !y_e || n == 0 || n % 16)
    return fail(BFP200_EINVAL, "rtl_swiglu: bad arguments (n a multiple of 16)");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<int16_t> gm, um, ym, lut;
  DBuf<int8_t> ge, ue, ye;
  CKR(upload(gm, gate_m, n, h->stream)); CKR(upload(ge, gate_e, n / 16, h->stream));
  CKR(upload(um, up_m, n, h->stream)); CKR(upload(ue, up_e, n / 16, h->stream));
  CKR(upload(lut, silu_lut, 65536, h->stream));
  CK(ym.ensure(n)); CK(ye.ensure(n / 16));
  CK(launch_rtl_swiglu(gm.p, ge.p, um.p, ue.p, (long long)(n / 16), lut.p, ym.p, ye.p, h->stream));
  CKR(download(y_m, ym, n, h->stream)); CKR(download(y_e, ye, n / 16, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_rtl_residual(bfp200_handle* h, const int16_t* a_m, const int8_t* a_e, const int16_t* b_m,
                        const int8_t* b_e, size_t n, int16_t* y_m, int8_t* y_e) {
  if (!h || !a_m || !a_e || !b_m || !b_e || !y_m || !y_e || n == 0 || n % 16)
    return fail(BFP200_EINVAL, "rtl_residual: bad arguments (n a multiple of 16)");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  DBuf<int16_t> am, bm, ym;
  DBuf<int8_t> ae, be, ye;
  CKR(upload(am, a_m, n, h->stream)); CKR(upload(ae, a_e, n / 16, h->stream));
  CKR(upload(bm, b_m, n, h->stream)); CKR(upload(be, b_e, n / 16, h->stream));
  CK(ym.ensure(n)); CK(ye.ensure(n / 16));
  CK(launch_rtl_residual(am.p, ae.p, bm.p, be.p, (long long)(n / 16), ym.p, ye.p, h->stream));
  CKR(download(y_m, ym, n, h->stream)); CKR(download(y_e, ye, n / 16, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  return BFP200_OK;
}

int bfp200_stage_dims(bfp200_handle* h, int32_t* dims) {
  if (!h || !dims) return fail(BFP200_EINVAL, "null argument");
  const int32_t v[BFP200_NSTAGES] = {h->D, h->QD, h->KVD, h->KVD, h->QD, h->D, h->D, h->D, h->FFN, h->FFN, h->FFN, h->D};
  std::memcpy(dims, v, sizeof(v));
  return BFP200_OK;
}

static int fwd_layer_impl(bfp200_handle* h, int layer, const double* h_in, const int32_t* pos, const int32_t* kv_pos,
                          int ncols, double* k_cache, double* v_cache, int max_ctx, double* h_out, double* stages,
                          bool decode_kernels);

int bfp200_fwd_layer(bfp200_handle* h, int layer, const double* h_in, const int32_t* pos, const int32_t* kv_pos,
                     int ncols, double* k_cache, double* v_cache, int max_ctx, double* h_out, double* stages) {
  return fwd_layer_impl(h, layer, h_in, pos, kv_pos, ncols, k_cache, v_cache, max_ctx, h_out, stages, false);
}

int bfp200_fwd_layer_decode(bfp200_handle* h, int layer, const double* h_in, const int32_t* pos,
                            const int32_t* kv_pos, int ncols, double* k_cache, double* v_cache, int max_ctx,
                            double* h_out, double* stages) {
  return fwd_layer_impl(h, layer, h_in, pos, kv_pos, ncols, k_cache, v_cache, max_ctx, h_out, stages, true);
}

static int fwd_layer_impl(bfp200_handle* h, int layer, const double* h_in, const int32_t* pos, const int32_t* kv_pos,
                          int ncols, double* k_cache, double* v_cache, int max_ctx, double* h_out, double* stages,
                          bool decode_kernels) {
  if (!h || !h_in || !pos || !kv_pos || !k_cache || !v_cache || !h_out || ncols <= 0)
    return fail(BFP200_EINVAL, "fwd_layer: null argument");
  if (decode_kernels && !small_path_ok(h, ncols))
    return fail(BFP200_EINVAL, "fwd_layer_decode: the decode-path kernels take 1..4 columns of this configuration");
  if (!h->have_image) return fail(BFP200_ESTATE, "fwd_layer before load_image");
  if (layer < 0 || layer >= h->NL) return fail(BFP200_EINVAL, "fwd_layer: layer out of range");
  if (ncols > h->cfg.max_seqs || max_ctx <= 0) return fail(BFP200_EINVAL, "fwd_layer: ncols > max_seqs");
  for (int c = 0; c < ncols; ++c)
    if (pos[c] < 0 || pos[c] >= h->MAXC || kv_pos[c] < 0 || kv_pos[c] >= h->MAXC || kv_pos[c] >= max_ctx ||
        pos[c] != kv_pos[c])
      return fail(BFP200_EINVAL, "fwd_layer: positions must satisfy pos == kv_pos < min(MAX_CTX, max_ctx)");
  DeviceGuard dguard(h->device);
  CK(dguard.err);
  CKR(ensure_kv(h, ncols));
  CKR(ensure_cols(h, ncols));
  const int D = h->D, HKV = h->HKV, HD = h->HD;
  // h_in and the cache prefix in exact BFP form
  std::vector<int16_t> hm((size_t)ncols * D);
  std::vector<int8_t> he((size_t)ncols * h->NTD);
  for (size_t t = 0; t < (size_t)ncols * h->NTD; ++t)
    if (!grid_encode_tile(h_in + t * 16, hm.data() + t * 16, he.data() + t))
      return fail(BFP200_EINVAL, "fwd_layer: h_in is not on the BFP grid");
  CK(cudaMemcpyAsync(h->h_m.p, hm.data(), hm.size() * 2, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(h->h_e.p, he.data(), he.size(), cudaMemcpyHostToDevice, h->stream));
  const size_t slot_stride = (size_t)h->NL * HKV * h->MAXC;   // rows of HD per slot
  for (int c = 0; c < ncols; ++c) {
    for (int kvh = 0; kvh < HKV; ++kvh) {
      const int T = kv_pos[c];
      if (T == 0) continue;
      std::vector<int16_t> kmh((size_t)T * HD), vmh((size_t)T * HD);
      std::vector<int8_t> keh((size_t)T * HD / 16), veh((size_t)T * HD / 16);
      for (int t = 0; t < T; ++t)
        for (int q = 0; q < HD / 16; ++q) {
          const size_t src = (((size_t)c * max_ctx + t) * HKV + kvh) * HD + q * 16;
          if (!grid_encode_tile(k_cache + src, kmh.data() + (size_t)t * HD + q * 16, keh.data() + (size_t)t * HD / 16 + q) ||
              !grid_encode_tile(v_cache + src, vmh.data() + (size_t)t * HD + q * 16, veh.data() + (size_t)t * HD / 16 + q))
            return fail(BFP200_EINVAL, "fwd_layer: KV cache value not on the BFP grid");
        }
      const size_t row0 = (size_t)c * slot_stride + ((size_t)layer * HKV + kvh) * h->MAXC;
      CK(cudaMemcpyAsync(h->km.p + row0 * HD, kmh.data(), kmh.size() * 2, cudaMemcpyHostToDevice, h->stream));
      CK(cudaMemcpyAsync(h->vm.p + row0 * HD, vmh.data(), vmh.size() * 2, cudaMemcpyHostToDevice, h->stream));
      CK(cudaMemcpyAsync(h->ke.p + row0 * HD / 16, keh.data(), keh.size(), cudaMemcpyHostToDevice, h->stream));
      CK(cudaMemcpyAsync(h->ve.p + row0 * HD / 16, veh.data(), veh.size(), cudaMemcpyHostToDevice, h->stream));
    }
  }
  std::vector<int> slots(ncols);
  std::iota(slots.begin(), slots.end(), 0);
  CK(cudaMemcpyAsync(h->col_slot.p, slots.data(), ncols * 4, cudaMemcpyHostToDevice, h->stream));
  CK(cudaMemcpyAsync(h->col_pos.p, pos, ncols * 4, cudaMemcpyHostToDevice, h->stream));
  CK(cudaStreamSynchronize(h->stream));
  StageSink sink;
  sink.st.resize(BFP200_NSTAGES);
  if (decode_kernels) {
    // the production 1..4-column kernels, each dumping the stages it computes
    const int ld = stage_stride(h);
    CK(h->stage_buf.ensure((size_t)ncols * ld));
    CK(cudaMemsetAsync(h->stage_buf.p, 0, (size_t)ncols * ld * 8, h->stream));
    h->stage_dbg = stages ? h->stage_buf.p : nullptr;
    h->stage_ld = ld;
    const int r = enqueue_layer_small(h, layer, ncols, /*first_pdl=*/false, /*early_kv=*/false);
    h->stage_dbg = nullptr;
    CKR(r);
    if (stages) {
      std::vector<double> buf((size_t)ncols * ld);
      CK(cudaMemcpyAsync(buf.data(), h->stage_buf.p, buf.size() * 8, cudaMemcpyDeviceToHost, h->stream));
      CK(cudaStreamSynchronize(h->stream));
      int32_t dims[BFP200_NSTAGES];
      bfp200_stage_dims(h, dims);
      for (int st = 0; st < BFP200_NSTAGES; ++st) {
        sink.st[st].assign((size_t)ncols * dims[st], 0.0);
        for (int c = 0; c < ncols; ++c)
          std::memcpy(sink.st[st].data() + (size_t)c * dims[st], buf.data() + (size_t)c * ld + stage_off(h, st),
                      (size_t)dims[st] * 8);
      }
      // activations the kernels materialise: attn and h1 (multi-kernel path), mlp
      if (!attn_block_ok(h, ncols)) {
        CKR(download_decoded(h, h->a_m.p, h->a_e.p, h->QD, h->QD, 0, ncols, sink.st[4]));
        CKR(download_decoded(h, h->h1_m.p, h->h1_e.p, h->D, h->D, 0, ncols, sink.st[6]));
      }
      CKR(download_decoded(h, h->mlp_m.p, h->mlp_e.p, h->FFN, h->FFN, 0, ncols, sink.st[10]));
    }
  } else {
    CKR(enqueue_layer(h, layer, ncols, stages ? &sink : nullptr, /*first_pdl=*/false));
  }
  std::vector<double> hout;
  CKR(download_decoded(h, h->h_m.p, h->h_e.p, D, D, 0, ncols, hout));
  std::memcpy(h_out, hout.data(), hout.size() * 8);
  // KV slot kv_pos written back (post-RoPE k, raw v)
  for (int c = 0; c < ncols; ++c)
    for (int kvh = 0; kvh < HKV; ++kvh) {
      const size_t row = (size_t)c * slot_stride + ((size_t)layer * HKV + kvh) * h->MAXC + kv_pos[c];
      int16_t km_[64], vm_[64];
      int8_t ke_[4], ve_[4];
      CK(cudaMemcpyAsync(km_, h->km.p + row * HD, HD * 2, cudaMemcpyDeviceToHost, h->stream));
      CK(cudaMemcpyAsync(vm_, h->vm.p + row * HD, HD * 2, cudaMemcpyDeviceToHost, h->stream));
      CK(cudaMemcpyAsync(ke_, h->ke.p + row * HD / 16, HD / 16, cudaMemcpyDeviceToHost, h->stream));
      CK(cudaMemcpyAsync(ve_, h->ve.p + row * HD / 16, HD / 16, cudaMemcpyDeviceToHost, h->stream));
      CK(cudaStreamSynchronize(h->stream));
      const size_t dst = (((size_t)c * max_ctx + kv_pos[c]) * HKV + kvh) * HD;
      for (int i = 0; i < HD; ++i) {
        k_cache[dst + i] = bfp_decode(km_[i], ke_[i / 16]);
        v_cache[dst + i] = bfp_decode(vm_[i], ve_[i / 16]);
      }
    }
  if (stages) {
    // k stage = post-RoPE k (just read back), per column
    sink.st[2].assign((size_t)ncols * h->KVD, 0.0);
    for (int c = 0; c < ncols; ++c)
      for (int i = 0; i < h->KVD; ++i)
        sink.st[2][(size_t)c * h->KVD + i] = k_cache[(((size_t)c * max_ctx + kv_pos[c]) * HKV + i / HD) * HD + i % HD];
    int32_t dims[BFP200_NSTAGES];
    bfp200_stage_dims(h, dims);
    size_t o = 0;
    for (int c = 0; c < ncols; ++c)
      for (int s = 0; s < BFP200_NSTAGES; ++s) {
        std::memcpy(stages + o, sink.st[s].data() + (size_t)c * dims[s], (size_t)dims[s] * 8);
        o += dims[s];
      }
  }
  if (read_and_clear_error_flag(h->stream)) return fail(BFP200_ETIMEOUT, "a bounded device wait timed out");
  return BFP200_OK;
}

}  // extern "C"
