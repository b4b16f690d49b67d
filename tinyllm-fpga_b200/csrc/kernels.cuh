// kernels.cuh -- argument structs and launchers for the BFP decode kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace bfp {

// One BFP weight matrix in the device layout used by bfp_matmul:
//   wm: [G][NT][2 planes][16 rows][16 k] bytes; plane 0 = m >> 8 (signed),
//       plane 1 = m & 0xFF (unsigned).  512 B per (row group, K tile).
//   we: [G][NT][16 rows] int8 tile exponents.
struct DevMat {
  const uint8_t* wm = nullptr;
  const int8_t* we = nullptr;
  int G = 0;    // row groups of 16 (rows = 16 G)
  int NT = 0;   // K tiles of 16 (K = 16 NT)
};

enum MatmulEpilogue : int {
  EPI_STORE = 0,     // out = quant(matvec)                      (q, k, v, generic)
  EPI_RESIDUAL = 1,  // out = quant(decode(res) + decode(quant(matvec)))   (:285, :293)
  EPI_SWIGLU = 2,    // groups (2i, 2i+1) = (g, u): out = requant(quant(quant(silu(g)) * u))  (:290-291)
};

struct MatmulArgs {
  DevMat W;
  // activations: column c at xm + c*x_ld (int16, K elements), xe + c*x_lde (int8, NT)
  const int16_t* xm = nullptr;
  const int8_t* xe = nullptr;
  int x_ld = 0, x_lde = 0;
  int ncols = 0;
  int epi = EPI_STORE;
  int16_t* om = nullptr;  // output mantissas, column stride o_ld
  int8_t* oe = nullptr;   // output exponents, column stride o_lde
  int o_ld = 0, o_lde = 0;
  const int16_t* rm = nullptr;  // residual (EPI_RESIDUAL), same layout as the output
  const int8_t* re = nullptr;
  long long* acc = nullptr;      // K-split scratch [rows][ncols_cap], zero between uses
  unsigned* counters = nullptr;  // K-split arrival counters, zero between uses
  int acc_ld = 0;                // columns per accumulator row
  int ksplit = 1;
  int cluster = 0;               // 1: the ksplit CTAs of a tile form a cluster and reduce through
                                 //    distributed shared memory (ksplit <= 8); 0: global atomics
  int rg = 1;                    // row groups per CTA (1, 2 or 4)
  int bn = 1;                    // columns per CTA
};

struct KvArena {
  int16_t* km = nullptr;  // [slot][layer][kvh][MAX_CTX][HD]
  int8_t* ke = nullptr;   // [slot][layer][kvh][MAX_CTX][HD/16]
  int16_t* vm = nullptr;
  int8_t* ve = nullptr;
  int NL = 0, HKV = 0, HD = 64, MAX_CTX = 0;
};

// Small-batch matvec family (gemv.cu), 1..4 columns.
enum GemvMode : int {
  GV_STORE = 0,     // out = quant(matvec)
  GV_RESIDUAL = 1,  // out = quant(res + quant(matvec))
  GV_SWIGLU = 2,    // interleaved gate/up groups -> requant(quant(quant(silu(g)) * u))
  GV_QKV_ROPE = 3,  // fused Q/K/V rows: RoPE on q/k heads, q -> qr buffer, k/v -> KV arena
};

struct GemvArgs {
  DevMat W;
  const int16_t* xm = nullptr;   // input columns (NORM: un-normalised)
  const int8_t* xe = nullptr;
  int x_ld = 0, x_lde = 0;
  int ncols = 0;
  int mode = GV_STORE;
  int norm = 0;                  // 1: tile_quantize(rmsnorm_fp(x, gamma)) prologue
  const double* gamma = nullptr;
  double eps = 1e-5;
  int16_t* om = nullptr;
  int8_t* oe = nullptr;
  int o_ld = 0, o_lde = 0;
  const int16_t* rm = nullptr;   // residual (GV_RESIDUAL)
  const int8_t* re = nullptr;
  // GV_QKV_ROPE
  const double* rope_cs = nullptr;
  const int* col_slot = nullptr;
  const int* col_pos = nullptr;
  KvArena kv;
  int layer = 0, HQ = 0, HKV = 0;
  int16_t* qr_m = nullptr;
  int8_t* qr_e = nullptr;
  // stage dump (bfp200_fwd_layer_decode), or nullptr; column c at + c * dbg_ld:
  // dbg_in: the normalised input (NORM, written by CTA 0); dbg_mid: the
  // matvec output before the residual (GV_RESIDUAL), q | k | v after RoPE
  // (GV_QKV_ROPE) or g (GV_SWIGLU); dbg_mid2: u (GV_SWIGLU)
  double* dbg_in = nullptr;
  double* dbg_mid = nullptr;
  double* dbg_mid2 = nullptr;
  int dbg_ld = 0;
};

// The attention half of a one-column decode layer in one launch of one
// thread-block cluster (layer1.cu): RMSNorm + Q/K/V + RoPE + KV write +
// attention + O + residual, h -> h1.
struct L1Args {
  DevMat Wqkv;                    // fused q | k | v rows of this layer (G = 4 (HQ + 2 HKV))
  DevMat Wo;                      // G = D / 16
  const double* gamma = nullptr;  // g1 of this layer, D doubles
  double eps = 1e-5;
  const int16_t* hm = nullptr;    // h (input), D mantissas + D/16 exponents
  const int8_t* he = nullptr;
  int16_t* h1m = nullptr;         // h1 (output)
  int8_t* h1e = nullptr;
  const double* rope_cs = nullptr;   // [MAX_CTX][32][cos, sin]
  const int* col_slot = nullptr;     // column 0's KV slot and position
  const int* col_pos = nullptr;
  KvArena kv;
  int layer = 0;
  const int* pw_off = nullptr;       // numpy pairwise-sum plans per length
  const unsigned short* pw_data = nullptr;
  int* err = nullptr;                // bounded-wait error flag
  int D = 0, HQ = 0, HKV = 0;
  double sqrt_hd = 8.0, inv_hd = 0.125;   // inv_hd: exact 1/sqrt(HD), or 0 when not a power of two
  // stage dump (bfp200_fwd_layer_decode), or nullptr: decoded n1, q, k, v,
  // attn, o, h1 at the stage offsets of that entry point's layout
  double* dbg = nullptr;
  // filled by attn_block_plan
  int og_other = 0, og_att = 0, ch = 0;
};
// Fills the plan fields; false when the configuration does not fit.
bool attn_block_plan(L1Args& a, int smem_budget);
size_t attn_block_smem(const L1Args& a);
cudaError_t launch_attn_block(const L1Args& a, cudaStream_t s, bool pdl);
cudaError_t init_attn_block_attributes(int smem_optin, int* dyn_budget);

// Batched BFP matvec on the tcgen05 tensor cores (tc.cu), for >= 64 columns.
// The weights are repacked once (launch_tc_pack) from DevMat into records of
// 128 rows x one K tile; rows are padded to a multiple of 128.
struct TcArgs {
  const uint8_t* rec = nullptr;   // records of one matrix (one layer), tc_records_bytes(rows, NT) bytes
  const int8_t* we = nullptr;     // the same matrix's DevMat tile exponents [G][NT][16]
  int rows = 0, NT = 0;
  const int16_t* xm = nullptr;    // input columns: column c at xm + c*x_ld, xe + c*x_lde
  const int8_t* xe = nullptr;
  int x_ld = 0, x_lde = 0;
  int ncols = 0;
  int mode = EPI_STORE;           // EPI_STORE / EPI_RESIDUAL / EPI_SWIGLU (rows interleave g/u groups)
  int16_t* om = nullptr;
  int8_t* oe = nullptr;
  int o_ld = 0, o_lde = 0;
  const int16_t* rm = nullptr;    // residual (EPI_RESIDUAL), output layout
  const int8_t* re = nullptr;
  int* err = nullptr;             // bounded-wait error flag
  int ncb = 0, ks = 0;            // columns per CTA (16 / 32) and K split (1..8); 0: built-in choice
  int ew = 0;                     // epilogue warps: 16 (0) or 8 (16 columns per CTA, two CTAs per SM)
};
size_t tc_records_bytes(int rows, int NT);
cudaError_t launch_tc_pack(const uint8_t* wm, const int8_t* we, int rows, int NT, uint8_t* rec, cudaStream_t s);
bool tc_supported(int NT, int ncols);
cudaError_t launch_tc_matmul(const TcArgs& a, cudaStream_t s, bool pdl);
bool tc_config_valid(int NT, int ncb, int ks);

// Device address of the flag that bounded waits set when they give up.
int* error_flag_device_ptr();

// Per-column descriptors of a forward pass.
struct ColDesc {
  const int* slot = nullptr;  // KV slot of the column
  const int* pos = nullptr;   // position (step) of the column
};


struct Dims {
  int D, HQ, HKV, HD, FFN, NL, VOCAB, MAX_CTX;
};

size_t matmul_smem_bytes(int rg, int bn, int ntc, int NT);
cudaError_t launch_matmul(const MatmulArgs& a, cudaStream_t s, bool pdl);
// The matmul reading weights in the reference's quantize_W layout
// (a.W.wm = int16 [rows][NT][16], a.W.we = int8 [rows][NT]); EPI_STORE only,
// rg 1 or 2, no programmatic dependent launch.
cudaError_t launch_matmul_refw(const MatmulArgs& a, cudaStream_t s);
size_t matmul_refw_smem_bytes(int rg, int bn, int ntc, int NT);
cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t s, bool pdl);
bool gemv_supported(int mode, bool norm, int NT, int ncols);
cudaError_t init_gemv_attributes();
// Raises the dynamic shared memory limit of every kernel (call once per device).
cudaError_t init_kernel_attributes();
// Launches a kernel that waits (at most limit_ns) for *flag to become non-zero
// and sets the bounded-wait error flag when it gives up (self-test).
cudaError_t launch_wait_probe(const int* flag, unsigned long long limit_ns, cudaStream_t s);
// Reads and clears the device flag a bounded wait sets when it gives up.
int read_and_clear_error_flag(cudaStream_t s);

cudaError_t launch_rmsnorm(const int16_t* xm, const int8_t* xe, const double* gamma, double eps,
                           int D, int ncols, int16_t* om, int8_t* oe, cudaStream_t s, bool pdl);
cudaError_t launch_rope_kv(const int16_t* qkv_m, const int8_t* qkv_e, int16_t* qr_m, int8_t* qr_e,
                           KvArena kv, int layer, ColDesc cols, const double* rope_cs, Dims d,
                           int ncols, cudaStream_t s, bool pdl);
// pw_off / pw_data: numpy pairwise-sum plans for lengths 1..MAX_CTX
// (build_pw_plan), or nullptr for the generic single-lane tree walk.
// early_kv: every column's K/V rows below its position were written by
// earlier launches (a decode step), so they are read before the dependency
// wait.
// qkv_m (non-null): the batched group kernel applies RoPE and writes the KV
// row itself from the fused q | k | v output (no rope_kv launch); only where
// attention_group_path() holds.
cudaError_t launch_attention(const int16_t* qr_m, const int8_t* qr_e, KvArena kv, int layer,
                             ColDesc cols, Dims d, int ncols, int16_t* am, int8_t* ae,
                             cudaStream_t s, bool pdl, const int* pw_off = nullptr,
                             const unsigned short* pw_data = nullptr, bool early_kv = false,
                             const int16_t* qkv_m = nullptr, const int8_t* qkv_e = nullptr,
                             const double* rope_cs = nullptr);
bool attention_group_path(Dims d, int ncols);
cudaError_t launch_embed(const int16_t* emb_m, const int8_t* emb_e, const int* tokens, int D,
                         int ncols, int16_t* hm, int8_t* he, cudaStream_t s, bool pdl);
cudaError_t launch_head_prep(const int16_t* hm, const int8_t* he, const double* norm_w, double eps,
                             int D, int ncols, double* hn, double* hn_norm, cudaStream_t s, bool pdl);
cudaError_t launch_head_logits(const int16_t* emb_m, const int8_t* emb_e, int VOCAB, int D,
                               const double* hn, int ncols, double* part_val, int* part_idx,
                               double* part_second, int* n_rowblocks, cudaStream_t s, bool pdl,
                               double* logits_out = nullptr);   // optional [ncols][VOCAB] logits
// Reduces per-row-block partials to the argmax; writes tok_out[c] and the
// certification flag (1 = the margin to the runner-up exceeds the fp64 dot
// error bound of any summation order).
cudaError_t launch_head_reduce(const double* part_val, const int* part_idx, const double* part_second,
                               int n_rowblocks, const double* hn_norm, double emb_norm_max, int D,
                               int ncols, int* tok_out, int* cert_out, cudaStream_t s, bool pdl,
                               int v_base = 0, double* xout = nullptr);
// Vocabulary sharding: with xout set, the head kernels write, per column,
// (best, global index = local + v_base, runner-up, ||hn||) to xout[4 c ..]
// instead of the token; head_combine reduces the records of all shards
// (rank-major [rank][column][4]) to the token and its certificate.
cudaError_t launch_head_combine(const double* gathered, int nranks, int ncols, double emb_norm_max, int D,
                                int VOCAB, int* tok_out, int* cert_out, cudaStream_t s);

// Head of 1..4 columns in one launch: hn, fp64 logits, and (last CTA) the
// certified argmax.  done_ctr: a zeroed word, left zeroed on return.
// Temperature / top-k sampling (sample.cu): one CTA per column reads the
// column's fp64 logits, the uniform of decode step *step + 1 and writes the
// token and its certificate.  work / cdf: [ncols][ld] doubles, incl:
// [ncols][ld] ints of scratch; plan: numpy's pairwise-sum plan for VOCAB.
struct SampleArgs {
  const double* logits = nullptr;
  int ld = 0, V = 0, D = 0;
  double temperature = 1.0;
  int top_k = 0;
  double* work = nullptr;
  double* cdf = nullptr;
  int* incl = nullptr;
  const unsigned short* plan = nullptr;
  const double* uniforms = nullptr;   // [ncols][u_ld]
  int u_ld = 0;
  const int* step = nullptr;
  const double* hn_norm = nullptr;
  double emb_norm_max = 0.0;
  int* tok = nullptr;
  int* cert = nullptr;
};
cudaError_t launch_sample(const SampleArgs& a, int ncols, int plan_leaves, cudaStream_t s);
// n uniforms of numpy's legacy generator after np.random.seed(seed)
void mt19937_uniforms(uint32_t seed, int n, double* out);

// Fixed-point ("rtl-exact") leaf ops of the FPGA modules (rtl.cu), batched;
// device pointers.  Layouts: tile-major mantissas [vec][D], tile exponents
// [vec][D/16]; matvec W [R][NT][16] + [R][NT], outputs [batch][R] with one
// exponent per element; rope exponents out [vec][HD] (per element); softmax
// one exponent per vector.
cudaError_t launch_rtl_matvec(const int16_t* xm, const int8_t* xe, const int16_t* wm, const int8_t* we, int R,
                              int NT, int batch, int16_t* ym, int8_t* ye, cudaStream_t s);
cudaError_t launch_rtl_rmsnorm(const int16_t* xm, const int8_t* xe, const int16_t* gm, const int8_t* ge, int D,
                               int nvec, int16_t* ym, int8_t* ye, cudaStream_t s);
cudaError_t launch_rtl_rope(const int16_t* xm, const int8_t* xe, const int* pos, const unsigned* turns, int HD,
                            int nvec, int16_t* ym, int8_t* ye, cudaStream_t s);
cudaError_t launch_rtl_softmax(const int16_t* xm, const int* xe, int n, int nvec, const uint16_t* lut, int16_t* ym,
                               int* ye, cudaStream_t s);
cudaError_t launch_rtl_swiglu(const int16_t* gm, const int8_t* ge, const int16_t* um, const int8_t* ue,
                              long long ntiles, const int16_t* lut, int16_t* ym, int8_t* ye, cudaStream_t s);
cudaError_t launch_rtl_residual(const int16_t* am, const int8_t* ae, const int16_t* bm, const int8_t* be,
                                long long ntiles, int16_t* ym, int8_t* ye, cudaStream_t s);

bool head_small_supported(int ncols, int D);
// The decode step's token feedback, done by the single-launch head's last CTA
// instead of a separate kernel: gen_out[c][*step] = token (step < n_gen),
// col_tok[c] = token, col_pos[c] += 1, uncertified decisions added to
// *uncert, *step += 1.  gen_out == nullptr: no feedback.
struct HeadAdvance {
  int* gen_out = nullptr;
  int* col_tok = nullptr;
  int* col_pos = nullptr;
  int* step = nullptr;
  long long* uncert = nullptr;
  int n_gen = 0;
};
cudaError_t launch_head_small(const int16_t* hm, const int8_t* he, const double* norm_w, double eps,
                              const int16_t* emb_m, const int8_t* emb_e, int VOCAB, int D, int ncols,
                              double emb_norm_max, double* part_val, int* part_idx, double* part_second,
                              unsigned* done_ctr, int* tok_out, int* cert_out, cudaStream_t s, bool pdl,
                              int v_base = 0, double* xout = nullptr, HeadAdvance adv = HeadAdvance());

// Standalone ops (the reference's module-level functions).
cudaError_t launch_tile_quantize(const double* v, long long ntiles, int16_t* m, int8_t* e, cudaStream_t s);
cudaError_t launch_tile_decode(const int16_t* m, const int8_t* e, long long ntiles, double* v, cudaStream_t s);
cudaError_t launch_rmsnorm_fp(const double* x, const double* gamma, double eps, int n, int ncols,
                              double* out, cudaStream_t s);
cudaError_t launch_silu_fp(const double* x, long long n, double* out, cudaStream_t s);
// numpy's float64 add.reduce (pairwise summation) of ncols rows of n values.
cudaError_t launch_np_sum(const double* x, int n, int ncols, double* out, cudaStream_t s);
// Same sum evaluated from a host-built plan of the pairwise tree (np_sum_warp_plan).
cudaError_t launch_np_sum_plan(const double* x, int n, int ncols, const unsigned short* plan, double* out,
                               cudaStream_t s);
cudaError_t launch_softmax_fp(const double* x, int n, int ncols, double* out, cudaStream_t s);
cudaError_t launch_rope_fp(const double* x, const double* cs, int HD, int nvec, double* out, cudaStream_t s);
// Converts reference-layout weights (m [R][NT][16], e [R][NT]) to DevMat layout.
// Destination row group of source group g is g * gstride + goff (interleaves
// the gate/up matrices as groups 2i / 2i+1).
cudaError_t launch_pack_weights(const int16_t* m_ref, const int8_t* e_ref, int R, int NT,
                                uint8_t* wm, int8_t* we, int gstride, int goff, cudaStream_t s);
// Converts the DDR3 wide-packed layout (entries [chunk][col][lane] int16 and
// [chunk][tile][lane] int8) to DevMat layout.
cudaError_t launch_pack_from_ddr(const int16_t* ddr_m, const int8_t* ddr_e, int R, int NT,
                                 uint8_t* wm, int8_t* we, int gstride, int goff, cudaStream_t s);
// L2-norm of each embedding row (for the head's error bound), in double.
cudaError_t launch_row_norms(const int16_t* m, const int8_t* e, int rows, int D, double* out, cudaStream_t s);

}  // namespace bfp
