/* bfp200.h -- C ABI of libbfp200.so, the B200 (sm_100a) implementation of the
 * block-floating-point (BFP) SmolLM2-135M greedy decode path of
 * jrrk2/tinyllm-fpga.
 *
 * The reference has no FFI on this path: its surfaces are the Python module
 * rtl/vc707/host/gen_smollm_blockfp_full.py (packer + bit-exact simulator)
 * and the files the packers write (<PREFIX>DDR3.bin, <PREFIX>*_m/_e.hex,
 * <PREFIX>PROMPT.hex) that rtl/vc707/host/bfp_client.cpp uploads.  Each entry
 * point below names the reference interface it replaces.
 *
 * Conventions: every function returns 0 on success or a negative BFP200_E*
 * code; bfp200_last_error() gives the message of the calling thread's last
 * failure.  All pointers are HOST pointers unless a name ends in _dev.  A
 * handle owns one CUDA device, one stream and all device memory it needs;
 * one call may be in flight per handle, handles on different devices (or
 * threads) are independent.  Nothing here falls back to the CPU: without a
 * usable sm_100 device bfp200_open fails with BFP200_ENODEV.
 */
#ifndef BFP200_H
#define BFP200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  BFP200_OK = 0,
  BFP200_EINVAL = -1,    /* bad argument (shape, length, range) */
  BFP200_ENODEV = -2,    /* no usable CUDA device */
  BFP200_ECUDA = -3,     /* CUDA runtime error */
  BFP200_EIMAGE = -4,    /* image / ROM content does not match the config */
  BFP200_ESTATE = -5,    /* call order (e.g. generate before load_image) */
  BFP200_ETIMEOUT = -6,  /* a bounded device-side wait gave up */
  BFP200_ENOMEM = -7,    /* device allocation failed */
};

/* Model / run configuration.  Field names follow the reference's environment
 * variables (gen_smollm_blockfp_full.py:53-64, gen_smollm_blockfp_cfg.py:44). */
typedef struct bfp200_cfg {
  int D;            /* model width (576) */
  int H_Q;          /* query heads (9) */
  int H_KV;         /* key/value heads (3) */
  int HD;           /* head dim (64; the only supported value) */
  int FFN;          /* MLP width (1536) */
  int NL;           /* layers (30) */
  int VOCAB;        /* vocabulary rows in the image (49152, multiple of 16) */
  int MAX_CTX;      /* KV positions per sequence (<= 3072) */
  int NPROMPT_MAX;  /* longest prompt accepted (48) */
  int max_seqs;     /* sequences one generate call may carry */
  double rope_base; /* 10000.0: the simulator's rope_fp default (:250) */
  double eps;       /* 1e-5 (:236, :438) */
} bfp200_cfg;

typedef struct bfp200_handle bfp200_handle;

/* Fills *cfg with the SmolLM2-135M defaults of the reference. */
void bfp200_default_cfg(bfp200_cfg* cfg);

/* Text of the calling thread's last error. */
int bfp200_last_error(char* buf, size_t len);

/* Replaces: the reference's process-level setup (module import, :53-85). */
int bfp200_open(const bfp200_cfg* cfg, int device, bfp200_handle** out);
int bfp200_close(bfp200_handle* h);

/* Replaces: `bfp_client upload <DDR3.bin>` (bfp_client.cpp:1696-1701) feeding
 * the DDR3 image written by gen_smollm_blockfp_ddr.py:155-241 (region order
 * and 4 KiB alignment of lbfp_ddr3.svh:45-86).  The buffer is only read
 * during the call. */
int bfp200_load_image(bfp200_handle* h, const void* ddr3_bin, size_t len);

/* Replaces: `bfp_client load-roms` (bfp_client.cpp:1381-1437) -- same kind
 * numbering: 0 G1_m, 1 G1_e, 2 G2_m, 3 G2_e, 4 NORM_W_m, 5 NORM_W_e,
 * 6 PROMPT.  Entries are the 16-bit values of the .hex lines
 * (parse_hex_file, :1162-1183); exponents use the low 8 bits. */
int bfp200_load_rom(bfp200_handle* h, int kind, const uint16_t* entries, size_t n);

/* Replaces: the golden driver loop of gen_smollm_blockfp_full.py:425-449
 * (feed_mode 0 = "sim": prompt + n_gen ids, the argmax of the last prompt
 * step is discarded and the last prompt token is fed again) or the RTL feed
 * rule of autoregress_bfp_top.sv:358-384 (feed_mode 1 = "rtl": one argmax
 * per step, len + n_gen ids).
 *   prompt_ids   concatenated prompts (NULL: the ROM prompt, n_seq must be 1)
 *   prompt_lens  n_seq lengths, 1..NPROMPT_MAX (NULL with prompt_ids NULL)
 *   out_tokens   concatenated per-sequence outputs of len_i + n_gen ids
 * Requires len_i + n_gen <= MAX_CTX. */
int bfp200_generate(bfp200_handle* h, const int32_t* prompt_ids, const int32_t* prompt_lens, int n_seq, int n_gen,
                    int feed_mode, int32_t* out_tokens);

/* Replaces: the sampling head of the hardware emulator
 * (sim_rtl_fp_hw.py:204-216: TEMP / TOPK / SEED): scaled = logits / T, the
 * TOPK largest kept (TOPK 0 = all), p = softmax with numpy's pairwise sum,
 * token = np.random.choice(p) (cdf = sequential cumsum, searchsorted of one
 * random_sample).  Sequence s draws from np.random.seed(seed + s)'s stream
 * (sequence 0 = the reference's SEED); like the reference, one draw is made
 * and discarded at the last prompt position.  Feed rule "sim".  Among
 * logits equal to the TOPK-th largest the lowest ids are kept.  temperature
 * <= 0 is greedy decoding.  A draw whose u lies within the head's fp64
 * error bound of a cdf step is counted by bfp200_uncertified_steps. */
int bfp200_generate_sampled(bfp200_handle* h, const int32_t* prompt_ids, const int32_t* prompt_lens, int n_seq,
                            int n_gen, double temperature, int top_k, uint32_t seed, int32_t* out_tokens);
/* The uniforms the sampled decode draws for one sequence: the first n values
 * of np.random.seed(seed); np.random.random_sample() (host only, no device). */
int bfp200_sample_uniforms(uint32_t seed, int n, double* out);

/* Same as bfp200_generate, with the sequences split into contiguous blocks
 * over n_dev handles (one per GPU), run concurrently with no collectives.
 * Replaces: nothing in the reference (single FPGA, single stream). */
int bfp200_generate_multi(bfp200_handle* const* hs, int n_dev, const int32_t* prompt_ids, const int32_t* prompt_lens,
                          int n_seq, int n_gen, int feed_mode, int32_t* out_tokens);

/* Vocabulary-sharded head (single-stream latency over several GPUs).  Every
 * rank runs all layers on the same sequences; rank r scans embedding rows
 * [r V / n, (r+1) V / n) and the ranks exchange one (max logit, lowest index,
 * runner-up, ||hn||) record per sequence with an NCCL all-gather on the
 * handle's stream (captured in the decode graph), then every rank combines
 * them into the argmax of the whole vocabulary (np.argmax semantics,
 * gen_smollm_blockfp_full.py:439-440: lowest index on ties).  NCCL is loaded
 * at run time (libnccl.so.2 already in the process, else $BFP200_NCCL_LIB,
 * else the loader's search path); NVLS is left off unless NCCL_NVLS_ENABLE
 * is set, and peers connect at communicator creation unless
 * NCCL_RUNTIME_CONNECT is set (the first exchange then never blocks the host
 * inside a graph capture).  Joining a group makes one exchange.  A sharded
 * handle's generate must be called on every rank with the same arguments;
 * it runs one decode step at a time and waits for each with a poll limited
 * to $BFP200_NCCL_TIMEOUT_S seconds (default 120).  Past the limit (a rank
 * that never joins the step) or on an NCCL error it aborts the communicator
 * (ncclCommAbort), waits at most 30 s for the stream to drain and returns
 * BFP200_ETIMEOUT with the handle back to an unsharded head; if the stream
 * does not drain, the call still returns BFP200_ETIMEOUT and the handle is
 * marked unusable (later calls fail with BFP200_ESTATE) -- no call on this
 * path waits without a limit.  ncclCommInitRank itself (bfp200_head_shard)
 * blocks until every rank has joined.
 * Replaces: nothing in the reference (single FPGA, unsharded head :437-440). */
#define BFP200_NCCL_ID_BYTES 128
/* A fresh NCCL unique id (rank 0 makes it, every rank passes it to
 * bfp200_head_shard). */
int bfp200_nccl_unique_id(uint8_t* id);
/* Joins rank `rank` of an `nranks`-rank vocabulary-sharded head (blocks until
 * every rank has joined).  id == NULL with nranks == 1 leaves sharding; a
 * one-rank group (id given, nranks == 1) runs the sharded head path over the
 * whole vocabulary. */
int bfp200_head_shard(bfp200_handle* h, const uint8_t* id, int nranks, int rank);
/* One process, n_dev handles on distinct devices: shards the head over all
 * of them (rank = position in hs). */
int bfp200_head_shard_group(bfp200_handle* const* hs, int n_dev);
/* Runs bfp200_generate on every handle of a sharded group concurrently (one
 * host thread each) and returns rank 0's tokens after checking that every
 * rank produced the same ones. */
int bfp200_generate_sharded(bfp200_handle* const* hs, int n_dev, const int32_t* prompt_ids,
                            const int32_t* prompt_lens, int n_seq, int n_gen, int feed_mode, int32_t* out_tokens);

/* Measurement: bfp200_matvec whose device time (the matvec launch alone,
 * after one untimed call) is averaged over `reps` back-to-back repetitions;
 * outputs as bfp200_matvec.  No reference counterpart (cfg4 sweep timing). */
int bfp200_matvec_timed(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* W_m,
                        const int8_t* W_e, int D_out, int D_in, int batch, int reps, int16_t* out_m, int8_t* out_e,
                        double* ms_per_call);

/* Fixed-point ("rtl-exact") leaf ops: the integer arithmetic of the FPGA
 * modules, as pinned by the reference's per-op golden generators
 * (rtl/vc707/host/gen_*_bfp_golden.py).  Host buffers; tiles of 16
 * elements; vectors are contiguous ([vec][D] mantissas, [vec][D/16] tile
 * exponents).  The ROMs are the caller's (as the RTL's $readmemh files):
 * exp_lut = exp_lut.hex (1024 x Q1.15), silu_lut = silu_lut.hex (65536 x
 * int16), turns_q31 = rope_freq_turns.svh (HD/2 x Q0.31).
 * Replaces: matvec_bfp_engine.sv via gen_matvec_bfp_golden.py:49-104 -- a
 * running-alignment 48-bit accumulation, one exponent per OUTPUT element
 * (y_e has D_out entries per column); W_m is [D_out][D_in/16][16]. */
int bfp200_rtl_matvec(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* W_m, const int8_t* W_e,
                      int D_out, int D_in, int batch, int16_t* y_m, int8_t* y_e);
/* Replaces: rmsnorm_bfp.sv via gen_rmsnorm_bfp_golden.py:43-144 (Newton-Raphson
 * 1/sqrt from a seed table, Q12.12). */
int bfp200_rtl_rmsnorm(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* g_m, const int8_t* g_e,
                       int D, int nvec, int16_t* y_m, int8_t* y_e);
/* Replaces: rope_bfp.sv via gen_rope_bfp_golden.py:25-124 (CORDIC sin/cos);
 * y_e has one exponent per ELEMENT ([vec][HD]). */
int bfp200_rtl_rope(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int32_t* pos, int nvec, int HD,
                    const uint32_t* turns_q31, int16_t* y_m, int8_t* y_e);
/* Replaces: softmax_bfp.sv via gen_softmax_bfp_golden.py:34-83; one shared
 * exponent per vector in and out (x_e, y_e: nvec entries). */
int bfp200_rtl_softmax(bfp200_handle* h, const int16_t* x_m, const int32_t* x_e, int n, int nvec,
                       const uint16_t* exp_lut, int16_t* y_m, int32_t* y_e);
/* Replaces: swiglu_bfp.sv via gen_swiglu_bfp_golden.py:45-77; n elements. */
int bfp200_rtl_swiglu(bfp200_handle* h, const int16_t* gate_m, const int8_t* gate_e, const int16_t* up_m,
                      const int8_t* up_e, size_t n, const int16_t* silu_lut, int16_t* y_m, int8_t* y_e);
/* Replaces: the residual adder via gen_residual_bfp_golden.py:20-45. */
int bfp200_rtl_residual(bfp200_handle* h, const int16_t* a_m, const int8_t* a_e, const int16_t* b_m,
                        const int8_t* b_e, size_t n, int16_t* y_m, int8_t* y_e);

/* Number of head argmax decisions of the last generate call whose fp64
 * margin did not certify agreement with every summation order (0 means the
 * token stream is independent of the reference's BLAS). */
int bfp200_uncertified_steps(bfp200_handle* h, long long* count);

/* Device time of the last generate call's phases, in milliseconds. */
int bfp200_last_timing(bfp200_handle* h, double* prefill_ms, double* decode_ms);

/* Self-test of the device-side bounded waits: launches a kernel that waits
 * for a flag nothing sets, gives up after limit_ms (1..2000) milliseconds,
 * records the timeout in the library's device error flag like every other
 * bounded wait (TMA barrier and tensor-memory waits), and returns; the call
 * then reports BFP200_ETIMEOUT and the handle stays usable.  No reference
 * counterpart: test support. */
int bfp200_wait_probe(bfp200_handle* h, int limit_ms);

/* Number of kernels the last bfp200_generate launched on the device (prefill
 * launches, plus one decode step's launches times n_gen).  No reference
 * counterpart: measurement support. */
int bfp200_last_launches(bfp200_handle* h, long long* launches);

/* Measurement: device time of one token's BFP matmuls (the 4 per layer of
 * every layer, production epilogues, `ncols` columns), replayed `reps` times
 * from a CUDA graph on the handle's stream between CUDA events.  Requires a
 * loaded image.  Replaces nothing in the reference. */
int bfp200_time_matmuls(bfp200_handle* h, int ncols, int reps, double* ms_per_token, int* launches_per_token);

/* Measurement: one forward pass (embedding, every layer, head) of `ncols`
 * columns at position `pos`, launched without programmatic overlap and with
 * a CUDA event before every kernel; per kernel kind k (0 embed, 1 rmsnorm,
 * 2 qkv matmul, 3 rope+kv, 4 attention, 5 o matmul, 6 gate/up matmul,
 * 7 down matmul, 8 head prep, 9 head logits, 10 head reduce) returns the
 * summed milliseconds and launch count (arrays of 11).  The KV content is
 * whatever the slots hold.  Replaces nothing in the reference. */
int bfp200_profile_forward(bfp200_handle* h, int ncols, int pos, double* ms_by_kind, int* launches_by_kind);

/* ---- op-level entry points (the reference's module functions) ---------- */

/* tile_quantize (gen_smollm_blockfp_full.py:90-97): n doubles (n % 16 == 0)
 * -> m[n] int16, e[n/16] int8. */
int bfp200_tile_quantize(bfp200_handle* h, const double* v, size_t n, int16_t* m, int8_t* e);
/* tile_decode (:100-102). */
int bfp200_tile_decode(bfp200_handle* h, const int16_t* m, const int8_t* e, size_t n, double* v);

/* matvec_hw_golden (:217-233) on `batch` independent columns.
 *   x_m [batch][D_in], x_e [batch][D_in/16]; W_m [D_out][D_in/16][16],
 *   W_e [D_out][D_in/16] (the reference's quantize_W layout);
 *   out_m [batch][D_out], out_e [batch][D_out/16] = tile_quantize of the
 *   result (decode gives the reference's fp_quantize_vec(out_real)).
 * Runs the kernel a decode step would use at this column count: the
 * small-batch GEMV at 1..4 columns, the tensor-core matmul from 16, the dp2a
 * matmul in between. */
int bfp200_matvec(bfp200_handle* h, const int16_t* x_m, const int8_t* x_e, const int16_t* W_m, const int8_t* W_e,
                  int D_out, int D_in, int batch, int16_t* out_m, int8_t* out_e);

/* rmsnorm_fp (:236-238) on ncols vectors of n doubles. */
int bfp200_rmsnorm_fp(bfp200_handle* h, const double* x, const double* gamma, int n, int ncols, double eps,
                      double* out);
/* silu_fp (:241-242), n % 16 == 0. */
int bfp200_silu_fp(bfp200_handle* h, const double* x, size_t n, double* out);
/* softmax_fp (:245-247) on ncols vectors of n doubles. */
int bfp200_softmax_fp(bfp200_handle* h, const double* x, int n, int ncols, double* out);
/* numpy's float64 reduction np.add.reduce / np.mean's sum (pairwise
 * summation), the order rmsnorm_fp (:237), softmax_fp (:247) and the head
 * (:438) sum in; ncols rows of n <= 3072 doubles. */
int bfp200_pairwise_sum(bfp200_handle* h, const double* x, int n, int ncols, double* out);
/* rope_fp (:250-258) on nvec vectors of HD doubles at positions pos[]. */
int bfp200_rope_fp(bfp200_handle* h, const double* x, const int32_t* pos, int nvec, int HD, double base,
                   double* out);
/* The (cos, sin) pairs rope_fp evaluates (:253-254), [n_pos][HD/2][2],
 * computed with the host libm exactly as Python's math module does. */
int bfp200_rope_table(double* out, int n_pos, int HD, double base);

/* One layer, fwd_layer (:261-293), for ncols independent columns using
 * layer `layer` of the loaded image.  h_in/h_out are [ncols][D] doubles on
 * the BFP grid.  k_cache/v_cache are the reference's per-layer float64
 * caches [ncols][max_ctx][H_KV][HD]: positions < kv_pos[c] are read, slot
 * kv_pos[c] is written back (fwd_layer mutates kv in place, :270-272).
 * pos[c] is the RoPE position.  If stages is non-NULL it receives, per
 * column, BFP200_NSTAGES vectors of D_stage doubles (see bfp200_stage_dims). */
int bfp200_fwd_layer(bfp200_handle* h, int layer, const double* h_in, const int32_t* pos, const int32_t* kv_pos,
                     int ncols, double* k_cache, double* v_cache, int max_ctx, double* h_out, double* stages);

/* No counterpart in the reference.  bfp200_matvec for callers that cannot
 * allocate device memory -- a framework that owns every byte through its own
 * caching allocator or fixed pool, or a latency-critical loop that cannot
 * take cudaMalloc/cudaFree's implicit device synchronisation.  Every pointer
 * is a DEVICE pointer on the current device, in the layouts of
 * bfp200_matvec; x_m and W_m must be 16-byte aligned and out_m 2-byte
 * aligned (otherwise BFP200_EINVAL, before anything runs).  The call is
 * asynchronous on `stream` (a cudaStream_t, NULL for the default stream) and
 * allocates nothing.  Its scratch (the matmul's K-split accumulators and
 * counters) is a fixed file-scope device array of 2 MiB + 64 KiB that every
 * GPU loading the library holds until exit: D_out * batch must not exceed
 * 262144 (larger sizes fail with BFP200_EINVAL).  The first call on a device
 * does a one-time set-up (it looks up the scratch array's device address and
 * sets kernel attributes), so make that first call before any stream
 * capture, and after any cudaDeviceReset (a reset discards the set-up's
 * results; the library does not notice).  Each process has its own copy of
 * the scratch on each device, and every call in that process on that device
 * shares it: calls that overlap on the GPU (different streams or threads of
 * one process, same device) race and must be serialised by the caller. */
int bfp200_matvec_noalloc(const int16_t* x_m, const int8_t* x_e, const int16_t* W_m, const int8_t* W_e, int D_out,
                          int D_in, int batch, int16_t* out_m, int8_t* out_e, void* stream);

/* bfp200_fwd_layer through the kernels a decode step uses for 1..4 columns
 * (gen_smollm_blockfp_full.py:261-293, the same contract as bfp200_fwd_layer):
 * at one column the fused attention-block launch plus the gate/up and down
 * launches, at 2..4 columns the five small-batch launches.  Each kernel
 * writes the stages it computes into the stage dump, so every intermediate
 * tensor of the production decode path can be compared with the
 * simulator's.  ncols must be 1..4 (BFP200_EINVAL otherwise). */
int bfp200_fwd_layer_decode(bfp200_handle* h, int layer, const double* h_in, const int32_t* pos,
                            const int32_t* kv_pos, int ncols, double* k_cache, double* v_cache, int max_ctx,
                            double* h_out, double* stages);

/* Stage dump layout of bfp200_fwd_layer (mirrors the N1..D dumps of
 * gen_smollm_blockfp_bfp.py:393-426): n1 q k v attn o h1 n2 g u mlp d, where
 * n1/n2/attn/mlp are the matvec inputs tile_quantize(.) decoded, q/k are
 * post-RoPE and every other stage is the matvec output. */
#define BFP200_NSTAGES 12
int bfp200_stage_dims(bfp200_handle* h, int32_t* dims_out /* [BFP200_NSTAGES] */);

#ifdef __cplusplus
}
#endif
#endif /* BFP200_H */
