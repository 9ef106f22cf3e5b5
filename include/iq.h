/*
 * iq.h -- C ABI of the B200 (sm_100a) Q16.48 integer inference library (libiq.so).
 *
 * The library replaces the hot path of int-llm's llama_int.c: the Q16.48
 * fixed-point matvec `matmul_vec` (llama_int.c:1014-1046) and the integer
 * Llama layer / forward / greedy generate around it (llama_int.c:1326-1569,
 * 2807-2886, 3067-3135). Every result is bit-identical to the CPU reference:
 * int64 x int64 products are summed exactly (mod 2^128) and the output is
 * low64(sum >> 48), an arithmetic (floor) shift with no rounding term.
 *
 * Conventions (kept from the reference):
 *   - fixed-point values are int64_t Q16.48 (fp_math.h:186, FP_PRECISION 48);
 *   - weights are row-major [M][N]: M = output rows, N = input length
 *     (llama_int.c:1014 argument order);
 *   - every entry point returns IQ_OK (0) or a negative iq_status; nothing
 *     in the library calls exit() or prints.
 * Pointers named d_* are device pointers; `stream` is a cudaStream_t passed
 * as void* (NULL = the library's own stream for the current device).
 */
#ifndef IQ_H
#define IQ_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define IQ_API __attribute__((visibility("default")))
#else
#define IQ_API
#endif

typedef enum iq_status {
    IQ_OK = 0,
    IQ_ERR_ARG = -1,          /* bad pointer / shape / argument */
    IQ_ERR_CUDA = -2,         /* CUDA runtime error (iq_last_cuda_error has the code) */
    IQ_ERR_OOM = -3,          /* device or host allocation failed */
    IQ_ERR_NCCL = -4,         /* NCCL error */
    IQ_ERR_TIMEOUT = -5,      /* a bounded device/host wait ran out */
    IQ_ERR_RANGE = -6,        /* token / position outside the model's range */
    IQ_ERR_STATE = -7,        /* object not in the state the call needs */
    IQ_ERR_UNSUPPORTED = -8   /* no device / not built for this GPU */
} iq_status;

/* fp_math function codes for iq_fp_dev (fp_math.h:491-921). */
typedef enum iq_fn {
    IQ_FN_MUL = 0, IQ_FN_DIV = 1, IQ_FN_SQRT = 2, IQ_FN_SQRT_FAST = 3, IQ_FN_INV_SQRT = 4,
    IQ_FN_EXP = 5, IQ_FN_LOG = 6, IQ_FN_COS = 7, IQ_FN_SIN = 8, IQ_FN_SIGMOID = 9,
    IQ_FN_SILU = 10, IQ_FN_SAFE_EXP = 11, IQ_FN_EXP_DYADIC = 12
} iq_fn;

/* ---------------------------------------------------------------- library */

IQ_API const char *iq_status_str(int status);
IQ_API int iq_last_cuda_error(void);     /* last cudaError_t seen by the library */
IQ_API int iq_version(void);             /* major*10000 + minor*100 + patch */
/* Selects the CUDA device used by host-pointer entry points (default 0) and
 * makes it current on the calling thread for the device entry points. */
IQ_API int iq_set_device(int device);

/* ------------------------------------------------ drop-in for matmul_vec */

/* Replaces `static void matmul_vec(fixed_t *out, const int64_t *weight,
 * const fixed_t *in, int M, int N)` (llama_int.c:1014-1015) with the same
 * argument order and meaning on HOST pointers: out[M] is written in full,
 * weight [M][N] and in[N] are read. Returns IQ_OK or an iq_status (the
 * reference returns void and has no error path).
 * Weights are uploaded to HBM on first use, packed and cached. A cached copy is
 * used only while the host matrix still holds what was uploaded (see
 * iq_weight_check_mode): the reference's streaming path frees each layer after
 * use and the next malloc can return the same address with other weights
 * (llama_int.c:2840-2872). Calls are not thread-safe against each other
 * (the reference is single-threaded); serialise them. */
IQ_API int iq_matmul_vec(int64_t *out, const int64_t *weight, const int64_t *in, int M, int N);

/* Explicit residency control for iq_matmul_vec's cache (no reference
 * counterpart: the reference reads weights in place from host memory). */
IQ_API int iq_weight_register(const int64_t *weight, int M, int N);
IQ_API int iq_weight_unregister(const int64_t *weight);
IQ_API int iq_weight_cache_clear(void);

/* How iq_matmul_vec decides that a cached copy still matches the host matrix:
 *   IQ_WCHECK_NONE    - by address and shape only (weights that never change:
 *                       mmap'd .mgw, --cache-layers);
 *   IQ_WCHECK_SAMPLED - (default) plus a 64-bit fingerprint of 1,152 fixed
 *                       positions, recomputed every call (microseconds); a
 *                       matrix that differs from the cached one in none of
 *                       those positions is not detected;
 *   IQ_WCHECK_FULL    - plus a hash of every value, every call (host memory
 *                       bandwidth); copies are also found by content, so the
 *                       streaming path's re-read layers hit the cache. */
enum { IQ_WCHECK_NONE = 0, IQ_WCHECK_SAMPLED = 1, IQ_WCHECK_FULL = 2 };
IQ_API int iq_weight_check_mode(int mode);
/* Device bytes the cache may hold (default 64 GiB); least recently used
 * entries are freed beyond it. */
IQ_API int iq_weight_cache_limit(int64_t bytes);
IQ_API int iq_weight_cache_stats(int *entries, int64_t *device_bytes);

/* ------------------------------------------------------- device kernels */

/* matmul_vec on device memory (llama_int.c:1014-1046): d_out[M] from
 * d_w [M][N] row-major and d_in[N]. d_out must not alias d_in. */
IQ_API int iq_matvec_dev(int64_t *d_out, const int64_t *d_w, const int64_t *d_in,
                         int M, int N, void *stream);

/* Weights repacked for the int8 tensor cores: each int64 weight split into
 * its bytes (byte planes), stored in mma fragment order, plus 128-bit row
 * sums. Only a window of planes is stored: the bytes no weight needs at the
 * top, and low bytes that few weights use, whose values go to an exact sparse
 * per-row residual (at most 8 bytes per weight in all). No reference
 * counterpart: the reference multiplies the int64 matrix directly
 * (llama_int.c:1014-1046). iq_matvec_packed_dev gives results bit-identical
 * to matmul_vec. */
typedef struct iq_packed iq_packed;
IQ_API int iq_pack_weights_dev(const int64_t *d_w, int M, int N, void *stream, iq_packed **out);
IQ_API int iq_packed_free(iq_packed *p);
/* The stored window: planes p0 .. p0 + np - 1 (bytes of each weight), and
 * the number of residual entries (weights with nonzero bytes below p0). */
IQ_API int iq_packed_info(const iq_packed *p, int *np, int *p0, int *residual_entries);
IQ_API int iq_matvec_packed_dev(int64_t *d_out, const iq_packed *w, const int64_t *d_in, void *stream);
/* Which stored form packing chose: IQ_FMT_PLANES (the byte-plane window
 * above) or IQ_FMT_BF16, two bytes per weight for matrices whose weights are
 * bf16 values (bfloat16_to_q1648, safetensors.h:115-152) of magnitude below
 * 0.25: each weight is kept as the bf16 number w / 2^48 and converted to its
 * byte planes inside the kernel, weights outside that form (at most 1 in
 * 1024) going whole to the exact sparse residual; chosen when it is smaller
 * and N <= 12768. Results are bit-identical either way. IQ_MV_FORMAT=planes
 * in the environment disables it. */
enum { IQ_FMT_PLANES = 0, IQ_FMT_BF16 = 1 };
IQ_API int iq_packed_format(const iq_packed *p, int *fmt);
/* iq_pack_weights_dev with the form given: -1 = chosen as above,
 * IQ_FMT_PLANES, or IQ_FMT_BF16 for any weights (those it cannot hold all go
 * to the residual; IQ_ERR_UNSUPPORTED when N > 12768). */
IQ_API int iq_pack_weights_fmt_dev(const int64_t *d_w, int M, int N, int fmt, void *stream, iq_packed **out);
/* Bytes of the stored form one iq_matvec_packed_dev launch reads (planes, row
 * sums, residual; not x or out): the numerator of its HBM roofline. */
IQ_API int iq_packed_bytes(const iq_packed *p, int64_t *bytes);

/* Same result as iq_matvec_packed_dev, but allocates no device memory: for
 * callers that cannot call cudaMalloc when they run (a process whose device
 * memory is owned by an external pool or budget, or a latency-critical loop
 * that must not hit an allocation's implicit synchronisation). No counterpart
 * in the reference, which has no device memory at all.
 * Its scratch is a fixed array inside the library, one per GPU, kept until the
 * process exits; it holds IQ_NOALLOC_MAX_ROWS = 32768 rows (the padded row
 * count, M rounded up to 16), and larger matrices are rejected with
 * IQ_ERR_RANGE. The first call on each device looks up and clears that array
 * (make it before any stream capture). All calls share the array: calls that
 * overlap on one GPU (on different streams, or issued from several host
 * threads) race and give wrong results; serialise them. */
IQ_API int iq_matvec_packed_noalloc_dev(int64_t *d_out, const iq_packed *w, const int64_t *d_in,
                                        void *stream);

/* Weights packed for the tcgen05 tensor-core GEMM (byte planes, row-major
 * per plane, plus a TMA descriptor); N (the reduction length) <= 32768.
 * iq_gemm_tc_dev: d_out[r][i] = matmul_vec(d_w, d_X[r])[i] for r < rows, the
 * same values as `rows` calls of llama_int.c:1014, on the int8 tensor cores.
 * No reference counterpart (the reference has no batched form). */
typedef struct iq_packed_tc iq_packed_tc;
IQ_API int iq_pack_weights_tc_dev(const int64_t *d_w, int M, int N, void *stream, iq_packed_tc **out);
IQ_API int iq_packed_tc_free(iq_packed_tc *p);
/* The GEMM form's stored window and residual size, as iq_packed_info (the
 * GEMM keeps a residual only when it is nearly empty: its epilogue pays more
 * per entry than the matvec's). */
IQ_API int iq_packed_tc_info(const iq_packed_tc *p, int *np, int *p0, int *residual_entries);
IQ_API int iq_gemm_tc_dev(int64_t *d_out, const iq_packed_tc *w, const int64_t *d_X, int rows, void *stream);

/* sample_token (llama_int.c:2958-3039) on the device for each row of
 * d_logits [rows][V]: temperature (Q16.48; below 0.01 the argmax), top-k (0 =
 * off), top-p (Q16.48; 0 or >= 1.0 = off), then a draw from the row's
 * xoroshiro128+ state rng [rows][2] (host, advanced in place exactly as the
 * reference advances sample_params_t.rng). out [rows] (host) receives the
 * token ids, identical to the reference's. */
IQ_API int iq_sample_dev(const int64_t *d_logits, int rows, int V, int64_t temperature, int top_k, int64_t top_p,
                         uint64_t *rng, int *out);
/* rng_seed (llama_int.c:2909-2919): SplitMix64 seeding of a state {s0, s1}. */
IQ_API int iq_rng_seed(uint64_t seed, uint64_t state[2]);

/* Synchronises the current device and returns (and clears) the status that
 * kernels with bounded waits record: IQ_OK or IQ_ERR_TIMEOUT. */
IQ_API int iq_device_status(void);
/* Self-test of that mechanism (no reference counterpart): launches one thread
 * that waits on an mbarrier nothing arrives at, giving up after limit_ns
 * (<= 100 ms). Returns IQ_OK when the wait gave up as designed; the status it
 * recorded (IQ_ERR_TIMEOUT) is then read and cleared by iq_device_status. */
IQ_API int iq_wait_selftest(int64_t limit_ns);
/* Measured ceiling for the GEMM roofline (no reference counterpart): one CTA
 * per SM issues iters x 4 tcgen05.mma.kind::i8 (M=128, N=256, K=32) on
 * shared-memory operands only; *tops = int8 tera-ops/s (2 per MAC), *ms the
 * kernel's CUDA-event time. */
IQ_API int iq_bench_i8_peak(int iters, double *tops, float *ms);

/* Batched rows: d_out[r][i] = matmul_vec(d_w, d_X[r])[i] for r < rows, i.e.
 * exactly `rows` independent calls of llama_int.c:1014 (the reference has no
 * batched form; its prefill loops M=1 calls, llama_int.c:3081-3092).
 * d_X is [rows][N], d_out is [rows][M]. */
IQ_API int iq_gemm_dev(int64_t *d_out, const int64_t *d_w, const int64_t *d_X,
                       int rows, int M, int N, void *stream);

/* Elementwise fp_math primitives on device (fp_math.h:491-921):
 * d_out[i] = fn(d_x[i], d_y[i]); d_y is read only by IQ_FN_MUL, IQ_FN_DIV and
 * IQ_FN_EXP_DYADIC (where d_y[i] is the round count k) and may be NULL otherwise. */
IQ_API int iq_fp_dev(int fn, const int64_t *d_x, const int64_t *d_y, int64_t *d_out,
                     int64_t n, void *stream);

/* rmsnorm (llama_int.c:1048-1058) of `rows` vectors of length dim. */
IQ_API int iq_rmsnorm_dev(int64_t *d_out, const int64_t *d_x, const int64_t *d_w,
                          int rows, int dim, void *stream);

/* softmax (llama_int.c:1060-1072), in place, on `rows` vectors of length n. */
IQ_API int iq_softmax_dev(int64_t *d_x, int rows, int n, void *stream);

/* ----------------------------------------------------------------- model */

/* llama_config_t (llama_int.c:788-798), same fields and meaning. */
typedef struct iq_config {
    int hidden_dim, num_heads, num_kv_heads, head_dim, num_layers;
    int intermediate_dim, vocab_size, max_seq_len, rope_theta;
} iq_config;

/* A device-resident integer Llama model (the reference's llama_model_t with
 * cached layers, llama_int.c:1575-1602): all weights in HBM, an exact int64
 * KV cache [layer][seq][max_seq_len][num_kv_heads*head_dim] for max_batch
 * sequences, RoPE tables built on the device by the fp_math ports
 * (rope_init, llama_int.c:960-986). One handle = one device, one stream;
 * calls on one handle must not overlap. */
typedef struct iq_model iq_model;

IQ_API int iq_model_create(const iq_config *cfg, int max_batch, int device, iq_model **out);

/* Tensor-parallel model: rank tp_rank of tp_size, one process (or thread) per
 * GPU, every rank calling every model entry point in lockstep. Each rank keeps
 * the output rows it owns of every projection (a contiguous block of q heads
 * with the kv heads they read, 1/tp_size of the rows of O, gate, up, down and
 * the LM head) and all-gathers each projection's output over NCCL, so results
 * are bit-identical to tp_size = 1. Load / synth calls take the FULL tensors;
 * each rank copies its rows. nccl_id: 128 bytes from iq_nccl_unique_id on one
 * rank, shared with the others (no reference counterpart: the reference is
 * single-threaded). num_heads, hidden_dim, intermediate_dim and vocab_size
 * must divide by tp_size. */
IQ_API int iq_nccl_unique_id(void *id_out);
/* Rows owned by tp_rank (host-only query, no device work): info = {first q
 * head, q heads, first kv head, kv heads, first O/down row, O/down rows, first
 * gate/up row, gate/up rows}; LM-head rows are [rank*V/P, (rank+1)*V/P). */
IQ_API int iq_tp_shard_info(const iq_config *cfg, int tp_size, int tp_rank, int info[8]);
IQ_API int iq_model_create_tp(const iq_config *cfg, int max_batch, int device, int tp_rank, int tp_size,
                              const void *nccl_id, iq_model **out);
IQ_API int iq_model_destroy(iq_model *m);
/* Global tensors from host memory: embed_tokens [vocab][dim], final norm [dim],
 * lm_head [vocab][dim] (llama_int.c:1575-1580; an untied head). */
IQ_API int iq_model_load_globals(iq_model *m, const int64_t *embed, const int64_t *final_norm,
                                 const int64_t *lm_head);
/* One layer's 9 tensors in layer_weights_t order (llama_int.c:1250-1260):
 * input_layernorm, q, k, v, o, post_attention_layernorm, gate, up, down. */
IQ_API int iq_model_load_layer(iq_model *m, int layer, const int64_t *const w[9]);
/* The configuration a model was created with. */
IQ_API int iq_model_config(const iq_model *m, iq_config *cfg);

/* int-llm's native .mgw container (llama_int.c:386-454). iq_mgw_read_config
 * reads its config block (so the caller can create a matching model, with or
 * without tensor parallelism); iq_model_load_mgw maps the file and loads every
 * tensor into the model as mgw_load does (llama_int.c:2344-2560: same header,
 * bounds and completeness checks; lm_head_tied uses the embedding), each rank
 * taking its own rows. IQ_ERR_ARG for a malformed file or one whose config
 * differs from the model's. */
IQ_API int iq_mgw_read_config(const char *path, iq_config *cfg, int *lm_head_tied);
IQ_API int iq_model_load_mgw(iq_model *m, const char *path);
/* Fills every weight with the seeded synthetic generator (below) for the
 * given config index, generating on `threads` host threads. */
IQ_API int iq_model_synth(iq_model *m, int config_index, int threads);
/* kv_cache_reset (llama_int.c:1160-1172) for every sequence. */
IQ_API int iq_model_reset(iq_model *m);

/* llama_forward (llama_int.c:2807-2886) for sequence 0: one token at pos.
 * logits (host, may be NULL) receives vocab_size values; *argmax_out (may be
 * NULL) the first-maximum index (llama_int.c:2888-2893). Returns IQ_ERR_RANGE
 * where the reference returns NULL (token or pos out of range). */
IQ_API int iq_forward(iq_model *m, int token, int pos, int64_t *logits, int *argmax_out);

/* generate() with greedy sampling (llama_int.c:3067-3135): resets the cache,
 * prefills prompt[0..prompt_len), decodes while i < max_new, stops at EOS (2).
 * out_tokens needs prompt_len + max_new entries; *n_out gets the reference's
 * return value (total length). logit_hash (may be NULL) receives FNV-1a-64
 * over every logit of every forward call in order (costs a logits copy per
 * step). */
IQ_API int iq_generate(iq_model *m, const int *prompt, int prompt_len, int max_new,
                       int *out_tokens, int *n_out, uint64_t *logit_hash);

/* generate() with sampling parameters (llama_int.c:3067-3135 with a
 * sample_params_t): temperature and top_p in Q16.48 (the values the reference
 * holds after parsing its CLI floats), top_k (0 = off), and the generator seed
 * (rng_seed once per call, llama_int.c:2909-2919). Every sample -- the one at
 * the end of the prompt and each decode step's -- is sample_token
 * (llama_int.c:2958-3039) computed on the device; tokens equal the
 * reference's. Other arguments as iq_generate. */
IQ_API int iq_generate_sampled(iq_model *m, const int *prompt, int prompt_len, int max_new, int64_t temperature,
                               int top_k, int64_t top_p, uint64_t seed, int *out_tokens, int *n_out,
                               uint64_t *logit_hash);

/* Batched greedy decode of B = max_batch independent sequences in lockstep
 * (the reference runs each sequence alone; rows are independent, so results
 * equal B separate generate() calls). prompts [B][prompt_len], out_tokens
 * [B][prompt_len + max_new], n_out[B]. logit_hashes (may be NULL) receives per
 * sequence the FNV-1a-64 over every logit of every forward that sequence's
 * generate() would run, as iq_generate's logit_hash (costs a logits copy per
 * step). */
IQ_API int iq_generate_batch(iq_model *m, const int *prompts, int prompt_len, int max_new,
                             int *out_tokens, int *n_out, uint64_t *logit_hashes);

/* Timing helper: runs `steps` greedy decode steps (graph replays) of all
 * max_batch sequences from position pos0 with no host synchronisation and no
 * EOS check, and returns the device time in *ms (CUDA events on the model's
 * stream). The cache must hold valid entries below pos0. */
IQ_API int iq_decode_steps_timed(iq_model *m, int pos0, int steps, float *ms);

/* Attention kernel choice (no reference counterpart: the arithmetic is the same
 * either way). Decode steps whose context length T = pos + 1 is at most
 * short_max use one CTA per (row, head); longer ones use the phased kernels
 * (tiles of 64 positions). 0 = always phased. Returns IQ_ERR_UNSUPPORTED if
 * the single-kernel form does not fit shared memory at this max_seq_len. */
IQ_API int iq_model_set_attention(iq_model *m, int short_max);

/* Decode-step implementation (no reference counterpart; identical bits either
 * way). mode 0 (default): one kernel per operation, the step captured in a
 * CUDA graph. mode 1: at batch 1 without tensor parallelism, when every decode
 * matrix is in the bf16 form, a decode step is ONE persistent cooperative
 * kernel (all SMs resident, grid-wide barriers between the layer's phases);
 * elsewhere mode 1 falls back to mode 0. On B200 mode 1 is slower today (each
 * barrier costs ~2.5 us and the phases are latency-bound), so it is off by
 * default. iq_model_decode_info reports whether the persistent kernel is in
 * use and its grid size. */
IQ_API int iq_model_set_decode(iq_model *m, int mode);

/* Packed KV cache, the reference's --kv-packed KbVb (llama_int.c:1078-1235,
 * 1392-1501): each (position, kv head) vector is stored as b-bit codes
 * against its L-inf magnitude, K codes of k_bits (1..8) in bytes, V codes of
 * v_bits (1..16) in 16-bit words, and attention reads the reconstructed
 * values. Lossy against the exact cache but the same integers as the
 * reference with the same flag, so tokens and logits still equal its output.
 * (0, 0) returns to the exact cache. Resets the cache; the persistent decode
 * kernel is not used in this mode. */
IQ_API int iq_model_set_kv_packed(iq_model *m, int k_bits, int v_bits);

/* Bounded host waits under tensor parallelism (no reference counterpart; the
 * reference has no collectives). Every host wait of a multi-GPU model polls
 * its stream together with NCCL's asynchronous error state; a communicator
 * error returns IQ_ERR_NCCL, and a step that does not finish within the
 * timeout (default 60 s: a peer rank that died or stopped calling) returns
 * IQ_ERR_TIMEOUT. Both abort the communicator (ncclCommAbort), which ends the
 * pending collectives; the model is then unusable (IQ_ERR_STATE) and must be
 * destroyed. iq_selftest_watchdog runs that wait logic on scripted events
 * without a GPU (scenario 0: completes; 1: communicator error; 2: never
 * completes; 3: stream error) and reports whether it aborted. */
IQ_API int iq_model_set_timeout(iq_model *m, int64_t ms);
/* Host-side liveness of the other tensor-parallel ranks (a store, heartbeat or
 * process table the host keeps): fn(ctx) is called at the start of every call
 * that launches work on a model with tp_size > 1; nonzero means a peer left,
 * and the call returns IQ_ERR_NCCL before enqueueing anything (no collective
 * is ever posted towards the missing rank); the model then refuses further
 * work (IQ_ERR_STATE) and iq_model_destroy aborts its communicator. fn NULL:
 * no check (the default; the bounded wait above still applies). */
IQ_API int iq_model_set_peer_check(iq_model *m, int (*fn)(void *ctx), void *ctx);
IQ_API int iq_selftest_watchdog(int scenario, int *aborted, int *polls);
IQ_API int iq_model_decode_info(iq_model *m, int *persistent, int *grid);
/* Diagnostics of the persistent kernel: microseconds per grid barrier with
 * `grid` CTAs (mode 0); and, with IQ_DEC_STAMPS set in the environment when
 * the model first prepares it, the last step's event times (ns since its
 * start, event tag in the top byte; slots 400+ / 700+ of a 1024-entry buffer:
 * per matvec phase the latest staging end / loop end over all warps). */
IQ_API int iq_bench_grid_sync(int grid, int iters, int mode, float *us);
IQ_API int iq_model_decode_stamps(iq_model *m, int64_t *out, int n);

/* Bytes of stored weights this rank's decode step reads per token at batch 1
 * (every projection's matvec form plus the LM head; not the KV cache), and the
 * bytes of the GEMM forms (prefill / batched decode). The numerators of the
 * decode roofline; no reference counterpart. */
IQ_API int iq_model_weight_bytes(iq_model *m, int64_t *decode_bytes, int64_t *gemm_bytes);

/* ------------------------------------------------ synthetic inputs (host) */

/* Seeded inputs of the synthetic benchmark configurations. No reference
 * counterpart as a function: the value path is the reference's own pieces --
 * xoroshiro128+/SplitMix64 (llama_int.c:2909-2929), a CLT-12 Gaussian shaped
 * like fp_gaussian (fp_math.h:944-952), bf16 rounding and bfloat16_to_q1648
 * (safetensors.h:115-152). seed = 0x494E544C4C4D0000 ^ (config << 32) ^
 * fnv1a64(tensor name). */
IQ_API uint64_t iq_tensor_seed(int config_index, const char *name);
IQ_API int iq_synth_weights(uint64_t seed, int64_t *out, int64_t n);  /* N(0,0.02), bf16-exact */
IQ_API int iq_synth_acts(uint64_t seed, int64_t *out, int64_t n);     /* uniform [-8, 8) */
IQ_API int iq_synth_tokens(uint64_t seed, int *out, int n, int vocab);
/* bfloat16_to_q1648 (safetensors.h:115-152) and its round-to-nearest-even inverse. */
IQ_API int64_t iq_bf16_to_q1648(uint16_t bits);
IQ_API uint16_t iq_q1648_to_bf16(int64_t q);

#ifdef __cplusplus
}
#endif
#endif /* IQ_H */
