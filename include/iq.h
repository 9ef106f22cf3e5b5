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
 * weight [M][N] and in[N] are read. Weights are uploaded to HBM on first use
 * and cached, keyed by (weight, M, N); like the reference's loaded weights
 * (llama_int.c:2464) they must not change afterwards -- call
 * iq_weight_unregister first if they do. Returns IQ_OK or an iq_status
 * (the reference returns void and has no error path). */
IQ_API int iq_matmul_vec(int64_t *out, const int64_t *weight, const int64_t *in, int M, int N);

/* Explicit residency control for iq_matmul_vec's cache (no reference
 * counterpart: the reference reads weights in place from host memory). */
IQ_API int iq_weight_register(const int64_t *weight, int M, int N);
IQ_API int iq_weight_unregister(const int64_t *weight);
IQ_API int iq_weight_cache_clear(void);

/* ------------------------------------------------------- device kernels */

/* matmul_vec on device memory (llama_int.c:1014-1046): d_out[M] from
 * d_w [M][N] row-major and d_in[N]. d_out must not alias d_in. */
IQ_API int iq_matvec_dev(int64_t *d_out, const int64_t *d_w, const int64_t *d_in,
                         int M, int N, void *stream);

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
