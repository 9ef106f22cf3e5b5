// iq_elem.cuh -- elementwise and row-wise kernels built on the fp_math ports:
// vector fp_math evaluation, rmsnorm (llama_int.c:1048-1058) and softmax
// (llama_int.c:1060-1072).
#pragma once
#include "iq_fpmath.cuh"
#include "iq_matvec.cuh"

namespace iq {

// CORDIC tables live in device memory, written once per device by k_cordic_init.
__device__ CordicTables g_cordic;

__global__ void k_cordic_init() {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        CordicTables t;
        d_cordic_init(&t);
        g_cordic = t;
    }
}

__device__ __forceinline__ int64_t d_eval(int fn, int64_t x, int64_t y, const CordicTables &ct) {
    int64_t c, s;
    switch (fn) {
    case IQ_FN_MUL: return d_mul(x, y);
    case IQ_FN_DIV: return d_div(x, y);
    case IQ_FN_SQRT: return d_sqrt(x);
    case IQ_FN_SQRT_FAST: return d_sqrt_fast(x);
    case IQ_FN_INV_SQRT: return d_inv_sqrt(x);
    case IQ_FN_EXP: return d_exp(x);
    case IQ_FN_LOG: return d_log(x);
    case IQ_FN_COS: d_sincos(ct, x, &c, &s); return c;
    case IQ_FN_SIN: d_sincos(ct, x, &c, &s); return s;
    case IQ_FN_SIGMOID: return d_sigmoid(x);
    case IQ_FN_SILU: return d_silu(x);
    case IQ_FN_SAFE_EXP: return d_safe_exp(x);
    case IQ_FN_EXP_DYADIC: return d_exp_dyadic(x, (int)y);
    default: return 0;
    }
}

__global__ void k_fp_eval(int fn, const int64_t *__restrict__ x, const int64_t *__restrict__ y,
                          int64_t *__restrict__ out, int64_t n) {
    const CordicTables &ct = g_cordic;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = d_eval(fn, x[i], y ? y[i] : 0, ct);
}

// CTA-wide 128-bit sum (all threads receive it). red must hold 2*32 words.
__device__ __forceinline__ i128 cta_sum_i128(i128 v, uint64_t *red) {
    v = warp_sum_i128(v);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (l == 0) { red[2 * w] = (uint64_t)v; red[2 * w + 1] = (uint64_t)((u128)v >> 64); }
    __syncthreads();
    i128 t = 0;
    for (int i = 0; i < nw; i++) t += (i128)(((u128)red[2 * i + 1] << 64) | red[2 * i]);
    return t;
}

__device__ __forceinline__ int64_t cta_max_i64(int64_t v, int64_t *red) {
    for (int m = 16; m >= 1; m >>= 1) v = max(v, (int64_t)__shfl_xor_sync(0xffffffffu, v, m));
    int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    int64_t t = red[0];
    for (int i = 1; i < nw; i++) t = max(t, red[i]);
    return t;
}

// rmsnorm inverse-rms factor for one vector (the CTA cooperates):
// int128 sum of squares, (sum >> 48) / dim truncating, + eps, fp_inv_sqrt.
__device__ __forceinline__ int64_t cta_rms_inv(const int64_t *x, int dim, uint64_t *red) {
    i128 ss = 0;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += (i128)x[i] * x[i];
    ss = cta_sum_i128(ss, red);
    int64_t ms = (int64_t)d_sdiv128_64(ss >> 48, dim);
    ms += (int64_t)2814749767LL;  // 1e-5 in Q16.48 (llama_int.c:1053)
    return d_inv_sqrt(ms);
}

__global__ void k_rmsnorm(int64_t *__restrict__ out, const int64_t *__restrict__ x,
                          const int64_t *__restrict__ w, int dim) {
    __shared__ uint64_t red[64];
    const int64_t *xr = x + (size_t)blockIdx.x * dim;
    int64_t *orow = out + (size_t)blockIdx.x * dim;
    int64_t inv = cta_rms_inv(xr, dim, red);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) orow[i] = d_mul(d_mul(xr[i], inv), w[i]);
}

// softmax of one row held in global memory (in place).
__device__ __forceinline__ void cta_softmax(int64_t *v, int n, uint64_t *red) {
    int64_t mx = INT64_MIN;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = max(mx, v[i]);
    mx = cta_max_i64(mx, (int64_t *)red);
    uint64_t s = 0;  // int64 sum with wrap, kept unsigned
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        int64_t e = d_safe_exp((int64_t)((uint64_t)v[i] - (uint64_t)mx));
        v[i] = e;
        s += (uint64_t)e;
    }
    int64_t sum = (int64_t)(uint64_t)cta_sum_i128((i128)(u128)s, red);
    if (sum > 0)
        for (int i = threadIdx.x; i < n; i += blockDim.x) v[i] = d_div(v[i], sum);
}

__global__ void k_softmax(int64_t *__restrict__ x, int n) {
    __shared__ uint64_t red[64];
    cta_softmax(x + (size_t)blockIdx.x * n, n, red);
}

}  // namespace iq
