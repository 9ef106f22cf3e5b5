// iq_matvec.cuh -- M=1 Q16.48 matvec (matmul_vec, llama_int.c:1014-1046) on
// sm_100a CUDA cores.
//
// Exact arithmetic without 128-bit multiplies in the inner loop
// ---------------------------------------------------------------
// For x = in[j] and w = W[i][j] (both int64) write
//   x = a0 + a1*2^22 + a2*2^43     a0 in [0,2^22), a1 in [0,2^21), a2 = x>>43 in [-2^20,2^20)
//   w = wh*2^32 + wl               wh = w>>32 (signed), wl = low word (unsigned)
//   wl = ws + 2^31                 ws = wl ^ 0x80000000 read as int32
// so x*w = sum_k 2^{p_k} a_k (wh*2^32 + ws) + 2^31 x,  p = {0, 22, 43}.
// Every a_k*wh and a_k*ws is an int32 x int32 product of magnitude < 2^53,
// summed by one IMAD.WIDE into an int64 accumulator; 1024 such terms stay
// below 2^63, so each lane folds its six accumulators into 128 bits at least
// every 512 column pairs. The row sum is then
//   S = sum_k 2^{p_k} (2^32 A_k + B_k) + 2^31 * sum_j x_j      (mod 2^128)
// and out = low64(S >> 48), exactly the reference's (fixed_t)(acc >> 48).
// Integer addition is associative mod 2^128, so the split / reduction order
// does not change any bit of the result.
//
// Data movement: W is streamed once from HBM with 16-byte non-allocating
// loads, UNROLL loads in flight per row per lane; x is staged once per CTA
// in shared memory together with 2^31*sum(x). One warp owns ROWS rows at a
// time (the lane-to-column map is fixed, so the warp reduction happens once
// per row); CTAs are persistent (grid = resident CTAs) and walk row groups
// with a grid stride. With add != 0 the result is added to out (the residual
// adds of llama_int.c:1535 and 1556 fused into the O and down projections).
#pragma once
#include "iq_common.cuh"

namespace iq {

__device__ __forceinline__ longlong2 ld_stream_v2(const int64_t *p) {
    longlong2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.s64 {%0, %1}, [%2];"
                 : "=l"(v.x), "=l"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ int64_t ld_stream(const int64_t *p) {
    int64_t v;
    asm volatile("ld.global.nc.L1::no_allocate.s64 %0, [%1];" : "=l"(v) : "l"(p));
    return v;
}

// acc += (int64)a * b as one wide integer multiply-add
__device__ __forceinline__ void madw(int64_t &acc, int a, int b) {
    asm("mad.wide.s32 %0, %1, %2, %0;" : "+l"(acc) : "r"(a), "r"(b));
}

// six int64 partial accumulators of one row for one lane
struct Acc6 {
    int64_t A0, A1, A2, B0, B1, B2;
    __device__ __forceinline__ void zero() { A0 = A1 = A2 = B0 = B1 = B2 = 0; }
    __device__ __forceinline__ void mac(int a0, int a1, int a2, int64_t w) {
        int wh = (int)(w >> 32);
        int ws = (int)((uint32_t)w ^ 0x80000000u);
        madw(A0, a0, wh); madw(A1, a1, wh); madw(A2, a2, wh);
        madw(B0, a0, ws); madw(B1, a1, ws); madw(B2, a2, ws);
    }
    // sum_k 2^{p_k} (2^32 A_k + B_k) as a 128-bit value
    __device__ __forceinline__ i128 fold() const {
        i128 s = (i128)B0;
        s += (i128)B1 << 22;
        s += (i128)B2 << 43;
        s += (i128)A0 << 32;
        s += (i128)A1 << 54;
        s += (i128)A2 << 75;
        return s;
    }
};

__device__ __forceinline__ void limbs(int64_t x, int &a0, int &a1, int &a2) {
    a0 = (int)(x & 0x3FFFFF);
    a1 = (int)((x >> 22) & 0x1FFFFF);
    a2 = (int)(x >> 43);
}

__device__ __forceinline__ i128 shfl_xor_i128(i128 v, int m) {
    uint64_t lo = (uint64_t)v, hi = (uint64_t)((u128)v >> 64);
    lo = __shfl_xor_sync(0xffffffffu, lo, m);
    hi = __shfl_xor_sync(0xffffffffu, hi, m);
    return (i128)(((u128)hi << 64) | lo);
}
__device__ __forceinline__ i128 warp_sum_i128(i128 v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v += shfl_xor_i128(v, m);
    return v;
}

// 2^31 * sum(x) computed by the whole CTA; also stages x into shared memory
// when xs != nullptr. Returns the value to every thread.
__device__ __forceinline__ i128 cta_stage_x(const int64_t *__restrict__ x, int64_t *xs, int N) {
    __shared__ uint64_t red[2 * 32];
    i128 s = 0;
    for (int j = threadIdx.x; j < N; j += blockDim.x) {
        int64_t v = x[j];
        if (xs) xs[j] = v;
        s += (i128)v;
    }
    s = warp_sum_i128(s);
    int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (l == 0) { red[2 * w] = (uint64_t)s; red[2 * w + 1] = (uint64_t)((u128)s >> 64); }
    __syncthreads();
    i128 t = 0;
    for (int i = 0; i < nw; i++) t += (i128)(((u128)red[2 * i + 1] << 64) | red[2 * i]);
    return (i128)((u128)t << 31);
}

// Columns per fold: 512 column pairs per lane = 32768 columns.
#define IQ_MV_SEG 32768

// One warp computes a partial dot product for one row over the columns
// [seg-interleaved 64-column blocks kpart, kpart + WPR, ...]; returns this
// lane's 128-bit partial (not yet reduced across lanes).
template <int UNROLL, bool VEC>
__device__ __forceinline__ i128 warp_row_partial(const int64_t *__restrict__ wr, const int64_t *x,
                                                 int N, int lane, int kpart, int WPR) {
    i128 tot = 0;
    // columns handled by this lane per fold: at most 512 pairs (VEC) / 1024 (scalar)
    const int step = (VEC ? 64 : 32) * WPR;
    const int per_fold = VEC ? 512 : 1024;
    int c0 = (VEC ? 2 * lane : lane) + (VEC ? 64 : 32) * kpart;
    while (c0 < N) {
        Acc6 acc;
        acc.zero();
        for (int it = 0; it < per_fold && c0 < N; it += UNROLL, c0 += step * UNROLL) {
            if (VEC) {
                longlong2 wv[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    int c = c0 + step * u;
                    if (c < N) wv[u] = ld_stream_v2(wr + c);
                }
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    int c = c0 + step * u;
                    if (c < N) {
                        longlong2 xv = *reinterpret_cast<const longlong2 *>(x + c);
                        int p0, p1, p2, q0, q1, q2;
                        limbs(xv.x, p0, p1, p2);
                        limbs(xv.y, q0, q1, q2);
                        acc.mac(p0, p1, p2, wv[u].x);
                        acc.mac(q0, q1, q2, wv[u].y);
                    }
                }
            } else {
                int64_t wv[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    int c = c0 + step * u;
                    if (c < N) wv[u] = ld_stream(wr + c);
                }
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    int c = c0 + step * u;
                    if (c < N) {
                        int p0, p1, p2;
                        limbs(x[c], p0, p1, p2);
                        acc.mac(p0, p1, p2, wv[u]);
                    }
                }
            }
        }
        tot += acc.fold();
    }
    return tot;
}

// CTA of 8 warps; each row is split over WPR warps (split-K inside the CTA,
// reduced through shared memory), so a CTA handles 8/WPR rows per pass.
template <int WPR, int UNROLL, bool VEC, bool XSMEM>
__global__ void __launch_bounds__(256)
k_matvec(int64_t *__restrict__ out, const int64_t *__restrict__ W,
         const int64_t *__restrict__ xg, int M, int N, int add) {
    extern __shared__ __align__(16) int64_t xs_dyn[];
    __shared__ uint64_t part[8][2];
    const int64_t *x = XSMEM ? xs_dyn : xg;
    const i128 xcorr = cta_stage_x(xg, XSMEM ? xs_dyn : nullptr, N);
    __syncthreads();

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int RPC = 8 / WPR;  // rows per CTA pass
    const int slot = warp / WPR, kpart = warp % WPR;
    for (int r0 = blockIdx.x * RPC; r0 < M; r0 += gridDim.x * RPC) {
        const int row = r0 + slot;
        i128 t = 0;
        if (row < M) t = warp_row_partial<UNROLL, VEC>(W + (size_t)row * N, x, N, lane, kpart, WPR);
        t = warp_sum_i128(t);
        if (WPR > 1) {
            if (lane == 0) { part[warp][0] = (uint64_t)t; part[warp][1] = (uint64_t)((u128)t >> 64); }
            __syncthreads();
            if (kpart == 0) {
                for (int k = 1; k < WPR; k++)
                    t += (i128)(((u128)part[warp + k][1] << 64) | part[warp + k][0]);
            }
            __syncthreads();
        }
        if (kpart == 0 && lane == 0 && row < M) {
            // add != 0: residual epilogue out += result (int64 wrap, llama_int.c:1535, 1556)
            int64_t v = (int64_t)((t + xcorr) >> 48);
            out[row] = add ? (int64_t)((uint64_t)out[row] + (uint64_t)v) : v;
        }
    }
}

}  // namespace iq
