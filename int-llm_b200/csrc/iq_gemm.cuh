// iq_gemm.cuh -- batched rows of matmul_vec (rows >= 2) on CUDA cores.
//
// out[r][i] = low64((sum_j X[r][j] * W[i][j]) >> 48): the reference computes
// these as `rows` separate matmul_vec calls (llama_int.c:1014, prefill loop
// llama_int.c:3081-3092). Same exact limb arithmetic as iq_matvec.cuh.
//
// Tiling: a CTA owns a tile of BM output columns (rows of W) x BR rows of X.
// K is walked in chunks of BK: the W chunk [BM][BK] and X chunk [BR][BK] are
// staged in shared memory (X already split into its three limbs), and each
// thread accumulates a TM x TR register block of outputs (six int64
// accumulators per output). Accumulators fold into 128 bits every chunk.
#pragma once
#include "iq_matvec.cuh"

namespace iq {

template <int BM, int BR, int BK, int TM, int TR>
__global__ void __launch_bounds__((BM / TM) * (BR / TR))
k_gemm(int64_t *__restrict__ out, const int64_t *__restrict__ W,
       const int64_t *__restrict__ X, int rows, int M, int N, int add) {
    constexpr int NT = (BM / TM) * (BR / TR);
    __shared__ int2 ws[BK][BM + 1];      // (wh, ws) per weight, [k][m]
    __shared__ int xl[3][BK][BR + 1];    // limbs per activation, [limb][k][r]

    const int m0 = blockIdx.x * BM, r0 = blockIdx.y * BR;
    const int tm = threadIdx.x % (BM / TM), tr = threadIdx.x / (BM / TM);

    i128 tot[TM][TR];
#pragma unroll
    for (int a = 0; a < TM; a++)
#pragma unroll
        for (int b = 0; b < TR; b++) tot[a][b] = 0;

    for (int k0 = 0; k0 < N; k0 += BK) {
        __syncthreads();
        // stage W chunk: BM rows x BK cols (row-major source, coalesced along k)
        for (int e = threadIdx.x; e < BM * BK; e += NT) {
            int m = e / BK, k = e % BK;
            int64_t w = 0;
            bool ok = (m0 + m < M) && (k0 + k < N);
            if (ok) w = W[(size_t)(m0 + m) * N + k0 + k];
            // out-of-range entries become (0, -2^31) so that they contribute
            // exactly the bias 2^31*x, which is removed below by zeroing x.
            ws[k][m] = make_int2((int)(w >> 32), (int)((uint32_t)w ^ 0x80000000u));
        }
        for (int e = threadIdx.x; e < BR * BK; e += NT) {
            int r = e / BK, k = e % BK;
            int64_t x = 0;
            if ((r0 + r < rows) && (k0 + k < N)) x = X[(size_t)(r0 + r) * N + k0 + k];
            int a0, a1, a2;
            limbs(x, a0, a1, a2);
            xl[0][k][r] = a0; xl[1][k][r] = a1; xl[2][k][r] = a2;
        }
        __syncthreads();
        Acc6 acc[TM][TR];
#pragma unroll
        for (int a = 0; a < TM; a++)
#pragma unroll
            for (int b = 0; b < TR; b++) acc[a][b].zero();
#pragma unroll 4
        for (int k = 0; k < BK; k++) {
            int2 wv[TM];
            int xa[TR][3];
#pragma unroll
            for (int a = 0; a < TM; a++) wv[a] = ws[k][tm + a * (BM / TM)];
#pragma unroll
            for (int b = 0; b < TR; b++) {
                xa[b][0] = xl[0][k][tr + b * (BR / TR)];
                xa[b][1] = xl[1][k][tr + b * (BR / TR)];
                xa[b][2] = xl[2][k][tr + b * (BR / TR)];
            }
#pragma unroll
            for (int a = 0; a < TM; a++)
#pragma unroll
                for (int b = 0; b < TR; b++) {
                    Acc6 &c = acc[a][b];
                    madw(c.A0, xa[b][0], wv[a].x); madw(c.A1, xa[b][1], wv[a].x);
                    madw(c.A2, xa[b][2], wv[a].x);
                    madw(c.B0, xa[b][0], wv[a].y); madw(c.B1, xa[b][1], wv[a].y);
                    madw(c.B2, xa[b][2], wv[a].y);
                }
        }
#pragma unroll
        for (int a = 0; a < TM; a++)
#pragma unroll
            for (int b = 0; b < TR; b++) tot[a][b] += acc[a][b].fold();
    }
    // bias term 2^31 * sum_j X[r][j] per X row: computed by the owning threads.
#pragma unroll
    for (int b = 0; b < TR; b++) {
        int r = r0 + tr + b * (BR / TR);
        if (r >= rows) continue;
        i128 sx = 0;
        const int64_t *xr = X + (size_t)r * N;
        for (int j = 0; j < N; j++) sx += (i128)xr[j];
        i128 corr = (i128)((u128)sx << 31);
#pragma unroll
        for (int a = 0; a < TM; a++) {
            int m = m0 + tm + a * (BM / TM);
            if (m < M) {
                int64_t v = (int64_t)((tot[a][b] + corr) >> 48);
                int64_t *o = out + (size_t)r * M + m;
                *o = add ? (int64_t)((uint64_t)*o + (uint64_t)v) : v;  // fused residual add
            }
        }
    }
}

}  // namespace iq
