// iq_tc_gemm.cuh -- exact Q16.48 GEMM (rows of matmul_vec) on the 5th-gen
// tensor cores: tcgen05.mma kind::i8, operands staged by TMA, accumulators in
// TMEM.
//
// Same byte-plane identity as iq_planes.cuh: with W's bytes B_p (B_7 signed)
// and the unsigned digits D_j of x_u = x + 2^63,
//   out[r][i] = low64( (sum_{p,j} 2^{8(p+j)} P_pj[r][i] - 2^63 sum_k W[i][k]) >> 48 )
//   P_pj[r][i] = sum_k B_p(W[i][k]) * D_j(x_u[r][k])       (exact int32)
// Only the window of planes p0 .. p0+np-1 is stored (see iq_planes.cuh: the
// top stored plane is the signed one, and the low bytes below p0 that few
// weights use are an exact sparse per-row residual sum_k x[r][k] w_lo[i][k]
// added by the epilogue before the shift).
// For plane p the products for all digits are one GEMM: A = plane p of W
// ([Mpad][Kpad] bytes, K-major) times B = the digit matrix
// ([(row, digit)][Kpad] bytes, K-major, row = 8*r + j), so the MMA's N
// columns are (x-row, digit) pairs: N = 256 covers 32 x-rows.
//
// CTA tile: 128 output rows of W x 32 rows of X. Planes go in pairs
// (2q, 2q+1) that share every staged digit tile: per pair and 128-byte K
// block one stage holds A of both planes (2 x 128 x 128 B) and B (256 x 128 B),
// 64 KB for 8 MMAs, against 48 KB for 4 when each plane re-staged the digits
// (the GEMM was bound by delivering operands). Warp roles (320 threads):
//   warp 0      TMA producer: 3-stage ring of pair stages;
//   warp 1      owns TMEM (512 columns: one 256-column accumulator per plane
//               of the pair) and issues the MMAs from one thread,
//               4 x 2 x (M=128, N=256, K=32) per stage, committing each stage's
//               smem back to the producer and each finished pair to the
//               epilogue;
//   warps 2..9  epilogue: per pair, read the two 128 x 256 int32 tiles from
//               TMEM (warp w reads lanes 32*(w%4)..+31, half of the columns)
//               and fold them into 16 128-bit sums per thread (thread = one W
//               row, 16 x-rows), then release TMEM; finally subtract
//               2^63*rowsum and store.
// K per plane pass <= 32768 keeps every int32 partial exact (|u8*u8| <= 65025).
#pragma once
#include "iq_sync.cuh"
#include "iq_planes.cuh"

namespace iq {

constexpr int TC_BM = 128, TC_BR = 32, TC_BK = 128, TC_STAGES = 3;
constexpr int TC_A_BYTES = TC_BM * TC_BK;            // 16 KB per plane
constexpr int TC_B_BYTES = TC_BR * 8 * TC_BK;        // 32 KB
constexpr int TC_STAGE_BYTES = 2 * TC_A_BYTES + TC_B_BYTES;   // two planes share one digit tile
constexpr size_t TC_SMEM = 1024 + (size_t)TC_STAGES * TC_STAGE_BYTES + 256;
constexpr int TC_EPI_WARPS = 8;                          // 2 per TMEM lane quadrant
constexpr int TC_THREADS = 32 * (2 + TC_EPI_WARPS);      // producer, MMA issuer, epilogue
constexpr int TC_HR = TC_BR / 2;                         // x-rows per epilogue warp

// W [M][K] int64 -> planes [np][Mpad][Kpad] bytes p0 .. p0+np-1 (zero padded; top plane signed)
__global__ void k_pack_rowplanes(uint8_t *__restrict__ out, const int64_t *__restrict__ W, int M, int K,
                                 int Mpad, int Kpad, int np, int p0) {
    const int64_t n = (int64_t)Mpad * Kpad;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        int m = (int)(e / Kpad), k = (int)(e % Kpad);
        uint64_t w = (m < M && k < K) ? (uint64_t)W[(size_t)m * K + k] : 0ull;
        for (int p = 0; p < np; p++) out[(size_t)p * n + e] = (uint8_t)(w >> (8 * (p0 + p)));
    }
}

// X [R][K] int64 -> digits [Rpad*8][Kpad] bytes, row 8r+j = byte j of (x ^ 2^63)
__global__ void k_x_digits(uint8_t *__restrict__ out, const int64_t *__restrict__ X, int R, int K, int Rpad,
                           int Kpad) {
    const int64_t n = (int64_t)Rpad * Kpad;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        int r = (int)(e / Kpad), k = (int)(e % Kpad);
        uint64_t xu = (r < R && k < K) ? ((uint64_t)X[(size_t)r * K + k] ^ 0x8000000000000000ull) : 0ull;
#pragma unroll
        for (int j = 0; j < 8; j++) out[((size_t)r * 8 + j) * Kpad + k] = (uint8_t)(xu >> (8 * j));
    }
}

__global__ void __launch_bounds__(TC_THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB,
          int64_t *__restrict__ out, const PackedRes res, const int64_t *__restrict__ X, int K, int M, int R,
          int Mpad, int Kpad, int add, int64_t *__restrict__ part, int Rpad, int np) {
    const int64_t *__restrict__ rowsum = res.rowsum;
    extern __shared__ unsigned char smraw[];
    unsigned char *sm = smraw + ((1024 - (smem_u32(smraw) & 1023)) & 1023);  // 1024-aligned stages
    unsigned char *stage = sm;
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + TC_STAGES * TC_STAGE_BYTES);
    uint64_t *empty = full + TC_STAGES;
    uint64_t *afull = empty + TC_STAGES;   // [2]
    uint64_t *aempty = afull + 2;          // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(aempty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // grid x walks the X-row tiles, so the CTAs resident together share one
    // W tile (read once from HBM, then from L2) and the digit matrix stays in L2
    const int m0 = blockIdx.y * TC_BM, r0 = blockIdx.x * TC_BR;
    // split-K: this CTA covers K blocks [kb0, kb0 + KB) of every plane
    const int KBall = Kpad / TC_BK, KS = gridDim.z, ks = blockIdx.z;
    const int kb0 = (int)((int64_t)KBall * ks / KS), KB = (int)((int64_t)KBall * (ks + 1) / KS) - kb0;

    // planes are taken in pairs (2q, 2q+1) that share each staged digit tile
    const int ngrp = (np + 1) / 2;
    const int total = ngrp * KB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_STAGES; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(&afull[0], 1);
        mbar_init(&aempty[0], TC_EPI_WARPS);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            for (; it < total; it++) {
                const int q = it / KB, kb = it % KB, s = it % TC_STAGES;
                const bool pair = 2 * q + 1 < np;
                if (it >= TC_STAGES && !mbar_wait(&empty[s], (uint32_t)((it / TC_STAGES) - 1) & 1u)) break;
                mbar_expect_tx(&full[s], (pair ? 2 : 1) * TC_A_BYTES + TC_B_BYTES);
                unsigned char *a = stage + (size_t)s * TC_STAGE_BYTES;
                const int kx = (kb0 + kb) * TC_BK;
                tma_load_2d(a, &mapA, kx, (2 * q) * Mpad + m0, &full[s]);
                if (pair) tma_load_2d(a + TC_A_BYTES, &mapA, kx, (2 * q + 1) * Mpad + m0, &full[s]);
                tma_load_2d(a + 2 * TC_A_BYTES, &mapB, kx, r0 * 8, &full[s]);
            }
            // drain: the last copies into each stage have landed before the CTA can exit
            for (int j = (it > TC_STAGES ? it - TC_STAGES : 0); j < it; j++)
                mbar_wait(&full[j % TC_STAGES], (uint32_t)(j / TC_STAGES) & 1u);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            for (int q = 0; q < ngrp && ok; q++) {
                const bool pair = 2 * q + 1 < np;
                // the epilogue must have read the previous pair's accumulators
                if (q >= 1 && !mbar_wait(&aempty[0], (uint32_t)(q - 1) & 1u)) break;
                tc_fence_after();
                const uint32_t id0 = idesc_i8(2 * q == np - 1, false, TC_BM, TC_BR * 8);  // top plane signed
                const uint32_t id1 = idesc_i8(2 * q + 1 == np - 1, false, TC_BM, TC_BR * 8);
                for (int kb = 0; kb < KB; kb++) {
                    const int it = q * KB + kb, s = it % TC_STAGES;
                    if (!mbar_wait(&full[s], (uint32_t)(it / TC_STAGES) & 1u)) { ok = false; break; }
                    tc_fence_after();
                    const unsigned char *a = stage + (size_t)s * TC_STAGE_BYTES;
                    const uint64_t a0 = smem_desc_sw128(a), a1 = smem_desc_sw128(a + TC_A_BYTES),
                                   bd = smem_desc_sw128(a + 2 * TC_A_BYTES);
#pragma unroll
                    for (int k = 0; k < TC_BK / 32; k++) {  // advance 32 bytes of K = 2 descriptor units
                        tc_mma_i8(tmem, a0 + 2 * k, bd + 2 * k, id0, (kb | k) != 0);
                        if (pair) tc_mma_i8(tmem + 256u, a1 + 2 * k, bd + 2 * k, id1, (kb | k) != 0);
                    }
                    tc_commit(&empty[s]);
                }
                if (ok) tc_commit(&afull[0]);
            }
        }
    } else {
        // epilogue warps: TMEM lane quadrant = warp % 4; the two warps of a
        // quadrant take x-rows 0..15 and 16..31 (columns 0..127 / 128..255)
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int row = m0 + quad * 32 + lane;
        const int rb = r0 + half * TC_HR;   // this warp's first x-row
        i128 acc[TC_HR];
#pragma unroll
        for (int r = 0; r < TC_HR; r++) acc[r] = 0;
        bool ok = true;
        for (int q = 0; q < ngrp && ok; q++) {
            if (!mbar_wait(&afull[0], (uint32_t)q & 1u)) { ok = false; break; }
            tc_fence_after();
            for (int h = 0; h < 2; h++) {
                const int p = 2 * q + h;
                if (p >= np) break;
#pragma unroll
                for (int c = 0; c < 4; c++) {  // 32 columns = 4 x-rows x 8 digits
                    uint32_t v[32];
                    tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(h * 256 + half * 128 + c * 32), v);
                    tmem_ld_wait();
                    // digits 0..3 and 4..7 of one x-row each sum exactly in 64 bits
                    // (|v| < 2^31, shifts <= 24: < 2^57), then one 128-bit
                    // shift-add per x-row: sum_j v_j 2^(8(p0+p+j))
                    const int sh = 8 * (res.p0 + p);
#pragma unroll
                    for (int rr = 0; rr < 4; rr++) {
                        int64_t lo = 0, hi = 0;
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            lo += (int64_t)(int32_t)v[rr * 8 + j] * (1ll << (8 * j));
                            hi += (int64_t)(int32_t)v[rr * 8 + 4 + j] * (1ll << (8 * j));
                        }
                        acc[4 * c + rr] += (i128)((u128)((i128)lo + (i128)((u128)(i128)hi << 32)) << sh);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&aempty[0]);
        }
        if (ok && KS > 1) {
            // split-K: store this CTA's 128-bit partial sums; k_gemm_reduce finishes
#pragma unroll
            for (int r = 0; r < TC_HR; r++) {
                int64_t *pp = part + (((size_t)ks * Rpad + rb + r) * Mpad + row) * 2;
                pp[0] = (int64_t)(uint64_t)acc[r];
                pp[1] = (int64_t)(uint64_t)((u128)acc[r] >> 64);
            }
        } else if (ok && row < M) {
            if (res.ptr) {  // sparse residual: sum_k x[r][k] * w_lo[row][k]
#pragma unroll 1
                for (int e = res.ptr[row], e1 = res.ptr[row + 1]; e < e1; e++) {
                    const int k = res.col[e];
                    const int64_t wl = res.val[e];
#pragma unroll
                    for (int r = 0; r < TC_HR; r++)
                        if (rb + r < R) acc[r] += mul_wide(X[(size_t)(rb + r) * K + k], wl);
                }
            }
            const i128 ws = (i128)(((u128)(uint64_t)rowsum[2 * row + 1] << 64) | (uint64_t)rowsum[2 * row]);
            const u128 bias = (u128)ws << 63;
#pragma unroll
            for (int r = 0; r < TC_HR; r++) {
                if (rb + r < R) {
                    int64_t v = (int64_t)((i128)((u128)acc[r] - bias) >> 48);
                    int64_t *o = out + (size_t)(rb + r) * M + row;
                    *o = add ? (int64_t)((uint64_t)*o + (uint64_t)v) : v;  // fused residual add
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// split-K finish: out[r][m] (+)= low64((sum_ks part[ks][r][m] - 2^63 rowsum[m]) >> 48)
__global__ void k_gemm_reduce(int64_t *__restrict__ out, const int64_t *__restrict__ part, const PackedRes res,
                              const int64_t *__restrict__ X, int K, int M, int R, int Mpad, int Rpad, int KS,
                              int add) {
    const int64_t *__restrict__ rowsum = res.rowsum;
    const int64_t n = (int64_t)R * M;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / M), m = (int)(e % M);
        u128 acc = 0;
        for (int ks = 0; ks < KS; ks++) {
            const int64_t *pp = part + (((size_t)ks * Rpad + r) * Mpad + m) * 2;
            acc += ((u128)(uint64_t)pp[1] << 64) | (uint64_t)pp[0];
        }
        if (res.ptr)  // sparse residual: sum_k x[r][k] * w_lo[m][k]
            for (int q = res.ptr[m], q1 = res.ptr[m + 1]; q < q1; q++)
                acc += (u128)mul_wide(X[(size_t)r * K + res.col[q]], res.val[q]);
        const u128 ws = ((u128)(uint64_t)rowsum[2 * m + 1] << 64) | (uint64_t)rowsum[2 * m];
        int64_t v = (int64_t)((i128)(acc - (ws << 63)) >> 48);
        int64_t *o = out + (size_t)r * M + m;
        *o = add ? (int64_t)((uint64_t)*o + (uint64_t)v) : v;
    }
}

}  // namespace iq
