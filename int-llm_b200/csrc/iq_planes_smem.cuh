// iq_planes_smem.cuh -- the row-owned bf16-form matvec with its whole weight
// slice staged in shared memory by the bulk-copy engine (cp.async.bulk,
// global -> shared, completing on an mbarrier) BEFORE the kernel waits for
// its inputs (griddepcontrol.wait). Weights do not depend on the previous
// kernel, so under programmatic dependent launch the entire slice streams in
// while the previous kernel finishes; after the wait only the activations are
// staged and the MMAs read A fragments from shared memory. Same arithmetic
// and result as k_matvec_rows<3, true> (iq_planes.cuh).
//
// One row tile per CTA (the launcher uses it only when one wave of CTAs
// covers every row tile); a cluster of S CTAs splits the tile's column tiles
// into S contiguous ranges, each CTA copying its own range (ncols x 1 KB).
#pragma once
#include "iq_sync.cuh"
#include "iq_planes.cuh"

namespace iq {

// global -> shared bulk copy of `bytes` (a multiple of 16, both addresses
// 16-byte aligned), completing on bar (no multicast)
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__global__ void __launch_bounds__(256, 1)
k_matvec_rows_smem(int64_t *__restrict__ out, const uint4 *__restrict__ planes, const PackedRes R,
                   const int64_t *__restrict__ xg, int M, int N, int Kp, int add, const int64_t *__restrict__ nrm_w,
                   int wsm_off) {
    extern __shared__ __align__(128) unsigned char wsm_raw[];
    unsigned char *xd = wsm_raw;                                          // [8][Kp + 16] digit rows
    const uint4 *wsm = reinterpret_cast<const uint4 *>(wsm_raw + wsm_off);  // [ncols][64] (1 KB per tile)
    __shared__ __align__(16) unsigned long long wpart[8][16][2];
    __shared__ __align__(16) unsigned long long cpart[8][16][2];
    __shared__ __align__(8) uint64_t wbar;
    constexpr int TS = 64;   // uint4 per tile in the bf16 form
    const int ld = Kp + 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int KT = Kp / 32, RT = (M + 15) / 16;
    uint32_t S, crank;
    asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(S));
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
    const int rt = blockIdx.x / S;
    const bool live = rt < RT;
    const int per_cta = (KT + (int)S - 1) / (int)S;
    const int kc0 = min(KT, (int)crank * per_cta), kc1 = min(KT, kc0 + per_cta), ncols = kc1 - kc0;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (S > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    if (threadIdx.x == 0) {
        mbar_init(&wbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && live && ncols > 0) {   // the whole slice, before waiting for the inputs
        const uint32_t bytes = (uint32_t)ncols * TS * 16;
        mbar_expect_tx(&wbar, bytes);
        const unsigned char *src = reinterpret_cast<const unsigned char *>(planes + ((size_t)rt * KT + kc0) * TS);
        unsigned char *dst = wsm_raw + wsm_off;
        for (uint32_t off = 0; off < bytes; off += 32768u)
            bulk_g2s(dst + off, src + off, min(32768u, bytes - off), &wbar);
    }
    RowPre pre = {};
    if (threadIdx.x < 16 && live && rt * 16 + (int)threadIdx.x < M) pre = row_pre(rt * 16 + threadIdx.x, R);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    i128 xs = 0;
    stage_digits(xd, ld, xg, N, Kp, nrm_w, &xs);
    const unsigned char *xb = xd + g * ld + 4 * t;
    int c[3][4];
#pragma unroll
    for (int p = 0; p < 3; p++)
#pragma unroll
        for (int q = 0; q < 4; q++) c[p][q] = 0;
    if (live && ncols > 0) {
        if (!mbar_wait(&wbar, 0)) {
            // bulk copy never completed (recorded as IQ_ERR_TIMEOUT): skip the MMAs
        } else {
            // the CTA's 8 warps take its column tiles round robin
            for (int j = warp; j < ncols; j += 8) {
                const uint4 *tile = wsm + (size_t)j * TS + lane;
                const uint4 w2[2] = {tile[0], tile[32]};
                const int kt = kc0 + j;
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xb + kt * 32);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xb + kt * 32 + 16);
                mma_tile_bf(c, w2, b0, b1);
            }
        }
    }
    i128 r0 = 0, r1 = 0;
    fold_planes(c, t, r0, r1);
    if (!live) {
        if (S > 1) {  // keep the cluster barrier phases matched
            asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
            asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
            asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
        }
        return;
    }
    rows_tile_end(r0, r1, rt, rt, pre, S, crank, M, add, out, R, xd, ld, xg, xs, &wpart[0][0][0], &cpart[0][0][0]);
}

}  // namespace iq

namespace iq {

// Up to a few row tiles per CTA (more tiles than one wave of CTAs): CTA c
// takes row tiles c, c + G, c + 2G, ... through a ring of `stages`
// shared-memory slots of one whole row tile each (KT x 1 KB), refilled by the
// bulk-copy engine as soon as the CTA has consumed a slot; the first `stages`
// tiles are requested before the dependency wait. The digits of x are staged
// once per CTA for all its tiles. 8 warps split each tile's column tiles; the
// rows are reduced and written as in k_matvec_rows (S = 1).
__global__ void __launch_bounds__(256, 1)
k_matvec_rows_pipe(int64_t *__restrict__ out, const uint4 *__restrict__ planes, const PackedRes R,
                   const int64_t *__restrict__ xg, int M, int N, int Kp, int add, const int64_t *__restrict__ nrm_w,
                   int wsm_off, int stages) {
    extern __shared__ __align__(128) unsigned char wsm_raw[];
    unsigned char *xd = wsm_raw;
    __shared__ __align__(16) unsigned long long wpart[8][16][2];
    __shared__ __align__(16) unsigned long long cpart[8][16][2];
    __shared__ __align__(8) uint64_t full[4];
    constexpr int TS = 64;
    const int ld = Kp + 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int KT = Kp / 32, RT = (M + 15) / 16;
    const uint32_t tile_bytes = (uint32_t)KT * TS * 16;
    const int G = gridDim.x, ntiles = (int)blockIdx.x < RT ? (RT - 1 - (int)blockIdx.x) / G + 1 : 0;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto request = [&](int i) {   // tile i of this CTA into slot i % stages
        const int s = i % stages, rt = (int)blockIdx.x + i * G;
        mbar_expect_tx(&full[s], tile_bytes);
        const unsigned char *src = reinterpret_cast<const unsigned char *>(planes + (size_t)rt * KT * TS);
        unsigned char *dst = wsm_raw + wsm_off + (size_t)s * tile_bytes;
        for (uint32_t off = 0; off < tile_bytes; off += 32768u)
            bulk_g2s(dst + off, src + off, min(32768u, tile_bytes - off), &full[s]);
    };
    if (threadIdx.x == 0)
        for (int i = 0; i < stages && i < ntiles; i++) request(i);
    RowPre pre = {};
    if (threadIdx.x < 16 && ntiles > 0 && (int)(blockIdx.x * 16 + threadIdx.x) < M)
        pre = row_pre(blockIdx.x * 16 + threadIdx.x, R);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    i128 xs = 0;
    stage_digits(xd, ld, xg, N, Kp, nrm_w, &xs);
    const unsigned char *xb = xd + g * ld + 4 * t;
    bool ok = true;
    for (int i = 0; i < ntiles; i++) {
        const int s = i % stages, rt = (int)blockIdx.x + i * G;
        int c[3][4];
#pragma unroll
        for (int p = 0; p < 3; p++)
#pragma unroll
            for (int q = 0; q < 4; q++) c[p][q] = 0;
        if (ok && !mbar_wait(&full[s], (uint32_t)(i / stages) & 1u)) ok = false;
        if (ok) {
            const uint4 *wsm = reinterpret_cast<const uint4 *>(wsm_raw + wsm_off + (size_t)s * tile_bytes);
            for (int j = warp; j < KT; j += 8) {
                const uint4 *tile = wsm + (size_t)j * TS + lane;
                const uint4 w2[2] = {tile[0], tile[32]};
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xb + j * 32);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xb + j * 32 + 16);
                mma_tile_bf(c, w2, b0, b1);
            }
        }
        i128 r0 = 0, r1 = 0;
        fold_planes(c, t, r0, r1);
        // every warp is done with slot s once rows_tile_end's barriers pass
        rows_tile_end(r0, r1, rt, (int)blockIdx.x, pre, 1, 0, M, add, out, R, xd, ld, xg, xs, &wpart[0][0][0],
                      &cpart[0][0][0]);
        if (threadIdx.x == 0 && ok && i + stages < ntiles) request(i + stages);
    }
}

}  // namespace iq
