// iq_peak.cuh -- measured ceilings for the rooflines: the tcgen05 kind::i8
// tensor-pipe peak of this GPU (no memory traffic: every MMA reads the same
// shared-memory tiles). Used by the bench to state the GEMM's utilisation
// against a measured, not a nominal, peak.
#pragma once
#include "iq_sync.cuh"

namespace iq {

// One CTA per SM. Thread 0 issues `iters` x 4 MMAs (M=128, N=256, K=32,
// u8 x u8 -> s32) alternating between two 256-column TMEM accumulators,
// committing every 4 to an mbarrier and keeping at most 8 commits in flight.
__global__ void __launch_bounds__(128, 1) k_i8_peak(int iters, int *done) {
    extern __shared__ unsigned char smraw[];
    unsigned char *sm = smraw + ((1024 - (smem_u32(smraw) & 1023)) & 1023);
    unsigned char *a = sm;                  // 16 KB: 128 rows x 128 B
    unsigned char *b = sm + 16384;          // 32 KB: 256 rows x 128 B
    uint64_t *bar = reinterpret_cast<uint64_t *>(sm + 49152);  // [2]
    uint32_t *slot = reinterpret_cast<uint32_t *>(bar + 2);
    for (int i = threadIdx.x; i < 49152 / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(sm)[i] = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (threadIdx.x < 32) tmem_alloc(slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *slot;
    if (threadIdx.x == 0) {
        const uint32_t idesc = idesc_i8(false, false, 128, 256);
        const uint64_t ad = smem_desc_sw128(a), bd = smem_desc_sw128(b);
        bool ok = true;
        for (int it = 0; it < iters && ok; it++) {
            const int buf = it & 1;
            // before reusing barrier `buf`, wait for its previous commit
            if (it >= 2 && !mbar_wait(&bar[buf], (uint32_t)((it / 2) - 1) & 1u)) ok = false;
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 4; k++)
                tc_mma_i8(tmem + (uint32_t)(buf * 256), ad + 2 * k, bd + 2 * k, idesc, k != 0);
            tc_commit(&bar[buf]);
        }
        for (int it = iters - 2 > 0 ? iters - 2 : 0; it < iters && ok; it++)
            if (!mbar_wait(&bar[it & 1], (uint32_t)(it / 2) & 1u)) ok = false;
        if (ok) atomicAdd(done, 1);
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace iq
