// iq_planes.cuh -- exact Q16.48 matvec on the int8 tensor cores (sm_100a).
//
// Byte-plane decomposition
// ------------------------
// A weight w (int64) is the sum of its bytes: w = sum_{i<8} B_i(w) 2^{8i} with
// B_0..B_6 unsigned and B_7 signed (two's complement). An activation x is
// biased to x_u = x + 2^63 (an unsigned 64-bit value, the sign bit flipped)
// with unsigned bytes D_j(x_u). Then, summed over the row,
//   sum_k x_k w_k = sum_{i,j} 2^{8(i+j)} P_ij - 2^63 sum_k w_k      (mod 2^128)
//   P_ij = sum_k B_i(w_k) D_j(x_u,k)
// Each P_ij is an int8 x uint8 dot product accumulated exactly in int32 by the
// tensor cores (|u8*u8| <= 65025, so <= 33025 terms fit; the kernel folds into
// 128 bits every 1024 k-tiles = 32768 terms). sum_k w_k is a per-row constant
// computed when the weights are packed. out = low64(sum >> 48) exactly as
// matmul_vec (llama_int.c:1014-1046); every step is exact integer arithmetic.
//
// Only a window of np planes p0 .. p0+np-1 is stored. The top is the most
// bytes any weight needs as a signed integer (bf16-derived weights need 6),
// read as signed, the bytes above it being its sign extension. Below, planes
// p0 > 0 are dropped when few weights use them: each weight splits exactly
// into w = w_hi + w_lo with w_lo = w & (2^(8 p0) - 1) (unsigned) and w_hi
// having zero low bytes, so
//   sum_k x_k w_k = 2^(8 p0) sum_{i,j} 2^{8(i+j)} P_ij - 2^63 sum_k w_hi,k
//                   + sum_{k: w_lo,k != 0} x_k w_lo,k                 (mod 2^128)
// with P_ij over the stored planes of w_hi; the last sum is a sparse per-row
// residual (CSR) that the row's writer adds. Config weights (bf16-derived,
// N(0, 0.02)) keep bytes 3..5: 3 bytes per weight, residual ~0.02% of them.
// Packed layout (np bytes per weight, 8 for arbitrary int64): for each
// 16-row x 32-column tile, np planes x 32 lanes x 16 bytes, where lane l holds
// exactly its A fragment of mma.m16n8k32 (rows l/4 and l/4+8, columns
// 4(l%4)..+3 and 16+4(l%4)..+3), so one 16-byte load per plane per lane
// streams the tile. Rows are padded to 16 and columns to 32 with zeros.
//
// bf16 form (fmt IQ_FMT_BF16, 2 bytes per weight). Weights that came from
// bf16 (bfloat16_to_q1648, safetensors.h:115-152) are +-m 2^e with an 8-bit
// m; when w is a multiple of 2^24 and v = w / 2^24 lies in [-2^22, 2^22) with
// at most 8 significant bits, the bf16 number v 2^-24 holds w exactly and is
// stored as is (the config weights: all but ~0.03%). The kernel recovers
//   u = v + 2^22 = low 23 bits of fma.rm(f, 2^24, 1.5 * 2^23)
// exactly (f = the bf16 value as fp32; the sum lies in [2^23, 2^24), where fp32
// steps by 1, and rounding toward -inf of an exact integer changes nothing),
// splits u into three unsigned byte planes in registers and runs the same
// MMAs. Then, with U = sum_k u_k (a per-row constant) and X = sum_k x_k (per
// launch, from the staged activations),
//   sum_k x_k w_k = 2^24 (sum_{i,j} 2^{8(i+j)} P_ij - 2^63 U - 2^22 X) + residual
// where every other weight (not of that form) is stored as 0 (v = 0) and its
// whole value goes to the sparse residual, and padding columns are stored as
// -0.25 (u = 0), so they add nothing. Layout: per 16x32 tile, 32 lanes x 2 x
// 16 bytes: lane l's 16 weights (its A fragment, register r = 4 consecutive k)
// as bf16 pairs, words [r0 k0k1, r0 k2k3, r1 k0k1, r1 k2k3] then r2, r3.
//
// The x digits D_j form the MMA's B operand (N = 8 = one column per digit),
// staged once per CTA in shared memory as 8 byte-rows of Kp (+16 pad).
// Work split: stream-K over (row tile, column tile) units, equal slices per
// resident warp; row tiles split between warps meet in RowAcc scratch through
// exact 128-bit atomics, and the warp that completes a row writes it.
#pragma once
#include <cuda/atomic>
#include "iq_elem.cuh"

namespace iq {

// Stored forms (iq.h): IQ_FMT_PLANES = byte-plane window (np planes from p0),
// IQ_FMT_BF16 = bf16 words converted in the kernel (3 planes, p0 = 3).
struct Packed {
    int fmt = IQ_FMT_PLANES;
    int M = 0, N = 0;       // logical shape: M rows of N columns
    int Mp = 0, Kp = 0;     // padded to 16 rows / 32 columns
    int np = 8;             // byte planes stored (top plane signed)
    int p0 = 0;             // lowest stored plane
    int nnz = 0;            // weights with nonzero bytes below p0 (residual entries)
    uint4 *planes = nullptr;
    int64_t *rowsum = nullptr;  // [Mp][2] = 128-bit sum_k w_hi[row][k] (lo, hi); bf16 form: sum_k u
    int *res_ptr = nullptr;     // [Mp + 1] CSR row offsets (nullptr when nnz == 0)
    int *res_col = nullptr;     // [nnz] column
    int64_t *res_val = nullptr; // [nnz] w_lo
};

// Bytes of the stored form one matvec launch reads: planes, 128-bit row sums
// and the residual CSR (x and out not counted).
inline int64_t packed_bytes(const Packed &P) {
    int64_t b = (int64_t)(P.fmt == IQ_FMT_BF16 ? 2 : P.np) * P.Mp * P.Kp + 16 * (int64_t)P.Mp;
    if (P.nnz) b += 4 * ((int64_t)P.Mp + 1) + 12 * (int64_t)P.nnz;
    return b;
}

// What a kernel needs of a Packed beyond the planes (passed by value).
struct PackedRes {
    int p0;
    int bf;  // bf16 form: subtract 2^22 sum_k x_k too
    const int64_t *rowsum;
    const int *ptr, *col;
    const int64_t *val;
};

// Per-row scratch for rows whose columns are split between warps: a 128-bit
// accumulator kept as three limbs of 43, 43 and 42 bits in 64-bit words, and a
// count of column tiles done. Zero before the first launch; the warp that
// completes a row resets its entry.
struct RowAcc { unsigned long long l0, l1, l2; unsigned int done, pad; };

// Exact 128-bit accumulate without a carry chain: each limb of v (< 2^43)
// goes to its own word with a fire-and-forget atomic add; a row has at most
// 1024 adders here (2^53 per word at most), so no word can overflow, and the
// reader recombines l0 + 2^43 l1 + 2^86 l2 = sum of the v (mod 2^128).
__device__ __forceinline__ void racc_add(RowAcc *a, i128 v) {
    const u128 u = (u128)v;
    const uint64_t m43 = (1ull << 43) - 1;
    atomicAdd(&a->l0, (unsigned long long)((uint64_t)u & m43));
    atomicAdd(&a->l1, (unsigned long long)((uint64_t)(u >> 43) & m43));
    atomicAdd(&a->l2, (unsigned long long)(uint64_t)(u >> 86));
}
// Reads the sum and clears the entry (by the adder that completed the row).
__device__ __forceinline__ i128 racc_take(RowAcc *a) {
    const u128 l0 = atomicExch(&a->l0, 0ull), l1 = atomicExch(&a->l1, 0ull), l2 = atomicExch(&a->l2, 0ull);
    atomicExch(&a->done, 0u);
    return (i128)(l0 + (l1 << 43) + (l2 << 86));
}

// ---------------------------------------------------------------- packing

// Bytes needed to hold w as a signed (two's complement) integer, 1..8: the
// smallest n with -2^(8n-1) <= w < 2^(8n-1). A matrix whose weights all need
// <= n bytes is exactly sum_{p<n} B_p 2^{8p} with B_{n-1} read as signed (the
// bytes above it are its sign extension), so only n planes are stored.
__device__ __forceinline__ int bytes_needed(int64_t w) {
    uint64_t m = w < 0 ? ~(uint64_t)w : (uint64_t)w;  // magnitude bits below the sign
    int bits = 64 - __clzll((long long)m) + 1;          // + sign bit
    return (bits + 7) / 8;
}
// Plane statistics: st[0] = max bytes_needed; st[1 + b] (b = 0..7) = number of
// weights whose lowest nonzero byte is b (zero weights are not counted).
__global__ void k_plane_count(unsigned long long *__restrict__ st, const int64_t *__restrict__ W, int64_t n) {
    __shared__ unsigned long long hist[8];
    if (threadIdx.x < 8) hist[threadIdx.x] = 0;
    __syncthreads();
    int mx = 1;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t w = W[e];
        mx = max(mx, bytes_needed(w));
        if (w != 0) atomicAdd(&hist[(__ffsll(w) - 1) >> 3], 1ull);
    }
    for (int m = 16; m >= 1; m >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    if ((threadIdx.x & 31) == 0) atomicMax(&st[0], (unsigned long long)mx);
    __syncthreads();
    if (threadIdx.x < 8 && hist[threadIdx.x]) atomicAdd(&st[1 + threadIdx.x], hist[threadIdx.x]);
}

// Residual entries per row (weights with nonzero bytes below p0), one warp per row.
// The bf16 bits that hold w exactly in the bf16 form (w = v 2^24, v in
// [-2^22, 2^22) with at most 8 significant bits; v = 0 -> +0.0), else -1.
__host__ __device__ __forceinline__ int bf_encode(int64_t w) {
    if (w & 0xFFFFFF) return -1;
    const int64_t v = w >> 24;
    if (v < -(1 << 22) || v >= (1 << 22)) return -1;
    if (v == 0) return 0;
    const uint32_t a = (uint32_t)(v < 0 ? -v : v);
    int e2 = 31, tz = 0;
    while (!((a >> e2) & 1u)) e2--;
    while (!((a >> tz) & 1u)) tz++;
    if (e2 - tz >= 8) return -1;
    return (v < 0 ? 0x8000 : 0) | ((e2 + 103) << 7) | (int)(((a << 7) >> e2) & 0x7F);
}
// v of the bf16 form (0 where the weight is left to the residual)
__host__ __device__ __forceinline__ int64_t bf_v(int64_t w) { return bf_encode(w) < 0 ? 0 : (w >> 24); }
// Residual value of a weight: its bits in `mask` (plane window), or, with
// mask == 0 (bf16 form), the whole weight where the bf16 form cannot hold it.
__device__ __forceinline__ uint64_t res_value(int64_t w, uint64_t mask) {
    return mask ? ((uint64_t)w & mask) : (bf_encode(w) < 0 ? (uint64_t)w : 0ull);
}
__global__ void k_res_count(int *__restrict__ cnt, const int64_t *__restrict__ W, int M, int N, uint64_t mask) {
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
         row += gridDim.x * (blockDim.x >> 5)) {
        int c = 0;
        for (int k = lane; k < N; k += 32) c += res_value(W[(size_t)row * N + k], mask) != 0;
        for (int m = 16; m >= 1; m >>= 1) c += __shfl_xor_sync(0xffffffffu, c, m);
        if (lane == 0) cnt[row] = c;
    }
}
// Fills the CSR residual in column order (warp ballot per 32 columns).
__global__ void k_res_fill(int *__restrict__ col, int64_t *__restrict__ val, const int *__restrict__ ptr,
                           const int64_t *__restrict__ W, int M, int N, uint64_t mask) {
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < M;
         row += gridDim.x * (blockDim.x >> 5)) {
        int o = ptr[row];
        for (int k0 = 0; k0 < N; k0 += 32) {
            const int k = k0 + lane;
            const uint64_t lo = k < N ? res_value(W[(size_t)row * N + k], mask) : 0;
            const unsigned b = __ballot_sync(0xffffffffu, lo != 0);
            if (lo) {
                const int at = o + __popc(b & ((1u << lane) - 1));
                col[at] = k;
                val[at] = (int64_t)lo;
            }
            o += __popc(b);
        }
    }
}

// One thread per (row tile, column tile, lane): gathers the 16 weights of the
// lane's A fragment and writes its 16 bytes in each of the np planes.
__global__ void k_pack_planes(uint4 *__restrict__ planes, const int64_t *__restrict__ W, int M, int N,
                              int KT, int64_t total, int np, int p0) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int lane = (int)(e & 31);
        const int64_t tile = e >> 5;
        const int rt = (int)(tile / KT), kt = (int)(tile % KT);
        const int g = lane >> 2, t = lane & 3;
        uint64_t w[4][4];  // [reg][byte-lane]
#pragma unroll
        for (int r = 0; r < 4; r++) {
            int row = rt * 16 + g + ((r & 1) ? 8 : 0);
            int col0 = kt * 32 + 4 * t + ((r & 2) ? 16 : 0);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                int col = col0 + j;
                w[r][j] = (row < M && col < N) ? (uint64_t)W[(size_t)row * N + col] : 0ull;
            }
        }
        uint4 *dst = planes + (size_t)tile * np * 32 + lane;
#pragma unroll
        for (int p = 0; p < 8; p++) {
            if (p >= np) break;
            uint32_t v[4];
#pragma unroll
            for (int r = 0; r < 4; r++) {
                uint32_t b = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) b |= (uint32_t)((w[r][j] >> (8 * (p0 + p))) & 0xff) << (8 * j);
                v[r] = b;
            }
            dst[p * 32] = make_uint4(v[0], v[1], v[2], v[3]);
        }
    }
}

// ------------------------------------------------------------- bf16 form

#define IQ_BF_PAD 0xBE80u  // -0.25: u = 0

// Weights the bf16 form cannot hold exactly (its residual entries).
__global__ void k_bf_count(unsigned long long *__restrict__ cnt, const int64_t *__restrict__ W, int64_t n) {
    unsigned long long c = 0;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x)
        c += bf_encode(W[e]) < 0;
    for (int m = 16; m >= 1; m >>= 1) c += __shfl_xor_sync(0xffffffffu, c, m);
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(cnt, c);
}

// One thread per (row tile, column tile, lane): the lane's 16 weights as bf16.
__global__ void k_pack_bf(uint4 *__restrict__ words, const int64_t *__restrict__ W, int M, int N, int KT,
                          int64_t total) {
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int lane = (int)(e & 31);
        const int64_t tile = e >> 5;
        const int rt = (int)(tile / KT), kt = (int)(tile % KT);
        const int g = lane >> 2, t = lane & 3;
        uint32_t v[8];
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int row = rt * 16 + g + ((r & 1) ? 8 : 0);
            const int col0 = kt * 32 + 4 * t + ((r & 2) ? 16 : 0);
            uint32_t b[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int col = col0 + j;
                if (row < M && col < N) {
                    const int enc = bf_encode(W[(size_t)row * N + col]);
                    b[j] = enc < 0 ? 0u : (uint32_t)enc;
                } else {
                    b[j] = IQ_BF_PAD;
                }
            }
            v[2 * r] = b[0] | (b[1] << 16);
            v[2 * r + 1] = b[2] | (b[3] << 16);
        }
        uint4 *dst = words + (size_t)tile * 64 + lane;
        dst[0] = make_uint4(v[0], v[1], v[2], v[3]);
        dst[32] = make_uint4(v[4], v[5], v[6], v[7]);
    }
}

// 128-bit sum_k u_k = sum_k (v_k + 2^22) over the real columns (one warp per row).
__global__ void k_bf_row_sums(int64_t *__restrict__ rs, const int64_t *__restrict__ W, int M, int N, int Mp) {
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < Mp;
         row += gridDim.x * (blockDim.x >> 5)) {
        i128 s = 0;
        if (row < M)
            for (int k = lane; k < N; k += 32) s += (i128)(bf_v(W[(size_t)row * N + k]) + (1 << 22));
        s = warp_sum_i128(s);
        if (lane == 0) {
            rs[2 * row] = (int64_t)(uint64_t)s;
            rs[2 * row + 1] = (int64_t)(uint64_t)((u128)s >> 64);
        }
    }
}

// u of one bf16 weight held in the high half of f_bits: fp32 fma rounding
// toward -inf, exact (see the bf16 form above); the low 3 bytes are u's.
__device__ __forceinline__ uint32_t bf_u(uint32_t f_bits) {
    float r;
    asm("fma.rm.f32 %0, %1, 0f4B800000, 0f4B400000;" : "=f"(r) : "f"(__uint_as_float(f_bits)));
    return __float_as_uint(r);
}
// Four weights (bf16 pairs w01, w23; byte i = column k + i) -> their u bytes,
// one register per plane.
__device__ __forceinline__ void bf_quad(uint32_t w01, uint32_t w23, uint32_t &p0, uint32_t &p1, uint32_t &p2) {
    const uint32_t r0 = bf_u(w01 << 16), r1 = bf_u(w01 & 0xFFFF0000u);
    const uint32_t r2 = bf_u(w23 << 16), r3 = bf_u(w23 & 0xFFFF0000u);
    const uint32_t t01 = __byte_perm(r0, r1, 0x5140), t23 = __byte_perm(r2, r3, 0x5140);
    p0 = __byte_perm(t01, t23, 0x5410);
    p1 = __byte_perm(t01, t23, 0x7632);
    p2 = __byte_perm(__byte_perm(r0, r1, 0x0062), __byte_perm(r2, r3, 0x0062), 0x5410);
}

// 128-bit row sums of W with the bits in lo_mask cleared (one warp per row).
__global__ void k_row_sums(int64_t *__restrict__ rs, const int64_t *__restrict__ W, int M, int N, int Mp,
                           uint64_t lo_mask = 0) {
    const int lane = threadIdx.x & 31;
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < Mp;
         row += gridDim.x * (blockDim.x >> 5)) {
        i128 s = 0;
        if (row < M)
            for (int k = lane; k < N; k += 32) s += (i128)(int64_t)((uint64_t)W[(size_t)row * N + k] & ~lo_mask);
        s = warp_sum_i128(s);
        if (lane == 0) {
            rs[2 * row] = (int64_t)(uint64_t)s;
            rs[2 * row + 1] = (int64_t)(uint64_t)((u128)s >> 64);
        }
    }
}

// Fused gate|up rows [gate (half rows); up (half rows)] reordered so that each
// 16-row tile holds gate rows i..i+7 at tile rows 0..7 and the matching up
// rows at 8..15 (i = 8 * tile): a matvec epilogue that writes tile rows g and
// g + 8 together can then form SwiGLU directly (add mode IQ_EPI_SWIGLU).
// half must be a multiple of 8.
__global__ void k_interleave_pairs(int64_t *__restrict__ out, const int64_t *__restrict__ W, int half, int N) {
    const int64_t n = (int64_t)2 * half * N;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / N), k = (int)(e % N);
        const int tile = r >> 4, g = r & 15;
        const int src = g < 8 ? tile * 8 + g : half + tile * 8 + (g - 8);
        out[e] = W[(size_t)src * N + k];
    }
}

// Epilogue modes of the matvec kernels (their `add` argument).
#define IQ_EPI_STORE 0   // out[row] = result
#define IQ_EPI_ADD 1     // out[row] += result (residual, int64 wrap)
#define IQ_EPI_SWIGLU 2  // pair-interleaved gate|up rows: out[8 * tile + g] =
                         // fp_mul(fp_silu(gate), up) (llama_int.c:1549-1552)

// ----------------------------------------------------------------- kernel

__device__ __forceinline__ uint4 ld_stream_u4(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// D(16x8, s32) += A(16x32, u8 or s8) * B(32x8, u8)
template <bool ASIGNED>
__device__ __forceinline__ void mma_i8(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    if (ASIGNED)
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 "
                     "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
    else
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 "
                     "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// Folds the 8 plane accumulators of this lane into its two rows' 128-bit
// partials: lane (g, t) holds digits 2t, 2t+1 of rows g (c0, c1) and g+8 (c2, c3).
template <int NP>
__device__ __forceinline__ void fold_planes(int (&c)[NP][4], int t, i128 &r0, i128 &r1) {
#pragma unroll
    for (int p = 0; p < NP; p++) {
        const int s0 = 8 * (p + 2 * t);
        r0 += ((i128)c[p][0] << s0) + ((i128)c[p][1] << (s0 + 8));
        r1 += ((i128)c[p][2] << s0) + ((i128)c[p][3] << (s0 + 8));
#pragma unroll
        for (int q = 0; q < 4; q++) c[p][q] = 0;
    }
}

// Exact signed 64 x 64 -> 128-bit product from the two hardware halves (a
// plain (i128)a * b may be compiled as a full 128 x 128 multiply).
__device__ __forceinline__ i128 mul_wide(int64_t a, int64_t b) {
    const uint64_t lo = (uint64_t)a * (uint64_t)b;
    const int64_t hi = __mul64hi(a, b);
    return (i128)(((u128)(uint64_t)hi << 64) | lo);
}

// The row's result from its 128-bit plane sum `acc` (stored planes, before the
// 2^(8 p0) scale): scale, subtract 2^63 sum w_hi, add the sparse residual
// sum x_k w_lo,k (x from the staged digits when xd != nullptr, else from xg),
// then low64(>> 48) (llama_int.c:1044).
// The static per-row inputs of finish_row (row sum, residual range and its
// first entry), loadable before the kernel waits for its predecessor.
struct RowPre {
    i128 ws;
    int e0, e1, col0;
    int64_t val0;
};
__device__ __forceinline__ RowPre row_pre(int row, const PackedRes &R) {
    RowPre p;
    p.ws = (i128)(((u128)(uint64_t)R.rowsum[2 * row + 1] << 64) | (uint64_t)R.rowsum[2 * row]);
    p.e0 = p.e1 = p.col0 = 0;
    p.val0 = 0;
    if (R.ptr) {
        p.e0 = R.ptr[row];
        p.e1 = R.ptr[row + 1];
        if (p.e0 < p.e1) { p.col0 = R.col[p.e0]; p.val0 = R.val[p.e0]; }
    }
    return p;
}
__device__ __forceinline__ int64_t x_from_digits(const unsigned char *xd, int ld, int k) {
    uint64_t xu = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) xu |= (uint64_t)xd[j * ld + k] << (8 * j);
    return (int64_t)(xu ^ 0x8000000000000000ull);
}
__device__ __forceinline__ int64_t finish_row(i128 acc, const RowPre &p, const PackedRes &R,
                                              const unsigned char *xd, int ld, const int64_t *__restrict__ xg,
                                              i128 xs = 0) {
    // plane window: ws = sum w_hi (unscaled); bf16 form: ws = sum u, in units of
    // 2^24 like acc, and u = v + 2^22 also subtracts 2^22 sum x
    u128 v = R.bf ? ((u128)acc - ((u128)p.ws << 63) - ((u128)xs << 22)) << (8 * R.p0)
                  : ((u128)acc << (8 * R.p0)) - ((u128)p.ws << 63);
    for (int e = p.e0; e < p.e1; e++) {
        const int k = e == p.e0 ? p.col0 : R.col[e];
        const int64_t wl = e == p.e0 ? p.val0 : R.val[e];
        v += (u128)mul_wide(xd ? x_from_digits(xd, ld, k) : xg[k], wl);
    }
    return (int64_t)((i128)v >> 48);
}
__device__ __forceinline__ int64_t finish_row(i128 acc, int row, const PackedRes &R,
                                              const unsigned char *xd, int ld, const int64_t *__restrict__ xg,
                                              i128 xs = 0) {
    return finish_row(acc, row_pre(row, R), R, xd, ld, xg, xs);
}

// 4 digits j of x_u[k..k+3] packed into one word (byte i = element k+i)
__device__ __forceinline__ uint32_t digit_word(const int64_t *__restrict__ xg, int N, int k, int j) {
    uint32_t v = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint64_t xu = (k + i < N ? (uint64_t)__ldg(xg + k + i) : 0ull) ^ 0x8000000000000000ull;
        v |= (uint32_t)((xu >> (8 * j)) & 0xff) << (8 * i);
    }
    return v;
}

// Stages the 8 unsigned digit rows of x_u = x + 2^63 into shared memory
// (row j = byte j of every element, ld bytes apart; columns N..Kp are zero).
// Fused rmsnorm (llama_int.c:1048-1058) when nrm_w is given: the CTA computes
// the inverse rms of x itself and stages the digits of
// fp_mul(fp_mul(x, inv), w) instead of x.
// With xsum (bf16 form), every thread also receives sum_k x_k of the staged
// (normalised) values.
__device__ __forceinline__ void stage_digits(unsigned char *xd, int ld, const int64_t *__restrict__ xg, int N, int Kp,
                                             const int64_t *__restrict__ nrm_w, i128 *xsum = nullptr) {
    __shared__ uint64_t red[64];
    const int64_t inv = nrm_w ? cta_rms_inv(xg, N, red) : 0;
    i128 xs = 0;
    // each thread: 4 consecutive x values -> 8 digit words (one per digit row)
    for (int k = 4 * threadIdx.x; k < Kp; k += 4 * blockDim.x) {
        uint64_t xu[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int64_t xv = k + i < N ? __ldg(xg + k + i) : 0;
            if (nrm_w && k + i < N) xv = d_mul(d_mul(xv, inv), __ldg(nrm_w + k + i));
            xs += (i128)xv;
            xu[i] = (uint64_t)xv ^ 0x8000000000000000ull;
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t v = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) v |= (uint32_t)((xu[i] >> (8 * j)) & 0xff) << (8 * i);
            *reinterpret_cast<uint32_t *>(xd + j * ld + k) = v;
        }
    }
    if (xsum) *xsum = cta_sum_i128(xs, red);   // ends with a barrier-ordered read of red
    __syncthreads();
}

// Weight tiles in flight per warp: a register ring of D tiles, deeper when a
// tile is smaller (fewer planes), so the bytes in flight stay about constant.
// The ring is indexed statically (the unit loop is unrolled by D).
// (bf16 form: 2 x 16 bytes per lane and tile, like a 2-plane window.)
#ifndef IQ_BF_RING
#define IQ_BF_RING 6
#endif
template <int NP, bool BF = false>
__host__ __device__ constexpr int ring_depth() {
    return BF ? IQ_BF_RING : NP <= 2 ? 6 : NP == 3 ? 4 : NP == 4 ? 3 : 2;
}
// 16-byte loads per lane and tile
template <int NP, bool BF>
__host__ __device__ constexpr int tile_loads() { return BF ? 2 : NP; }

template <int NL>
__device__ __forceinline__ void load_tile(uint4 (&dst)[NL], const uint4 *src) {
#pragma unroll
    for (int p = 0; p < NL; p++) dst[p] = ld_stream_u4(src + p * 32);
}

template <int NP>
__device__ __forceinline__ void mma_tile(int (&c)[NP][4], const uint4 (&a)[NP], uint32_t b0, uint32_t b1) {
#pragma unroll
    for (int p = 0; p < NP - 1; p++) mma_i8<false>(c[p], a[p], b0, b1);
    mma_i8<true>(c[NP - 1], a[NP - 1], b0, b1);  // top plane: signed
}
// bf16 form: the lane's 16 weights -> u's three unsigned planes -> 3 MMAs
__device__ __forceinline__ void mma_tile_bf(int (&c)[3][4], const uint4 (&w)[2], uint32_t b0, uint32_t b1) {
    uint4 a[3];
    bf_quad(w[0].x, w[0].y, a[0].x, a[1].x, a[2].x);
    bf_quad(w[0].z, w[0].w, a[0].y, a[1].y, a[2].y);
    bf_quad(w[1].x, w[1].y, a[0].z, a[1].z, a[2].z);
    bf_quad(w[1].z, w[1].w, a[0].w, a[1].w, a[2].w);
#pragma unroll
    for (int p = 0; p < 3; p++) mma_i8<false>(c[p], a[p], b0, b1);
}
template <int NP, bool BF, int NL>
__device__ __forceinline__ void mma_any(int (&c)[NP][4], const uint4 (&a)[NL], uint32_t b0, uint32_t b1) {
    if constexpr (BF) {
        static_assert(NP == 3 && NL == 2, "bf16 form: 3 planes from 2 loads");
        mma_tile_bf(c, a, b0, b1);
    } else {
        mma_tile<NP>(c, a, b0, b1);
    }
}

// Pulls the flush's static row data (row sums, residual offsets) of row tile
// rt into L1 ahead of its use (lanes t == 0 of the 8 row groups: rows g, g+8).
__device__ __forceinline__ void prefetch_rows(const PackedRes &R, int rt, int M, int g, int t) {
    if (t != 0) return;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int row = rt * 16 + g + 8 * h;
        if (row >= M) continue;
        asm volatile("prefetch.global.L1 [%0];" :: "l"(R.rowsum + 2 * row));
        if (R.ptr) asm volatile("prefetch.global.L1 [%0];" :: "l"(R.ptr + row));
    }
}

// End of a warp's segment of row tile rt (column tiles k0 .. k1-1): the 4 lanes
// of each row group sum their digits' partials, then the row's writer either
// owns the whole row (k0 == 0, k1 == KT) or meets the other segments in the
// RowAcc scratch, and the one completing the row writes it. Kept out of line:
// inlined into every slot of the unrolled ring it multiplied the code size and
// the kernel stalled on instruction fetch.
__device__ __noinline__ void flush_segment(i128 r0, i128 r1, int rt, int k0, int k1, int KT, int M, int add,
                                           int64_t *__restrict__ out, RowAcc *__restrict__ racc, const PackedRes R,
                                           const unsigned char *xd, int ld, const int64_t *__restrict__ xg, i128 xs,
                                           int g, int t) {
    // the 4 lanes of a row group hold the 8 digits: reduce over t
#pragma unroll
    for (int m = 1; m <= 2; m <<= 1) {
        r0 += shfl_xor_i128(r0, m);
        r1 += shfl_xor_i128(r1, m);
    }
    if (t == 0 && add == IQ_EPI_SWIGLU) {
        // rows g (gate) and g + 8 (up) complete together: one counter
        const int row = rt * 16 + g;
        i128 f0 = r0, f1 = r1;
        bool write = k0 == 0 && k1 == KT;
        if (!write) {
            RowAcc *ra = racc + row, *rb = racc + row + 8;
            racc_add(ra, r0);
            racc_add(rb, r1);
            // release our limbs / acquire everyone else's with the counter
            cuda::atomic_ref<unsigned int, cuda::thread_scope_device> done(ra->done);
            unsigned int prev = done.fetch_add((unsigned int)(k1 - k0), cuda::memory_order_acq_rel);
            if (prev + (unsigned int)(k1 - k0) == (unsigned int)KT) {
                f0 = racc_take(ra);
                f1 = racc_take(rb);
                write = true;
            }
        }
        if (write) {
            const int64_t gate = finish_row(f0, row, R, xd, ld, xg, xs);
            const int64_t up = finish_row(f1, row + 8, R, xd, ld, xg, xs);
            out[rt * 8 + g] = d_mul(d_silu(gate), up);
        }
    } else if (t == 0) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int row = rt * 16 + g + 8 * h;
            if (row >= M) continue;
            i128 part = h ? r1 : r0;
            i128 fin = 0;
            bool write = false;
            if (k0 == 0 && k1 == KT) { fin = part; write = true; }
            else {
                RowAcc *ra = racc + row;
                racc_add(ra, part);
                // release our limbs / acquire everyone else's with the counter
                cuda::atomic_ref<unsigned int, cuda::thread_scope_device> done(ra->done);
                unsigned int prev = done.fetch_add((unsigned int)(k1 - k0), cuda::memory_order_acq_rel);
                if (prev + (unsigned int)(k1 - k0) == (unsigned int)KT) {
                    fin = racc_take(ra);
                    write = true;
                }
            }
            if (write) {
                int64_t val = finish_row(fin, row, R, xd, ld, xg, xs);
                // add != 0: residual epilogue out += result (int64 wrap, llama_int.c:1535, 1556)
                out[row] = add ? (int64_t)((uint64_t)out[row] + (uint64_t)val) : val;
            }
        }
    }
}

// Stream-K kernel. XSMEM: digits staged in shared memory (Kp small enough),
// else gathered from x in global memory (L1-cached) per column tile.
// Each warp walks its units linearly (row tile-major, the packed layout's
// order) with ring_depth<NP>() tiles in flight; the first D-1 are requested
// before griddepcontrol.wait (weights are static), overlapping the previous
// kernel's tail and the digit staging.
// Profiling hook of the persistent decode kernel (defined there).
__device__ __forceinline__ void mv_mark(int tag);

// The stream-K matvec over warps gw of nwarps (the whole grid for a kernel
// launch; a persistent kernel passes its own). xd: the CTA's digit staging
// area. PDL: programmatic dependent launch (the first ring loads go out
// before waiting for the previous kernel).
template <int NP, bool XSMEM, bool BF, bool PDL>
__device__ __forceinline__ void mv_stream(int64_t *__restrict__ out, const uint4 *__restrict__ planes,
                                          const PackedRes &R, const int64_t *__restrict__ xg, int M, int N, int Kp,
                                          int add, RowAcc *__restrict__ racc, const int64_t *__restrict__ nrm_w,
                                          unsigned char *xd, int64_t gw, int64_t nwarps) {
    static_assert(!BF || XSMEM, "the bf16 form needs the staged activations (their sum)");
    constexpr int D = ring_depth<NP, BF>();
    constexpr int NL = tile_loads<NP, BF>();
    constexpr int TS = NL * 32;  // uint4 per packed tile
    const int ld = Kp + 16;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int KT = Kp / 32, RT = (M + 15) / 16;
    const int64_t total = (int64_t)RT * KT;
    const int64_t u0 = total * gw / nwarps, u1 = total * (gw + 1) / nwarps;
    // Programmatic dependent launch: let the next kernel in the stream start its
    // own prologue now; it waits (griddepcontrol.wait) for this grid's results.
    if (PDL) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint4 *pl = planes + lane;
    uint4 buf[D][NL];
#pragma unroll
    for (int s = 0; s < D - 1; s++)
        if (u0 + s < u1) load_tile<NL>(buf[s], pl + (size_t)(u0 + s) * TS);
    // x and (with add) out are produced by the previous kernel
    if (PDL) asm volatile("griddepcontrol.wait;" ::: "memory");
    i128 xs = 0;
    if (XSMEM) stage_digits(xd, ld, xg, N, Kp, nrm_w, BF ? &xs : nullptr);
    if (!PDL) mv_mark(6);
    const unsigned char *xb = xd + g * ld + 4 * t;

    int c[NP][4];
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
        for (int q = 0; q < 4; q++) c[p][q] = 0;
    i128 r0 = 0, r1 = 0;
    int since_fold = 0;
    // current row tile and column tile; the segment of rt this warp owns began at k0
    int rt = (int)(u0 / KT), kt = (int)(u0 - (int64_t)rt * KT), k0 = kt;
    // units are consecutive tiles in memory: the ring's next request walks linearly
    const uint4 *pnext = pl + (size_t)(u0 + D - 1) * TS;
    const uint4 *const pend = pl + (size_t)u1 * TS;
    const int n = (int)(u1 - u0);
    if (n > 0) prefetch_rows(R, rt, M, g, t);
    for (int ib = 0; ib < n; ib += D) {
#pragma unroll
        for (int s = 0; s < D; s++) {
            if (ib + s >= n) break;
            if (pnext < pend) load_tile<NL>(buf[(s + D - 1) % D], pnext);
            pnext += TS;
            const int kk = kt * 32;
            uint32_t b0, b1;
            if (XSMEM) {
                b0 = *reinterpret_cast<const uint32_t *>(xb + kk);
                b1 = *reinterpret_cast<const uint32_t *>(xb + kk + 16);
            } else {
                b0 = digit_word(xg, N, kk + 4 * t, g);
                b1 = digit_word(xg, N, kk + 16 + 4 * t, g);
            }
            mma_any<NP, BF, NL>(c, buf[s], b0, b1);
            // staged rows have KT <= 399 tiles, so a segment never reaches the
            // 1024 tiles after which the int32 plane sums must be folded
            if (!XSMEM && ++since_fold >= 1024) { fold_planes(c, t, r0, r1); since_fold = 0; }
            if (++kt == KT) {  // row tile complete: flush this warp's part of it
                fold_planes(c, t, r0, r1);
                since_fold = 0;
                flush_segment(r0, r1, rt, k0, KT, KT, M, add, out, racc, R, XSMEM ? xd : nullptr, ld, xg, xs, g, t);
                r0 = 0;
                r1 = 0;
                rt += 1;
                kt = 0;
                k0 = 0;
                if (ib + s + 1 < n) prefetch_rows(R, rt, M, g, t);
            }
        }
    }
    if (kt != k0) {  // the warp's range ended inside row tile rt
        fold_planes(c, t, r0, r1);
        flush_segment(r0, r1, rt, k0, kt, KT, M, add, out, racc, R, XSMEM ? xd : nullptr, ld, xg, xs, g, t);
    }
    if (!PDL) mv_mark(7);
}


template <int NP, bool XSMEM, bool BF = false>
__global__ void __launch_bounds__(256, 2)
k_matvec_planes(int64_t *__restrict__ out, const uint4 *__restrict__ planes, const PackedRes R,
                const int64_t *__restrict__ xg, int M, int N, int Kp, int add, RowAcc *__restrict__ racc,
                const int64_t *__restrict__ nrm_w) {
    extern __shared__ __align__(16) unsigned char xd[];  // [8][Kp + 16] digit rows
    mv_stream<NP, XSMEM, BF, true>(out, planes, R, xg, M, N, Kp, add, racc, nrm_w, xd,
                                   (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5),
                                   (int64_t)gridDim.x * (blockDim.x >> 5));
}

// End of a row tile in k_matvec_rows (every thread of the CTA calls it): the
// warps' partials meet in shared memory, then (S > 1) the CTAs' in rank 0's
// over distributed shared memory, and 16 threads finish and write the rows.
// Returns true for cluster ranks > 0, which are done (one tile per cluster).
// Out of line, as flush_segment, so the unrolled ring stays small.
__device__ __noinline__ bool rows_tile_end(i128 r0, i128 r1, int rt, int rt0, const RowPre pre0, uint32_t S,
                                           uint32_t crank, int M, int add, int64_t *__restrict__ out,
                                           const PackedRes R, const unsigned char *xd, int ld,
                                           const int64_t *__restrict__ xg, i128 xs, unsigned long long *wpart,
                                           unsigned long long *cpart) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int m = 1; m <= 2; m <<= 1) {  // the 4 lanes of a row group hold the 8 digits
        r0 += shfl_xor_i128(r0, m);
        r1 += shfl_xor_i128(r1, m);
    }
    // wpart [8 warps][16 rows][2], cpart [8 ranks][16 rows][2]
    if (t == 0) {
        wpart[(warp * 16 + g) * 2] = (uint64_t)r0; wpart[(warp * 16 + g) * 2 + 1] = (uint64_t)((u128)r0 >> 64);
        wpart[(warp * 16 + g + 8) * 2] = (uint64_t)r1;
        wpart[(warp * 16 + g + 8) * 2 + 1] = (uint64_t)((u128)r1 >> 64);
    }
    __syncthreads();
    i128 v = 0;
    if (threadIdx.x < 16) {
#pragma unroll
        for (int w = 0; w < 8; w++)
            v += (i128)(((u128)wpart[(w * 16 + threadIdx.x) * 2 + 1] << 64) | wpart[(w * 16 + threadIdx.x) * 2]);
    }
    if (S > 1) {
        asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
        if (threadIdx.x < 16) {
            uint32_t remote;
            asm volatile("mapa.shared::cluster.u32 %0, %1, 0;"
                         : "=r"(remote)
                         : "r"((uint32_t)__cvta_generic_to_shared(&cpart[(crank * 16 + threadIdx.x) * 2])));
            asm volatile("st.shared::cluster.v2.u64 [%0], {%1, %2};"
                         :: "r"(remote), "l"((uint64_t)v), "l"((uint64_t)((u128)v >> 64)) : "memory");
        }
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
        if (crank != 0) return true;
        if (threadIdx.x < 16) {
            v = 0;
            for (uint32_t r = 0; r < S; r++)
                v += (i128)(((u128)cpart[(r * 16 + threadIdx.x) * 2 + 1] << 64) | cpart[(r * 16 + threadIdx.x) * 2]);
        }
    }
    const int row = rt * 16 + (int)threadIdx.x;
    int64_t val = 0;
    if (threadIdx.x < 16 && row < M) {
        const RowPre pre = rt != rt0 ? row_pre(row, R) : pre0;
        val = finish_row(v, pre, R, xd, ld, xg, xs);
        if (add != IQ_EPI_SWIGLU) out[row] = add ? (int64_t)((uint64_t)out[row] + (uint64_t)val) : val;
    }
    if (add == IQ_EPI_SWIGLU && warp == 0) {  // tile rows g (gate) and g + 8 (up)
        const int64_t up = __shfl_down_sync(0xffffffffu, val, 8);
        if (lane < 8 && rt * 16 + lane < M) out[rt * 8 + lane] = d_mul(d_silu(val), up);
    }
    __syncthreads();  // wpart is rewritten by the next tile
    return false;
}

// Row-owned variant: a cluster of S CTAs (S = 1, 2, 4 or 8) owns one 16-row
// tile (S = 1: a CTA owns every gridDim-th tile in turn), its 8*S warps split
// the column tiles evenly (nk each; the last ones may hold fewer or none),
// the warps' 128-bit partials are summed in shared memory and the S CTA sums
// in rank 0's shared memory (distributed shared memory), which writes the 16
// outputs. No global atomics and no scratch; the result is the same integer
// (addition mod 2^128 is associative). Every warp runs the same number of
// unit steps (ntiles * nk, empty ones skipped), so the per-tile barriers are
// reached in step. Staged digits only (Kp <= 12784: fewer than 1024 column
// tiles per warp, so the int32 plane sums cannot overflow before the fold).
template <int NP, bool BF = false>
__global__ void __launch_bounds__(256, 2)
k_matvec_rows(int64_t *__restrict__ out, const uint4 *__restrict__ planes, const PackedRes R,
              const int64_t *__restrict__ xg, int M, int N, int Kp, int add, const int64_t *__restrict__ nrm_w) {
    extern __shared__ __align__(16) unsigned char xd[];  // [8][Kp + 16] digit rows
    __shared__ __align__(16) unsigned long long wpart[8][16][2];  // per warp: 16 row partials (lo, hi)
    __shared__ __align__(16) unsigned long long cpart[8][16][2];  // per cluster rank (read in rank 0)
    constexpr int D = ring_depth<NP, BF>();
    constexpr int NL = tile_loads<NP, BF>();
    constexpr int TS = NL * 32;  // uint4 per packed tile
    const int ld = Kp + 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int KT = Kp / 32, RT = (M + 15) / 16;
    uint32_t S, crank;
    asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(S));
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
    // row tiles rt0, rt0 + stride, ... (one tile per cluster when S > 1)
    const int rt0 = blockIdx.x / S, stride = gridDim.x / S;
    const int ntiles = rt0 < RT ? (RT - 1 - rt0) / stride + 1 : 0;
    const int nwi = S * 8, nk = (KT + nwi - 1) / nwi;
    const int k0 = (crank * 8 + warp) * nk, k1 = min(KT, k0 + nk);
    const int total = ntiles * nk;  // unit steps, the same for every warp of the cluster
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // every CTA of the cluster must be running before rank 0's shared memory is
    // written: arrive now, wait just before the write
    if (S > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    // prefetch cursor: step pj of the tile whose column tile k0 starts at pbase
    // (unit step q is tile q / nk, column tile k0 + q % nk; empty past k1)
    int pj = 0;
    const uint4 *pbase = planes + lane + ((size_t)rt0 * KT + k0) * TS;
    const size_t tile_step = (size_t)stride * KT * TS;
    auto prefetch = [&](uint4 (&dst)[NL]) {
        if (k0 + pj < k1) load_tile<NL>(dst, pbase + (size_t)pj * TS);
        if (++pj == nk) { pj = 0; pbase += tile_step; }
    };
    uint4 buf[D][NL];
#pragma unroll
    for (int s = 0; s < D - 1; s++)
        if (s < total) prefetch(buf[s]);
    // the writers' static row data for the first tile (row sums, residual)
    RowPre pre = {};
    if (threadIdx.x < 16 && ntiles > 0 && rt0 * 16 + (int)threadIdx.x < M) pre = row_pre(rt0 * 16 + threadIdx.x, R);
    // x and (with add) out are produced by the previous kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    i128 xs = 0;
    stage_digits(xd, ld, xg, N, Kp, nrm_w, BF ? &xs : nullptr);
    const unsigned char *xb = xd + g * ld + 4 * t;
    int c[NP][4];
#pragma unroll
    for (int p = 0; p < NP; p++)
#pragma unroll
        for (int q = 0; q < 4; q++) c[p][q] = 0;
    int j = 0, rt = rt0;  // current step within the tile, current tile
    for (int qb = 0; qb < total; qb += D) {
#pragma unroll
        for (int s = 0; s < D; s++) {
            const int q = qb + s;
            if (q >= total) break;
            if (q + D - 1 < total) prefetch(buf[(s + D - 1) % D]);
            const int kt = k0 + j;
            if (kt < k1) {
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xb + kt * 32);
                const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xb + kt * 32 + 16);
                mma_any<NP, BF, NL>(c, buf[s], b0, b1);
            }
            if (++j < nk) continue;
            // ---- end of this warp's part of tile rt: reduce and write
            j = 0;
            i128 r0 = 0, r1 = 0;
            fold_planes(c, t, r0, r1);
            if (rows_tile_end(r0, r1, rt, rt0, pre, S, crank, M, add, out, R, xd, ld, xg, xs, &wpart[0][0][0],
                              &cpart[0][0][0]))
                return;  // cluster rank > 0: one tile per cluster
            rt += stride;
        }
    }
    if (S > 1 && total == 0) {  // keep the cluster barrier phases matched
        asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
}

}  // namespace iq
