// iq_layer.cuh -- device kernels of the integer Llama layer around the matvecs
// (transformer_layer_forward, llama_int.c:1326-1569; llama_forward,
// llama_int.c:2807-2886). All kernels take the token position (and token id)
// from device memory so a whole decode step can be captured in a CUDA graph
// and replayed per token. Layouts (int64 Q16.48 everywhere):
//   qkv     [B][dim + 2*kvd]   q | k | v as produced by the fused QKV matvec
//   kcache  [L][B][max_seq][kvd], vcache same  (per layer, per sequence)
//   rope    cos/sin [max_seq][hd/2]            (rope_init table layout, llama_int.c:960-986)
#pragma once
#include "iq_elem.cuh"

namespace iq {

// hidden[b] = embed[token[b]] (llama_int.c:2822-2824)
__global__ void k_embed(int64_t *__restrict__ hidden, const int64_t *__restrict__ embed,
                        const int *__restrict__ tokens, int dim) {
    const int b = blockIdx.y;
    const int64_t *src = embed + (size_t)tokens[b] * dim;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x)
        hidden[(size_t)b * dim + i] = src[i];
}

// RoPE on all q heads and the k heads (rope_apply, llama_int.c:997-1008), then the
// exact K/V cache write at pos (llama_int.c:1415-1416). One thread per rotation pair.
// Row r of qkv belongs to sequence seq_arr[r] at position pos_arr[r].
__global__ void k_rope_kv(int64_t *__restrict__ qkv, int64_t *__restrict__ kc, int64_t *__restrict__ vc,
                          const int64_t *__restrict__ rcos, const int64_t *__restrict__ rsin,
                          const int *__restrict__ pos_arr, const int *__restrict__ seq_arr, int nh, int nkv,
                          int hd, int max_seq) {
    const int b = blockIdx.y;
    const int half = hd / 2, dim = nh * hd, kvd = nkv * hd;
    const int pos = pos_arr[b], sq = seq_arr[b];
    int64_t *row = qkv + (size_t)b * (dim + 2 * kvd);
    const int64_t *c = rcos + (size_t)pos * half, *s = rsin + (size_t)pos * half;
    int64_t *kdst = kc + ((size_t)sq * max_seq + pos) * kvd;
    int64_t *vdst = vc + ((size_t)sq * max_seq + pos) * kvd;
    const int npairs = (nh + nkv) * half;
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < npairs + kvd; p += gridDim.x * blockDim.x) {
        if (p < npairs) {
            int h = p / half, i = p % half;
            int64_t *v = row + h * hd;  // q heads then k heads are contiguous
            int64_t x0 = v[i], x1 = v[i + half];
            int64_t a = d_mul(x0, c[i]) - d_mul(x1, s[i]);
            int64_t bb = d_mul(x1, c[i]) + d_mul(x0, s[i]);
            if (h < nh) { v[i] = a; v[i + half] = bb; }
            else {
                int kh = h - nh;
                kdst[kh * hd + i] = a;
                kdst[kh * hd + i + half] = bb;
            }
        } else {
            int j = p - npairs;
            vdst[j] = row[dim + kvd + j];
        }
    }
}

// signed 64x64 -> 128 product
__device__ __forceinline__ i128 d_mul128(int64_t a, int64_t b) {
    uint64_t lo = (uint64_t)a * (uint64_t)b;
    int64_t hi = __mul64hi(a, b);
    return (i128)(((u128)(uint64_t)hi << 64) | lo);
}

// Exact GQA attention for one (sequence, q head) per CTA, llama_int.c:1432-1529:
//   score_t = fp_mul((int64)(sum_d (i128)q[d]*k_t[d] >> 48), fp_inv_sqrt(fp_from_int(hd)))
//   p = softmax(score) (llama_int.c:1060-1072)
//   out[d] = sum_t fp_mul(p_t, v_t[d])   (int64 sum of floor-shifted terms)
// Scores live in dynamic shared memory ([T] int64); q_h in shared memory.
// Row b = (sequence seq_arr[b], position pos_arr[b]) attends to positions
// 0..pos of its sequence: a batched prefill row computes exactly what the
// reference's sequential call at that position computes.
// ROPE (decode steps, one row per sequence): the CTA also applies RoPE itself
// (rope_apply, llama_int.c:997-1008) to its q head and to its kv head's k, and
// writes the cache row at pos (llama_int.c:1415-1416) before reading the
// cache; every CTA of a kv group writes the same values, so each reads its own
// write and no separate RoPE / cache-write kernel runs.
template <bool ROPE>
__global__ void k_attention(int64_t *__restrict__ out, const int64_t *__restrict__ qkv,
                            int64_t *__restrict__ kc, int64_t *__restrict__ vc,
                            const int *__restrict__ pos_arr, const int *__restrict__ seq_arr, int nh, int nkv,
                            int hd, int max_seq, int64_t scale, const int64_t *__restrict__ rcos,
                            const int64_t *__restrict__ rsin) {
    extern __shared__ __align__(16) int64_t sm[];
    __shared__ uint64_t red[64];
    const int h = blockIdx.x, b = blockIdx.y;
    const int dim = nh * hd, kvd = nkv * hd, kvh = h / (nh / nkv);
    const int T = pos_arr[b] + 1;
    int64_t *qs = sm;            // [hd]
    int64_t *sc = sm + hd;       // [T]
    const int64_t *q = qkv + (size_t)b * (dim + 2 * kvd) + h * hd;
    if (ROPE) {
        const int pos = T - 1, half = hd / 2, sqr = seq_arr[b];
        const int64_t *c = rcos + (size_t)pos * half, *sn = rsin + (size_t)pos * half;
        const int64_t *k = qkv + (size_t)b * (dim + 2 * kvd) + dim + kvh * hd;
        int64_t *kdst = kc + ((size_t)sqr * max_seq + pos) * kvd + kvh * hd;
        int64_t *vdst = vc + ((size_t)sqr * max_seq + pos) * kvd + kvh * hd;
        for (int i = threadIdx.x; i < half; i += blockDim.x) {
            const int64_t x0 = q[i], x1 = q[i + half], k0 = k[i], k1 = k[i + half];
            qs[i] = d_mul(x0, c[i]) - d_mul(x1, sn[i]);
            qs[i + half] = d_mul(x1, c[i]) + d_mul(x0, sn[i]);
            kdst[i] = d_mul(k0, c[i]) - d_mul(k1, sn[i]);
            kdst[i + half] = d_mul(k1, c[i]) + d_mul(k0, sn[i]);
        }
        for (int i = threadIdx.x; i < hd; i += blockDim.x) vdst[i] = k[kvd + i];
    } else {
        for (int d = threadIdx.x; d < hd; d += blockDim.x) qs[d] = q[d];
    }
    __syncthreads();
    const int sq = seq_arr[b];
    const int64_t *kb = kc + (size_t)sq * max_seq * kvd + kvh * hd;
    const int64_t *vb = vc + (size_t)sq * max_seq * kvd + kvh * hd;
    // scores: groups of 8 lanes share one position and split its dims, so a
    // warp reads four key rows in 64-byte coalesced pieces; the int128 partial
    // dots combine exactly (addition mod 2^128). Each lane issues all its key
    // loads for two positions before multiplying, so the L2 latencies overlap.
    {
        const int sl = threadIdx.x & 7, nsg = blockDim.x >> 3;
        for (int tb = 0; tb < T; tb += 2 * nsg) {  // uniform trip count: every lane shuffles
            const int ta = tb + (threadIdx.x >> 3), tc = ta + nsg;
            const bool aa = ta < T, ac = tc < T;
            const int64_t *ka = kb + (size_t)(aa ? ta : 0) * kvd, *kc2 = kb + (size_t)(ac ? tc : 0) * kvd;
            i128 da = 0, dc = 0;
            for (int d0 = 0; d0 < hd; d0 += 64) {
                int64_t va[8], vc2[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int d = d0 + sl + 8 * j;
                    va[j] = aa && d < hd ? ka[d] : 0;
                    vc2[j] = ac && d < hd ? kc2[d] : 0;
                }
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int d = d0 + sl + 8 * j;
                    const int64_t qv = d < hd ? qs[d] : 0;
                    da += d_mul128(qv, va[j]);
                    dc += d_mul128(qv, vc2[j]);
                }
            }
#pragma unroll
            for (int m = 4; m >= 1; m >>= 1) {
                da += shfl_xor_i128(da, m);
                dc += shfl_xor_i128(dc, m);
            }
            if (sl == 0) {
                if (aa) sc[ta] = d_mul((int64_t)(da >> 48), scale);
                if (ac) sc[tc] = d_mul((int64_t)(dc >> 48), scale);
            }
        }
    }
    __syncthreads();
    cta_softmax(sc, T, red);
    __syncthreads();
    // PV: thread groups of hd threads split t; int64 partial sums combine
    // exactly (mod 2^64). Eight value loads are issued before their multiplies.
    const int groups = blockDim.x / hd;
    const int g = threadIdx.x / hd, d = threadIdx.x % hd;
    uint64_t acc = 0;
    if (g < groups) {
        int t = g;
        for (; t + 7 * groups < T; t += 8 * groups) {
            int64_t vv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) vv[j] = vb[(size_t)(t + j * groups) * kvd + d];
#pragma unroll
            for (int j = 0; j < 8; j++) acc += (uint64_t)d_mul(sc[t + j * groups], vv[j]);
        }
        for (; t < T; t += groups) acc += (uint64_t)d_mul(sc[t], vb[(size_t)t * kvd + d]);
    }
    __syncthreads();
    int64_t *part = sm + hd;  // reuse the score area: [groups][hd]
    if (g < groups) part[g * hd + d] = (int64_t)acc;
    __syncthreads();
    for (int dd = threadIdx.x; dd < hd; dd += blockDim.x) {
        uint64_t s = 0;
        for (int gg = 0; gg < groups; gg++) s += (uint64_t)part[gg * hd + dd];
        out[(size_t)b * dim + h * hd + dd] = (int64_t)s;
    }
}

// fp_inv_sqrt(fp_from_int(hd)): the attention score scale (llama_int.c:1433),
// computed once per model on the device.
__global__ void k_att_scale(int64_t *out, int hd) { *out = d_inv_sqrt(d_from_int(hd)); }

// Exact attention with coalesced K tiles: one CTA per (row b, block of hpc
// query heads that share one kv head; hpc divides nh / nkv). Keys are staged
// ATT_TT positions at a time into shared memory with coalesced loads, and
// each thread computes whole dots from there; V is read coalesced across d.
// Heads of one kv group are adjacent CTAs, so their K/V re-reads hit L2.
// Same arithmetic as k_attention (llama_int.c:1432-1529): int128 QK dots,
// fp_mul by 1/sqrt(hd), integer softmax, int64 sum of fp_mul(p_t, v_t[d]).
// Shared memory: q [hpc][hd] | scores [hpc][Tcap] | K tile [ATT_TT][hd + 1].
#define ATT_TT 64
__global__ void __launch_bounds__(256)
k_attention_gqa(int64_t *__restrict__ out, const int64_t *__restrict__ qkv, const int64_t *__restrict__ kc,
                const int64_t *__restrict__ vc, const int *__restrict__ pos_arr, const int *__restrict__ seq_arr,
                int nh, int nkv, int hd, int max_seq, int Tcap, int hpc) {
    extern __shared__ __align__(16) int64_t sm[];
    __shared__ uint64_t red[64];
    const int b = blockIdx.y, h0 = blockIdx.x * hpc;
    const int grp = hpc, dim = nh * hd, kvd = nkv * hd, g = h0 / (nh / nkv);
    const int T = pos_arr[b] + 1, sq = seq_arr[b];
    int64_t *qs = sm;                       // [grp][hd]
    int64_t *sc = qs + grp * hd;            // [grp][Tcap]
    int64_t *kt = sc + (size_t)grp * Tcap;  // [ATT_TT][hd + 1]
    const int kld = hd + 1;
    const int64_t *q = qkv + (size_t)b * (dim + 2 * kvd) + (size_t)h0 * hd;
    for (int e = threadIdx.x; e < grp * hd; e += blockDim.x) qs[e] = q[e];
    const int64_t scale = d_inv_sqrt(d_from_int(hd));
    const int64_t *kb = kc + (size_t)sq * max_seq * kvd + g * hd;
    const int64_t *vb = vc + (size_t)sq * max_seq * kvd + g * hd;
    for (int t0 = 0; t0 < T; t0 += ATT_TT) {
        const int nt = min(ATT_TT, T - t0);
        __syncthreads();
        for (int e = threadIdx.x; e < nt * hd; e += blockDim.x) {  // coalesced K tile load
            int tt = e / hd, dd = e % hd;
            kt[tt * kld + dd] = kb[(size_t)(t0 + tt) * kvd + dd];
        }
        __syncthreads();
        for (int e = threadIdx.x; e < grp * ATT_TT; e += blockDim.x) {
            int hh = e / ATT_TT, tt = e % ATT_TT;
            if (tt < nt) {
                const int64_t *qh = qs + hh * hd, *kr = kt + tt * kld;
                i128 dot = 0;
                for (int dd = 0; dd < hd; dd++) dot += d_mul128(qh[dd], kr[dd]);
                sc[(size_t)hh * Tcap + t0 + tt] = d_mul((int64_t)(dot >> 48), scale);
            }
        }
    }
    __syncthreads();
    for (int hh = 0; hh < grp; hh++) {
        cta_softmax(sc + (size_t)hh * Tcap, T, red);
        __syncthreads();
    }
    for (int e = threadIdx.x; e < grp * hd; e += blockDim.x) {
        const int hh = e / hd, dd = e % hd;
        const int64_t *p = sc + (size_t)hh * Tcap;
        uint64_t acc = 0;
        for (int t = 0; t < T; t++) acc += (uint64_t)d_mul(p[t], vb[(size_t)t * kvd + dd]);
        out[(size_t)b * dim + (size_t)(h0 + hh) * hd + dd] = (int64_t)acc;
    }
}

// ---------------------------------------------------------------------------
// Packed KV cache (the reference's --kv-packed KbVb, llama_int.c:1197-1235,
// 1392-1411, 1435-1501): per (position, kv head) vector an L-inf magnitude M
// and b-bit codes q = ((x + M) * 2^b) / (2M) (int128, truncating, clamped to
// [0, 2^b - 1]); attention reads back ((2q + 1) M) / 2^b - M. Lossy, but the
// same integers as the reference, so still bit-exact against it.
struct KVView {
    const int64_t *x;       // exact cache (packed == 0)
    const uint8_t *k8;      // K codes (packed, keys)
    const uint16_t *v16;    // V codes (packed, values)
    const int64_t *mag;     // [seq][max_seq][nkv] magnitudes
    int bits, nkv, hd;
    // element e of vector vec (= (seq * max_seq + t) * nkv + head)
    __device__ __forceinline__ int64_t at(size_t elem, size_t vec) const {
        if (!k8 && !v16) return x[elem];
        const int64_t M = mag[vec];
        if (M == 0) return 0;
        const int64_t q = k8 ? (int64_t)k8[elem] : (int64_t)v16[elem];
        // (2q + 1) M >= 0: the division by 2^b is a floor, i.e. a shift
        return (int64_t)(((i128)(2 * q + 1) * M) >> bits) - M;
    }
    // elements elem .. elem + 3 of vector vec (elem a multiple of 4)
    __device__ __forceinline__ void at4(size_t elem, size_t vec, int64_t (&e)[4]) const {
        if (!k8 && !v16) {
            const longlong2 *p = reinterpret_cast<const longlong2 *>(x + elem);
            const longlong2 a = p[0], c = p[1];
            e[0] = a.x; e[1] = a.y; e[2] = c.x; e[3] = c.y;
            return;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) e[i] = at(elem + i, vec);
    }
};

// kv_pack_vector (llama_int.c:1197-1218) for the rows' K and V at their
// positions: one warp per (row, kv head), reading the exact values k_rope_kv
// wrote into the exact cache.
__global__ void k_kv_pack(uint8_t *__restrict__ kq, uint16_t *__restrict__ vq, int64_t *__restrict__ kmag,
                          int64_t *__restrict__ vmag, const int64_t *__restrict__ kc, const int64_t *__restrict__ vc,
                          const int *__restrict__ pos_arr, const int *__restrict__ seq_arr, int R, int nkv, int hd,
                          int max_seq, int kbits, int vbits) {
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= R * nkv) return;
    const int r = gw / nkv, h = gw % nkv;
    const size_t vec = ((size_t)seq_arr[r] * max_seq + pos_arr[r]) * nkv + h;
    const size_t e0 = vec * hd;
    for (int which = 0; which < 2; which++) {
        const int64_t *src = (which ? vc : kc) + e0;
        const int b = which ? vbits : kbits;
        int64_t M = 0;
        for (int i = lane; i < hd; i += 32) {
            const int64_t x = src[i];
            const int64_t a = x < 0 ? (int64_t)(0 - (uint64_t)x) : x;   // wraps like -fwrapv
            if (a > M) M = a;
        }
        for (int m = 16; m >= 1; m >>= 1) M = max(M, (int64_t)__shfl_xor_sync(0xffffffffu, M, m));
        if (lane == 0) (which ? vmag : kmag)[vec] = M;
        const int64_t Q = (int64_t)1 << b;
        for (int i = lane; i < hd; i += 32) {
            int64_t q = 0;
            if (M != 0) {
                const i128 num = (i128)(int64_t)((uint64_t)src[i] + (uint64_t)M) * Q;
                i128 t = d_sdiv128_64(num, (int64_t)((uint64_t)M * 2));
                if (t < 0) t = 0;
                if (t >= (i128)Q) t = Q - 1;
                q = (int64_t)t;
            }
            if (which) vq[e0 + i] = (uint16_t)q;
            else kq[e0 + i] = (uint8_t)q;
        }
    }
}

// ---------------------------------------------------------------------------
// Phased exact attention (llama_int.c:1432-1529), parallel over (row, kv
// group, 64-position tile). Per row b (sequence seq[b], position pos[b]) and
// query head h the reference computes, in order:
//   s_t = fp_mul((int64)(sum_d (i128)q_h[d] k_t[d] >> 48), fp_inv_sqrt(hd))
//   m = max_t s_t;  e_t = fp_safe_exp(s_t - m);  S = sum_t e_t (int64, wrapping)
//   p_t = S > 0 ? fp_div(e_t, S) : e_t;  out_h[d] = sum_t fp_mul(p_t, v_t[d]) (int64)
// Every reduction here is exact and order-free: max, wrapping int64 sums.
// scratch: sc [R][nh][Tcap] scores/numerators, mx [R][nh], sm_ [R][nh] (u64).
#define ATT_TILE 64

// zero the outputs and sums, max = INT64_MIN
__global__ void k_attn_init(int64_t *__restrict__ out, int64_t *__restrict__ mx, uint64_t *__restrict__ sm_,
                            int R, int nh, int hd) {
    const int64_t n = (int64_t)R * nh * hd;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        out[e] = 0;
        if (e < (int64_t)R * nh) { mx[e] = INT64_MIN; sm_[e] = 0; }
    }
}

// phase 1: scores of one 64-position tile for the grp query heads of kv head g
// (keys from the exact cache, or unpacked from the packed one: kv)
__global__ void __launch_bounds__(256)
k_attn_scores(int64_t *__restrict__ sc, int64_t *__restrict__ mx, const int64_t *__restrict__ qkv,
              const KVView kv, const int *__restrict__ pos_arr, const int *__restrict__ seq_arr,
              int nh, int nkv, int hd, int max_seq, int Tcap,
              int64_t scale) {
    extern __shared__ __align__(16) int64_t smem[];
    const int tile = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int T = pos_arr[b] + 1, t0 = tile * ATT_TILE;
    if (t0 >= T) return;
    const int nt = min(ATT_TILE, T - t0);
    const int grp = nh / nkv, dim = nh * hd, kvd = nkv * hd, kld = hd + 1;
    // Exact int128 dots in 32-bit limbs (six mad.wide.s32 per MAC instead of a
    // 64 x 64 -> 128 product): q = a0 + a1 2^22 + a2 2^44 (a0, a1 unsigned
    // 22-bit, a2 signed), k = kh 2^32 + ks + 2^31 (kh = k >> 32, ks = low word
    // - 2^31, both signed 32-bit), so
    //   sum q k = sum_i 2^(22 i) (2^32 H_i + L_i) + 2^31 sum q   (mod 2^128)
    // with H_i = sum a_i kh, L_i = sum a_i ks; every term is < 2^53, so the
    // int64 sums are exact for hd <= 256.
    i128 *qsum = reinterpret_cast<i128 *>(smem);                        // [grp]
    int32_t *qa = reinterpret_cast<int32_t *>(qsum + grp);               // [3][grp * hd]
    int2 *kt = reinterpret_cast<int2 *>(smem + 2 * grp + (3 * grp * hd + 1) / 2);  // [ATT_TILE][hd + 1]
    const int64_t *q = qkv + (size_t)b * (dim + 2 * kvd) + (size_t)g * grp * hd;
    for (int e = threadIdx.x; e < grp * hd; e += blockDim.x) {
        const int64_t v = q[e];
        qa[e] = (int32_t)(v & 0x3FFFFF);
        qa[grp * hd + e] = (int32_t)((v >> 22) & 0x3FFFFF);
        qa[2 * grp * hd + e] = (int32_t)(v >> 44);
    }
    {   // sum q per head: one warp per head
        const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
        for (int hh = w; hh < grp; hh += blockDim.x >> 5) {
            i128 t = 0;
            for (int d = l; d < hd; d += 32) t += (i128)q[hh * hd + d];
            t = warp_sum_i128(t);
            if (l == 0) qsum[hh] = t;
        }
    }
    const size_t vb0 = ((size_t)seq_arr[b] * max_seq + t0) * nkv + g;   // vector of position t0, head g
    for (int e = threadIdx.x; e < nt * hd; e += blockDim.x) {
        const size_t vec = vb0 + (size_t)(e / hd) * nkv;
        const int64_t v = kv.at(vec * hd + e % hd, vec);
        kt[(e / hd) * kld + e % hd] = make_int2((int32_t)(v >> 32), (int32_t)((uint32_t)v ^ 0x80000000u));
    }
    __syncthreads();
    for (int e = threadIdx.x; e < grp * ATT_TILE; e += blockDim.x) {
        const int hh = e / ATT_TILE, tt = e % ATT_TILE;
        int64_t v = INT64_MIN;
        if (tt < nt) {
            const int32_t *a0 = qa + hh * hd, *a1 = a0 + grp * hd, *a2 = a1 + grp * hd;
            const int2 *kr = kt + tt * kld;
            int64_t h0 = 0, h1 = 0, h2 = 0, l0 = 0, l1 = 0, l2 = 0;
#pragma unroll 4
            for (int dd = 0; dd < hd; dd++) {
                const int2 kv = kr[dd];
                const int32_t x0 = a0[dd], x1 = a1[dd], x2 = a2[dd];
                madw(h0, x0, kv.x); madw(h1, x1, kv.x); madw(h2, x2, kv.x);
                madw(l0, x0, kv.y); madw(l1, x1, kv.y); madw(l2, x2, kv.y);
            }
            const u128 dot = ((u128)(i128)h0 << 32) + ((u128)(i128)h1 << 54) + ((u128)(i128)h2 << 76) +
                             (u128)(i128)l0 + ((u128)(i128)l1 << 22) + ((u128)(i128)l2 << 44) +
                             ((u128)qsum[hh] << 31);
            v = d_mul((int64_t)((i128)dot >> 48), scale);
            sc[((size_t)b * nh + g * grp + hh) * Tcap + t0 + tt] = v;
        }
        // tile max per head: the 64 tt of one head are two consecutive warps
        for (int m = 16; m >= 1; m >>= 1) v = max(v, (int64_t)__shfl_xor_sync(0xffffffffu, v, m));
        if ((threadIdx.x & 31) == 0 && v != INT64_MIN)
            atomicMax((long long *)&mx[(size_t)b * nh + g * grp + hh], (long long)v);
    }
}

// One m16n8k32 integer MMA, D += A B, A (16 x 32, row) and B (32 x 8, col)
// bytes unsigned or signed (AS, BS).
template <bool AS, bool BS>
__device__ __forceinline__ void mma_s32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
#define IQ_MMA_S32(TA, TB)                                                                               \
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32." TA "." TB ".s32 "                             \
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"                                 \
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])                                        \
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1))
    if (AS && BS) IQ_MMA_S32("s8", "s8");
    else if (AS) IQ_MMA_S32("s8", "u8");
    else if (BS) IQ_MMA_S32("u8", "s8");
    else IQ_MMA_S32("u8", "u8");
#undef IQ_MMA_S32
}

// Byte planes of four consecutive int64 (two's complement, little endian):
// o[i] holds byte i of e[0], e[1], e[2], e[3] in its bytes 0..3.
__device__ __forceinline__ void byte_planes4(const int64_t (&e)[4], uint32_t (&o)[8]) {
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const uint32_t w0 = (uint32_t)((uint64_t)e[0] >> (32 * half)), w1 = (uint32_t)((uint64_t)e[1] >> (32 * half));
        const uint32_t w2 = (uint32_t)((uint64_t)e[2] >> (32 * half)), w3 = (uint32_t)((uint64_t)e[3] >> (32 * half));
        const uint32_t x01 = __byte_perm(w0, w1, 0x5140), x23 = __byte_perm(w2, w3, 0x5140);
        const uint32_t y01 = __byte_perm(w0, w1, 0x7362), y23 = __byte_perm(w2, w3, 0x7362);
        o[4 * half + 0] = __byte_perm(x01, x23, 0x5410);
        o[4 * half + 1] = __byte_perm(x01, x23, 0x7632);
        o[4 * half + 2] = __byte_perm(y01, y23, 0x5410);
        o[4 * half + 3] = __byte_perm(y01, y23, 0x7632);
    }
}

// Phase 1 on the int8 tensor cores: the same scores as k_attn_scores.
// Each int64 is 7 unsigned bytes and a signed top byte, x = sum_i x_i 2^(8i),
// so q . k = sum_(i,j) 2^(8(i+j)) sum_d q_i k_j. The (7, 7) pair only adds
// multiples of 2^112 and is dropped: (q . k >> 48) mod 2^64, the value the
// reference keeps, depends on q . k mod 2^112 alone. The pairs of each
// diagonal s = i + j accumulate into one s32 (at most 8 pairs x hd terms of
// |byte product| < 2^16: < 2^27 for hd <= 256) and the 14 diagonals are
// recombined in 128 bits.
// A warp takes 16-position tiles (MMA rows: keys) against 8 query heads (MMA
// columns; a kv group of more than 8 heads takes several passes, missing heads
// read as zero). K and Q fragments come straight from global memory into
// registers and are transposed to byte planes with byte permutes; the raw K of
// the warp's next (tile, 32-wide d step) is loaded before the MMAs of the
// current one, so the loads overlap the tensor work. 8 warps x ATT_TC_TPW
// tiles = ATT_TC_POS positions per CTA; no shared memory.
#define ATT_TC_TPW 2
#define ATT_TC_POS (128 * ATT_TC_TPW)
#ifndef IQ_SC_MINB
#define IQ_SC_MINB 1
#endif
__global__ void __launch_bounds__(256, IQ_SC_MINB)
k_attn_scores_tc(int64_t *__restrict__ sc, int64_t *__restrict__ mx, const int64_t *__restrict__ qkv,
                 const KVView kv, const int *__restrict__ pos_arr, const int *__restrict__ seq_arr,
                 int nh, int nkv, int hd, int max_seq, int Tcap, int64_t scale) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
    const int g = blockIdx.y, b = blockIdx.z;
    const int T = pos_arr[b] + 1;
    const int tbase = blockIdx.x * ATT_TC_POS + warp * 16;   // tile k of this warp: tbase + 128 k
    if (tbase >= T) return;   // warp-uniform; the kernel has no CTA-wide barrier
    const int ntile = min(ATT_TC_TPW, (T - tbase + 127) / 128);
    const int grp = nh / nkv, dim = nh * hd, kvd = nkv * hd, KS = hd / 32;
    const int64_t *qb = qkv + (size_t)b * (dim + 2 * kvd) + (size_t)g * grp * hd;
    const size_t vbase = (size_t)seq_arr[b] * max_seq;
    for (int n0 = 0; n0 < grp; n0 += 8) {
        const int hq = n0 + gq;
        const int U = ntile * KS;
        int64_t raw[4][4];
        auto load_k = [&](int u) {   // a0..a3 of unit u: rows gq, gq + 8 x columns tq*4, tq*4 + 16
            const int t0 = tbase + 128 * (u / KS), ks = (u % KS) * 32;
#pragma unroll
            for (int f = 0; f < 4; f++) {
                const int row = t0 + gq + ((f & 1) ? 8 : 0), d = ks + tq * 4 + (f >> 1) * 16;
                raw[f][0] = raw[f][1] = raw[f][2] = raw[f][3] = 0;
                if (row < T) {
                    const size_t vec = (vbase + row) * nkv + g;
                    kv.at4(vec * hd + d, vec, raw[f]);
                }
            }
        };
        load_k(0);
        int acc[14][4];
        for (int u = 0; u < U; u++) {
            const int ks = (u % KS) * 32, t0 = tbase + 128 * (u / KS);
            if (ks == 0) {
#pragma unroll
                for (int s = 0; s < 14; s++) acc[s][0] = acc[s][1] = acc[s][2] = acc[s][3] = 0;
            }
            uint32_t A[4][8], B[2][8];
#pragma unroll
            for (int f = 0; f < 4; f++) byte_planes4(raw[f], A[f]);
            if (u + 1 < U) load_k(u + 1);
#pragma unroll
            for (int f = 0; f < 2; f++) {   // b0, b1: rows (d) tq*4, tq*4 + 16 x column (head) hq
                int64_t e[4] = {0, 0, 0, 0};
                if (hq < grp) {
                    const longlong2 *p =
                        reinterpret_cast<const longlong2 *>(qb + (size_t)hq * hd + ks + tq * 4 + f * 16);
                    const longlong2 x = p[0], y = p[1];
                    e[0] = x.x; e[1] = x.y; e[2] = y.x; e[3] = y.y;
                }
                byte_planes4(e, B[f]);
            }
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (i + j > 13) continue;
                    if (i == 7) mma_s32<true, false>(acc[i + j], A[0][i], A[1][i], A[2][i], A[3][i], B[0][j], B[1][j]);
                    else if (j == 7) mma_s32<false, true>(acc[i + j], A[0][i], A[1][i], A[2][i], A[3][i], B[0][j], B[1][j]);
                    else mma_s32<false, false>(acc[i + j], A[0][i], A[1][i], A[2][i], A[3][i], B[0][j], B[1][j]);
                }
            if (ks + 32 < hd) continue;
            // c0, c1: position t0 + gq, heads n0 + 2 tq + {0, 1}; c2, c3: position t0 + gq + 8
            int64_t hmax[2] = {INT64_MIN, INT64_MIN};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint64_t G0 = 0, G1 = 0, G2 = 0;   // diagonals 0-4, 5-9, 10-13 (|G| < 2^61)
#pragma unroll
                for (int s = 0; s < 5; s++) G0 += (uint64_t)(int64_t)acc[s][c] << (8 * s);
#pragma unroll
                for (int s = 5; s < 10; s++) G1 += (uint64_t)(int64_t)acc[s][c] << (8 * (s - 5));
#pragma unroll
                for (int s = 10; s < 14; s++) G2 += (uint64_t)(int64_t)acc[s][c] << (8 * (s - 10));
                const u128 dot = (u128)(i128)(int64_t)G0 + ((u128)(i128)(int64_t)G1 << 40) +
                                 ((u128)(i128)(int64_t)G2 << 80);
                const int pos = t0 + gq + (c < 2 ? 0 : 8), head = n0 + 2 * tq + (c & 1);
                if (pos < T && head < grp) {
                    const int64_t v = d_mul((int64_t)(uint64_t)(dot >> 48), scale);
                    sc[((size_t)b * nh + g * grp + head) * Tcap + pos] = v;
                    hmax[c & 1] = max(hmax[c & 1], v);
                }
            }
#pragma unroll
            for (int k = 0; k < 2; k++) {
                int64_t v = hmax[k];
                for (int m = 4; m <= 16; m <<= 1) v = max(v, (int64_t)__shfl_xor_sync(0xffffffffu, v, m));
                const int head = n0 + 2 * tq + k;
                if (gq == 0 && head < grp && v != INT64_MIN)
                    atomicMax((long long *)&mx[(size_t)b * nh + g * grp + head], (long long)v);
            }
        }
    }
}

// shared memory of k_attn_scores: q sums, q limbs, key tile of int2 (int64 units)
__host__ __device__ constexpr size_t att_scores_smem(int grp, int hd) {
    return ((size_t)2 * grp + (3 * (size_t)grp * hd + 1) / 2 + (size_t)ATT_TILE * (hd + 1)) * 8;
}

// phase 2: e_t = fp_safe_exp(s_t - max) in place, S = wrapping int64 sum
__global__ void __launch_bounds__(256)
k_attn_exp(int64_t *__restrict__ sc, const int64_t *__restrict__ mx, uint64_t *__restrict__ sm_,
           const int *__restrict__ pos_arr, int nh, int Tcap) {
    const int h = blockIdx.y, b = blockIdx.z;
    const int T = pos_arr[b] + 1, t = blockIdx.x * blockDim.x + threadIdx.x;
    if (blockIdx.x * blockDim.x >= T) return;
    const size_t base = ((size_t)b * nh + h) * Tcap;
    const int64_t m = mx[(size_t)b * nh + h];
    uint64_t e = 0;
    if (t < T) {
        int64_t v = d_safe_exp((int64_t)((uint64_t)sc[base + t] - (uint64_t)m));
        sc[base + t] = v;
        e = (uint64_t)v;
    }
    for (int k = 16; k >= 1; k >>= 1) e += __shfl_xor_sync(0xffffffffu, e, k);
    if ((threadIdx.x & 31) == 0) atomicAdd((unsigned long long *)&sm_[(size_t)b * nh + h], (unsigned long long)e);
}

// phase 3: p_t = fp_div(e_t, S) (if S > 0) for the tile, then int64 partial
// sums of fp_mul(p_t, v_t[d]) added atomically into out (wrapping, exact).
//
// Limb form of the per-term floor (SPT > 0): with 0 <= p < 2^49 (p is a
// probability, at most 2^48) and R_t = (p_t v_t) mod 2^48 >= 0,
//   sum_t fp_mul(p_t, v_t) = (sum_t p_t v_t - sum_t R_t) / 2^48   exactly,
// since every p v - R is 2^48 floor(p v / 2^48). The exact sum of products is
// taken in four 32 x 32 -> 64 partial sums, p = p0 + 2^25 p1 (p0 < 2^25,
// p1 < 2^24), v = vl + 2^32 vh (vl unsigned, vh signed):
//   A = sum p0 vl, B = sum p1 vl, C = sum p0 vh, D = sum p1 vh,
//   sum p v = A + 2^25 B + 2^32 C + 2^57 D,
// all int64-exact over one 64-position tile; R_t is the low 48 bits of the
// 64-bit product. Thread slots: with grp*hd >= 256 a thread owns one d and
// SPT heads (d = tid % hd, heads tid / hd + k * 256 / hd), sharing each v load
// across them; with fewer slots, 256 / (grp*hd) position groups split the tile
// and each adds its own partial sum. A tile holding a p outside [0, 2^49)
// (never produced by fp_div of a softmax numerator) takes the direct
// fp_mul loop (SPT == 0 is that loop for every tile).
template <int SPT>
__global__ void __launch_bounds__(256)
k_attn_pv(int64_t *__restrict__ out, const int64_t *__restrict__ sc, const uint64_t *__restrict__ sm_,
          const KVView kv, const int *__restrict__ pos_arr, const int *__restrict__ seq_arr,
          int nh, int nkv, int hd, int max_seq, int Tcap) {
    extern __shared__ __align__(16) int64_t smem[];
    const int tile = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int T = pos_arr[b] + 1, t0 = tile * ATT_TILE;
    if (t0 >= T) return;
    const int nt = min(ATT_TILE, T - t0);
    const int grp = nh / nkv, dim = nh * hd;
    int4 *ps = reinterpret_cast<int4 *>(smem);                 // [grp][ATT_TILE] {p0, p1, lo32(p), p >> 32}
    int64_t *vt = smem + 2 * grp * ATT_TILE;                  // [ATT_TILE][hd]
    int bad = 0;
    for (int e = threadIdx.x; e < grp * ATT_TILE; e += blockDim.x) {
        const int hh = e / ATT_TILE, tt = e % ATT_TILE;
        int64_t p = 0;
        if (tt < nt) {
            const int h = g * grp + hh;
            p = sc[((size_t)b * nh + h) * Tcap + t0 + tt];
            const int64_t S = (int64_t)sm_[(size_t)b * nh + h];
            if (S > 0) p = d_div(p, S);
        }
        bad |= (uint64_t)p >= (1ull << 49);
        ps[e] = make_int4((int)(p & 0x1FFFFFF), (int)((uint64_t)p >> 25), (int)(uint32_t)p, (int)(p >> 32));
    }
    const size_t vb0 = ((size_t)seq_arr[b] * max_seq + t0) * nkv + g;
    for (int e = threadIdx.x; e < nt * hd; e += blockDim.x) {
        const size_t vec = vb0 + (size_t)(e / hd) * nkv;
        vt[e] = kv.at(vec * hd + e % hd, vec);
    }
    if (SPT == 0 || __syncthreads_or(bad)) {
        __syncthreads();
        for (int e = threadIdx.x; e < grp * hd; e += blockDim.x) {
            const int hh = e / hd, dd = e % hd;
            const int4 *pp = ps + hh * ATT_TILE;
            uint64_t acc = 0;
            for (int tt = 0; tt < nt; tt++) {
                const int64_t p = (int64_t)(uint32_t)pp[tt].z | ((int64_t)pp[tt].w << 32);
                acc += (uint64_t)d_mul(p, vt[tt * hd + dd]);
            }
            atomicAdd((unsigned long long *)&out[(size_t)b * dim + (size_t)(g * grp + hh) * hd + dd],
                      (unsigned long long)acc);
        }
        return;
    }
    if constexpr (SPT > 0) {
        const int nslots = grp * hd, tid = threadIdx.x;
        const int pg_n = nslots >= 256 ? 1 : 256 / nslots;            // position groups
        const int slot = nslots >= 256 ? tid : tid % nslots, pg = nslots >= 256 ? 0 : tid / nslots;
        const int dd = slot % hd, h0 = slot / hd, hstep = 256 / hd;
        uint64_t A[SPT], B[SPT], Rs[SPT];
        int64_t C[SPT], D[SPT];
#pragma unroll
        for (int k = 0; k < SPT; k++) { A[k] = B[k] = Rs[k] = 0; C[k] = D[k] = 0; }
        const int2 *vcol = reinterpret_cast<const int2 *>(vt) + dd;
#pragma unroll 2
        for (int tt = pg; tt < nt; tt += pg_n) {
            const int2 v = vcol[tt * hd];
#pragma unroll
            for (int k = 0; k < SPT; k++) {
                const int4 p = ps[(h0 + k * hstep) * ATT_TILE + tt];
                asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(A[k]) : "r"(p.x), "r"(v.x));
                asm("mad.wide.u32 %0, %1, %2, %0;" : "+l"(B[k]) : "r"(p.y), "r"(v.x));
                asm("mad.wide.s32 %0, %1, %2, %0;" : "+l"(C[k]) : "r"(p.x), "r"(v.y));
                asm("mad.wide.s32 %0, %1, %2, %0;" : "+l"(D[k]) : "r"(p.y), "r"(v.y));
                const uint64_t lo = ((uint64_t)(uint32_t)p.w << 32 | (uint32_t)p.z) *
                                    ((uint64_t)(uint32_t)v.y << 32 | (uint32_t)v.x);
                Rs[k] += lo & 0xFFFFFFFFFFFFull;
            }
        }
#pragma unroll
        for (int k = 0; k < SPT; k++) {
            const u128 sum = (u128)A[k] + ((u128)B[k] << 25) + ((u128)(i128)C[k] << 32) +
                             ((u128)(i128)D[k] << 57) - (u128)Rs[k];
            const uint64_t part = (uint64_t)(sum >> 48);
            atomicAdd((unsigned long long *)&out[(size_t)b * dim + (size_t)(g * grp + h0 + k * hstep) * hd + dd],
                      (unsigned long long)part);
        }
    }
}

// Phase 3 with the products on the int8 tensor cores. Same result as
// k_attn_pv: per (row, head, d), sum_t fp_mul(p_t, v_t[d]) =
// (sum_t p_t v_t - sum_t R_t) / 2^48 with R_t = (p_t v_t) mod 2^48, over any set
// of positions. The exact sum of products is taken in byte planes (p: 7
// unsigned bytes, as 0 <= p < 2^49; v: 7 unsigned and a signed top byte) with
// one m16n8k32 MMA per plane pair (A = values, 16 d x 32 positions; B =
// probabilities, 32 positions x 8 heads), the pairs of each diagonal summed in
// s32; every pair has i + j <= 13, all needed mod 2^112. R_t is taken on the
// CUDA cores from 32-bit pieces: w = lo(p) lo(v) (64-bit) and the low 16 bits
// of hi(w) + lo(p) hi(v) + hi(p) lo(v) (the bits 32..47). Both parts of each
// (head, d) meet in shared memory as four int64 partial sums weighted 2^0,
// 2^32, 2^64, 2^96 (each far from overflow), then the exact shift by 48.
// A CTA takes PV_CH positions of one (row, kv group) in 64-position sub-tiles;
// the host launches it when (hd / 16) x ceil(grp / 8) output blocks divide the
// 8 warps and att_pv_spt(grp, hd) > 0.
#define PV_CH 256
#ifndef IQ_PV_XMMA
#define IQ_PV_XMMA 0
#endif
#ifndef IQ_PV_XR
#define IQ_PV_XR 0
#endif
#ifndef IQ_PV_MINB
#define IQ_PV_MINB 2
#endif
template <int HB>
__global__ void __launch_bounds__(256, IQ_PV_MINB)
k_attn_pv_tc(int64_t *__restrict__ out, const int64_t *__restrict__ sc, const uint64_t *__restrict__ sm_,
             const KVView kv, const int *__restrict__ pos_arr, const int *__restrict__ seq_arr,
             int nh, int nkv, int hd, int max_seq, int Tcap) {
    extern __shared__ __align__(16) int64_t smem[];
    const int g = blockIdx.y, b = blockIdx.z, T = pos_arr[b] + 1, c0 = blockIdx.x * PV_CH;
    if (c0 >= T) return;
    const int nt = min(PV_CH, T - c0);
    const int grp = nh / nkv, dim = nh * hd, nslots = grp * hd, vld = hd + 2, tid = threadIdx.x;
    int64_t *ps = smem;                                        // [grp][PV_CH] probabilities
    int64_t *vt = ps + (size_t)grp * PV_CH;                    // [64][hd + 1] values of one sub-tile
    long long *gacc = reinterpret_cast<long long *>(vt + 64 * vld);   // [4][nslots]
    for (int e = tid; e < 4 * nslots; e += 256) gacc[e] = 0;
    int bad = 0;
    for (int e = tid; e < grp * PV_CH; e += 256) {
        const int hh = e / PV_CH, tt = e % PV_CH;
        int64_t p = 0;
        if (tt < nt) {
            const int h = g * grp + hh;
            p = sc[((size_t)b * nh + h) * Tcap + c0 + tt];
            const int64_t S = (int64_t)sm_[(size_t)b * nh + h];
            if (S > 0) p = d_div(p, S);
        }
        bad |= (uint64_t)p >= (1ull << 49);
        ps[e] = p;
    }
    bad = __syncthreads_or(bad);
    const size_t vb0 = ((size_t)seq_arr[b] * max_seq + c0) * nkv + g;   // vector of position c0, head g
    auto stage_v = [&](int st0, int snt) {
        __syncthreads();   // the previous sub-tile is consumed
        for (int e = tid * 4; e < 64 * hd; e += 1024) {
            const int t = e / hd, d = e % hd;
            int64_t v4[4] = {0, 0, 0, 0};
            if (t < snt) {
                const size_t vec = vb0 + (size_t)(st0 + t) * nkv;
                kv.at4(vec * hd + d, vec, v4);
            }
            longlong2 *dst = reinterpret_cast<longlong2 *>(vt + t * vld + d);
            dst[0] = make_longlong2(v4[0], v4[1]);
            dst[1] = make_longlong2(v4[2], v4[3]);
        }
        __syncthreads();
    };
    if (bad) {   // a probability outside [0, 2^49): the direct per-term loop for this chunk
        for (int st0 = 0; st0 < nt; st0 += 64) {
            const int snt = min(64, nt - st0);
            stage_v(st0, snt);
            for (int e = tid; e < nslots; e += 256) {
                const int hh = e / hd, dd = e % hd;
                uint64_t acc = 0;
                for (int tt = 0; tt < snt; tt++) acc += (uint64_t)d_mul(ps[hh * PV_CH + st0 + tt], vt[tt * vld + dd]);
                atomicAdd((unsigned long long *)&out[(size_t)b * dim + (size_t)g * nslots + e], (unsigned long long)acc);
            }
        }
        return;
    }
    const int warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
    const int ndt = hd / 16, OB = ndt * ((grp + 7) / 8), WB = 8 / OB;
    const int ob = warp % OB, wsub = warp / OB, d0 = (ob % ndt) * 16, n0 = (ob / ndt) * 8;
    // R slots: HB heads x 2 adjacent d per thread, position pairs split over pg_n groups
    const int nthr = nslots / (2 * HB), pg_n = 256 / nthr, r = tid % nthr, pg = tid / nthr;
    const int dd = (r % (hd / 2)) * 2, h0 = (r / (hd / 2)) * HB;
    int acc[14][4];
#pragma unroll
    for (int s = 0; s < 14; s++) acc[s][0] = acc[s][1] = acc[s][2] = acc[s][3] = 0;
    uint32_t Rl[HB][2], Rh[HB][2];   // sum_t R_t of each slot as (low, high) 32-bit words
#pragma unroll
    for (int k = 0; k < HB; k++) Rl[k][0] = Rl[k][1] = Rh[k][0] = Rh[k][1] = 0;
    const int hq = n0 + gq;
    for (int st0 = 0; st0 < nt; st0 += 64) {
        const int snt = min(64, nt - st0);
        stage_v(st0, snt);
        for (int ks = wsub; ks < 2 && ks * 32 < snt && !IQ_PV_XMMA; ks += WB) {
            uint32_t A[4][8], B[2][8];
#pragma unroll
            for (int f = 0; f < 4; f++) {   // a0..a3: rows (d) d0 + gq (+8) x columns (t) tq*4 (+16)
                const int d = d0 + gq + ((f & 1) ? 8 : 0), t = ks * 32 + tq * 4 + (f >> 1) * 16;
                const int64_t e[4] = {vt[t * vld + d], vt[(t + 1) * vld + d], vt[(t + 2) * vld + d],
                                      vt[(t + 3) * vld + d]};
                byte_planes4(e, A[f]);
            }
#pragma unroll
            for (int f = 0; f < 2; f++) {   // b0, b1: rows (t) tq*4 (+16) x column (head) hq
                int64_t e[4] = {0, 0, 0, 0};
                if (hq < grp) {
                    const longlong2 *p = reinterpret_cast<const longlong2 *>(ps + (size_t)hq * PV_CH + st0 + ks * 32 +
                                                                             tq * 4 + f * 16);
                    const longlong2 x = p[0], y = p[1];
                    e[0] = x.x; e[1] = x.y; e[2] = y.x; e[3] = y.y;
                }
                byte_planes4(e, B[f]);
            }
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 7; j++) {
                    if (i == 7) mma_s32<true, false>(acc[i + j], A[0][i], A[1][i], A[2][i], A[3][i], B[0][j], B[1][j]);
                    else mma_s32<false, false>(acc[i + j], A[0][i], A[1][i], A[2][i], A[3][i], B[0][j], B[1][j]);
                }
        }
        // R_t for this thread's (head, d) slots, two positions per step
        const int64_t *prow = ps + (size_t)h0 * PV_CH + st0;
#pragma unroll 2
        for (int tt = 2 * pg; tt < snt && !IQ_PV_XR; tt += 2 * pg_n) {
            const longlong2 va = *reinterpret_cast<const longlong2 *>(vt + tt * vld + dd);
            const longlong2 vb = *reinterpret_cast<const longlong2 *>(vt + (tt + 1) * vld + dd);
            const uint64_t v[2][2] = {{(uint64_t)va.x, (uint64_t)va.y}, {(uint64_t)vb.x, (uint64_t)vb.y}};
#pragma unroll
            for (int k = 0; k < HB; k++) {
                const longlong2 pp = *reinterpret_cast<const longlong2 *>(prow + k * PV_CH + tt);
                const uint64_t p2[2] = {(uint64_t)pp.x, (uint64_t)pp.y};
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const uint32_t plo = (uint32_t)p2[u], phi = (uint32_t)(p2[u] >> 32);
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        // R = lo(p) lo(v) mod 2^32 + 2^32 ((hi(lo(p) lo(v)) + lo(p) hi(v) + hi(p) lo(v)) mod 2^16)
                        const uint32_t vlo = (uint32_t)v[u][e], vhi = (uint32_t)(v[u][e] >> 32);
                        asm("{\n\t.reg .u32 wh, t;\n\t"
                            "mul.hi.u32 wh, %2, %3;\n\t"
                            "mad.lo.u32 t, %2, %4, wh;\n\t"
                            "mad.lo.u32 t, %5, %3, t;\n\t"
                            "and.b32 t, t, 65535;\n\t"
                            "mad.lo.cc.u32 %0, %2, %3, %0;\n\t"
                            "addc.u32 %1, %1, t;\n\t}"
                            : "+r"(Rl[k][e]), "+r"(Rh[k][e])
                            : "r"(plo), "r"(vlo), "r"(vhi), "r"(phi));
                    }
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < HB; k++)
#pragma unroll
        for (int e = 0; e < 2; e++)
            atomicAdd((unsigned long long *)&gacc[(h0 + k) * hd + dd + e],
                      (unsigned long long)(0 - (((uint64_t)Rh[k][e] << 32) | Rl[k][e])));
    // c0, c1: d = d0 + gq, heads n0 + 2 tq + {0, 1}; c2, c3: d + 8
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int head = n0 + 2 * tq + (c & 1), d = d0 + gq + (c < 2 ? 0 : 8);
        if (head >= grp) continue;
        uint64_t G[4] = {0, 0, 0, 0};
#pragma unroll
        for (int s = 0; s < 14; s++) G[s >> 2] += (uint64_t)(int64_t)acc[s][c] << (8 * (s & 3));
        const int sl = head * hd + d;
#pragma unroll
        for (int q = 0; q < 4; q++)
            if (G[q]) atomicAdd((unsigned long long *)&gacc[q * nslots + sl], (unsigned long long)G[q]);
    }
    __syncthreads();
    for (int e = tid; e < nslots; e += 256) {
        const u128 X = (u128)(i128)gacc[e] + ((u128)(i128)gacc[nslots + e] << 32) +
                       ((u128)(i128)gacc[2 * nslots + e] << 64) + ((u128)(i128)gacc[3 * nslots + e] << 96);
        atomicAdd((unsigned long long *)&out[(size_t)b * dim + (size_t)g * nslots + e], (unsigned long long)(X >> 48));
    }
}

// shared memory of k_attn_pv_tc, and whether (grp, hd) can take it
__host__ __device__ constexpr size_t att_pv_tc_smem(int grp, int hd) {
    return ((size_t)grp * PV_CH + (size_t)64 * (hd + 2) + (size_t)4 * grp * hd) * 8;
}
// heads per thread of the R part (0: the kernel does not apply): the MMA output
// blocks (hd / 16) x ceil(grp / 8) divide the 8 warps and the R threads
// grp * hd / (2 HB) divide 256
__host__ __device__ constexpr int att_pv_tc_hb(int grp, int hd) {
    return (hd % 32 != 0 || hd / 16 * ((grp + 7) / 8) > 8 || 8 % (hd / 16 * ((grp + 7) / 8)) != 0) ? 0
           : (grp >= 2 && grp % 2 == 0 && 256 % (grp * hd / 4) == 0) ? 2
           : (256 % (grp * hd / 2) == 0 && grp * hd / 2 <= 256) ? 1 : 0;
}

// the k_attn_pv instance for (grp, hd): SPT = grp*hd / 256 slots per thread
// when hd divides 256 and the slots fill the CTA evenly, else 0 (direct loop)
__host__ __device__ constexpr int att_pv_spt(int grp, int hd) {
    return (hd <= 0 || 256 % hd) ? 0
           : (grp * hd >= 256) ? ((grp * hd) % 256 == 0 && grp * hd / 256 <= 8 && ((grp * hd / 256) & (grp * hd / 256 - 1)) == 0
                                      ? grp * hd / 256 : 0)
           : (256 % (grp * hd) == 0 ? 1 : 0);
}
__host__ __device__ constexpr size_t att_pv_smem(int grp, int hd) {
    return ((size_t)2 * grp * ATT_TILE + (size_t)ATT_TILE * hd) * 8;
}

// SwiGLU: out[i] = fp_mul(fp_silu(gate[i]), up[i]) with gu = [gate | up] (llama_int.c:1549-1552)
__global__ void k_swiglu(int64_t *__restrict__ out, const int64_t *__restrict__ gu, int inter, int rows) {
    const int64_t n = (int64_t)inter * rows;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = e / inter, i = e % inter;
        const int64_t *row = gu + r * 2 * inter;
        out[e] = d_mul(d_silu(row[i]), row[inter + i]);
    }
}

// argmax, first maximum (strict >, llama_int.c:2888-2893), one CTA per row;
// also advances the decode state: next token -> tokens[b], pos[b] += 1, and
// records it in hist[b*hist_stride + pos+1] when hist != nullptr.
__global__ void k_argmax(int *__restrict__ result, const int64_t *__restrict__ logits, int vocab,
                         int *__restrict__ tokens, int *__restrict__ pos_arr, int *__restrict__ hist,
                         int hist_stride) {
    __shared__ int64_t bv[32];
    __shared__ int bi[32];
    const int b = blockIdx.x;
    const int64_t *lg = logits + (size_t)b * vocab;
    int64_t best = INT64_MIN;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        int64_t v = lg[i];
        if (v > best) { best = v; idx = i; }
    }
    for (int m = 16; m >= 1; m >>= 1) {
        int64_t ov = __shfl_xor_sync(0xffffffffu, best, m);
        int oi = __shfl_xor_sync(0xffffffffu, idx, m);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { bv[w] = best; bi[w] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); k++)
            if (bv[k] > best || (bv[k] == best && bi[k] < idx)) { best = bv[k]; idx = bi[k]; }
        // warp 0's value already folded in by the shuffle; recheck entry 0
        if (bv[0] > best || (bv[0] == best && bi[0] < idx)) { best = bv[0]; idx = bi[0]; }
        result[b] = idx;
        if (tokens) tokens[b] = idx;
        if (pos_arr) {
            int p = pos_arr[b] + 1;
            if (hist) hist[(size_t)b * hist_stride + p] = idx;
            pos_arr[b] = p;
        }
    }
}

// Tensor-parallel decode: the first maximum of this rank's logit rows
// [row][v_l] (columns v_lo .. v_lo + v_l - 1 of the vocabulary) as a
// (value, global index) pair per row, one CTA per row. The pairs of all ranks
// are then all-gathered (16 bytes per row and rank instead of the logits).
__global__ void k_argmax_local(int64_t *__restrict__ pairs, const int64_t *__restrict__ logits, int v_l, int v_lo) {
    __shared__ int64_t bv[32];
    __shared__ int bi[32];
    const int b = blockIdx.x;
    const int64_t *lg = logits + (size_t)b * v_l;
    int64_t best = INT64_MIN;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < v_l; i += blockDim.x) {
        const int64_t v = lg[i];
        if (v > best) { best = v; idx = i; }
    }
    for (int m = 16; m >= 1; m >>= 1) {
        const int64_t ov = __shfl_xor_sync(0xffffffffu, best, m);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, m);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { bv[w] = best; bi[w] = idx; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 0; k < (int)(blockDim.x >> 5); k++)
            if (bv[k] > best || (bv[k] == best && bi[k] < idx)) { best = bv[k]; idx = bi[k]; }
        pairs[2 * b] = best;
        pairs[2 * b + 1] = (int64_t)v_lo + idx;
    }
}

// The global first maximum from the gathered pairs g [P][B][2] (rank p holds
// the lower vocabulary block when p is lower, so among equal values the lowest
// index wins, llama_int.c:2888-2893), then the decode-state update of k_argmax.
__global__ void k_argmax_pairs(int *__restrict__ result, const int64_t *__restrict__ g, int P, int B,
                               int *__restrict__ tokens, int *__restrict__ pos_arr, int *__restrict__ hist,
                               int hist_stride) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int64_t best = INT64_MIN, idx = INT64_MAX;
    for (int p = 0; p < P; p++) {
        const int64_t v = g[((size_t)p * B + b) * 2], i = g[((size_t)p * B + b) * 2 + 1];
        if (v > best || (v == best && i < idx)) { best = v; idx = i; }
    }
    result[b] = (int)idx;
    if (tokens) tokens[b] = (int)idx;
    if (pos_arr) {
        const int np1 = pos_arr[b] + 1;
        if (hist) hist[(size_t)b * hist_stride + np1] = (int)idx;
        pos_arr[b] = np1;
    }
}

// ---------------------------------------------------------------- sampling

// Sampling parameters and generator state of one sequence (sample_params_t,
// llama_int.c:2936-2941; the xoroshiro128+ state of rng_state_t).
struct SampleState {
    int64_t temperature;  // Q16.48; below 0.01 (FP_ONE / 100) the argmax is taken
    int64_t top_p;        // Q16.48; 0 or >= FP_ONE: off
    int top_k, pad;       // 0 or >= vocab: off
    uint64_t s0, s1;      // generator state, advanced once per sampled token
};

#define IQ_SAMPLE_THREADS 1024

// First maximum of v[0..n) (strict >, lowest index among equals) over the CTA.
__device__ int cta_argmax(const int64_t *v, int n) {
    __shared__ int64_t bv[32];
    __shared__ int bi[32];
    int64_t best = INT64_MIN;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        if (v[i] > best) { best = v[i]; idx = i; }
    for (int m = 16; m >= 1; m >>= 1) {
        const int64_t ov = __shfl_xor_sync(0xffffffffu, best, m);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, m);
        if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) { bv[threadIdx.x >> 5] = best; bi[threadIdx.x >> 5] = idx; }
    __syncthreads();
    for (int k = 0; k < (int)(blockDim.x >> 5); k++)
        if (bv[k] > best || (bv[k] == best && bi[k] < idx)) { best = bv[k]; idx = bi[k]; }
    __syncthreads();
    return idx;
}

// CTA-wide exclusive prefix sum of one uint64 per thread (thread order).
__device__ uint64_t cta_exclusive_scan(uint64_t v, uint64_t *total) {
    __shared__ uint64_t ws[32];
    const int l = threadIdx.x & 31, w = threadIdx.x >> 5;
    uint64_t x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += y;
    }
    __syncthreads();
    if (l == 31) ws[w] = x;
    __syncthreads();
    uint64_t base = 0, all = 0;
    for (int k = 0; k < (int)(blockDim.x >> 5); k++) {
        if (k < w) base += ws[k];
        all += ws[k];
    }
    __syncthreads();
    if (total) *total = all;
    return base + x - v;
}

// The k-th largest of v[0..n) (radix selection on the order-preserving
// unsigned image of the int64 values, one byte per pass).
__device__ int64_t cta_kth_largest(const int64_t *v, int n, int k) {
    __shared__ unsigned int hist[256];
    uint64_t prefix = 0;
    unsigned int need = (unsigned int)k;
    for (int d = 7; d >= 0; d--) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint64_t u = (uint64_t)v[i] ^ 0x8000000000000000ull;
            if (d == 7 || (u >> (8 * (d + 1))) == prefix) atomicAdd(&hist[(u >> (8 * d)) & 0xFF], 1u);
        }
        __syncthreads();
        unsigned int cum = 0;
        int b = 255;
        for (; b > 0; b--) {
            if (cum + hist[b] >= need) break;
            cum += hist[b];
        }
        prefix = (prefix << 8) | (uint64_t)b;
        need -= cum;
        __syncthreads();
    }
    return (int64_t)(prefix ^ 0x8000000000000000ull);
}

// sum of v[i] over i with v[i] >= lo (v >= 0 here), CTA-wide
__device__ uint64_t cta_sum_at_least(const int64_t *v, int n, int64_t lo, uint64_t *red) {
    uint64_t s = 0;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        if (v[i] >= lo && v[i] > 0) s += (uint64_t)v[i];
    return (uint64_t)cta_sum_i128((i128)(u128)s, red);
}

// sample_token (llama_int.c:2958-3039) for row b of logits [rows][V], one CTA
// (IQ_SAMPLE_THREADS threads) per row, with the state of sequence seq_of(b);
// work [rows][V] is scratch. Same result as the reference, step for step:
//   temperature below 0.01: argmax; else w = fp_div(logit, T);
//   top-k: w < (k-th largest) -> INT64_MIN / 2;  softmax;
//   top-p: the reference adds the largest remaining probability (lowest index
//     among equals) until the running sum reaches p. That set is found
//     directly: t* = the largest t with sum_{w >= t} w >= p (bitwise search),
//     all w > t* and the first j of the w == t* (index order) with
//     j = ceil((p - sum_{w > t*} w) / t*); if all positive mass stays below p,
//     every positive w. Others are zeroed, kept ones renormalised (fp_div);
//   draw r = xoroshiro128+ >> 16; the first index whose running sum exceeds r,
//     else the argmax of the probabilities.
// Outputs as k_argmax (result, and the decode-state update when tokens != 0).
__global__ void __launch_bounds__(IQ_SAMPLE_THREADS)
k_sample(int *__restrict__ result, const int64_t *__restrict__ logits, int V, SampleState *__restrict__ st,
         int st_stride, int64_t *__restrict__ work, int *__restrict__ tokens, int *__restrict__ pos_arr,
         int *__restrict__ hist, int hist_stride) {
    __shared__ uint64_t red[64];
    __shared__ int sel_s;
    const int b = blockIdx.x;
    SampleState *S = st + (size_t)b * st_stride;
    const int64_t *lg = logits + (size_t)b * V;
    int64_t *w = work + (size_t)b * V;
    const int64_t ONE = (int64_t)1 << 48;
    const int64_t T = S->temperature;
    int sel;
    if (T <= 0 || T < ONE / 100) {
        sel = cta_argmax(lg, V);
    } else {
        for (int i = threadIdx.x; i < V; i += blockDim.x) w[i] = d_div(lg[i], T);
        __syncthreads();
        const int k = S->top_k;
        if (k > 0 && k < V) {
            const int64_t thr = cta_kth_largest(w, V, k);
            for (int i = threadIdx.x; i < V; i += blockDim.x)
                if (w[i] < thr) w[i] = INT64_MIN / 2;
            __syncthreads();
        }
        cta_softmax(w, V, red);
        __syncthreads();
        const int64_t P = S->top_p;
        if (P > 0 && P < ONE) {
            const uint64_t all = cta_sum_at_least(w, V, 1, red);
            int64_t tstar = 0;   // 0: keep every positive probability
            uint64_t s_gt = 0;
            int64_t j = 0;
            if (all >= (uint64_t)P) {
                for (int bit = 48; bit >= 0; bit--) {
                    const int64_t cand = tstar | ((int64_t)1 << bit);
                    if (cta_sum_at_least(w, V, cand, red) >= (uint64_t)P) tstar = cand;
                }
                s_gt = cta_sum_at_least(w, V, tstar + 1, red);
                j = (int64_t)(((uint64_t)P - s_gt + (uint64_t)tstar - 1) / (uint64_t)tstar);
            }
            // ties at t*: keep the first j in index order (a contiguous chunk per thread)
            const int C = (V + blockDim.x - 1) / blockDim.x, i0 = threadIdx.x * C, i1 = min(V, i0 + C);
            uint64_t eq = 0;
            for (int i = i0; i < i1; i++) eq += (tstar > 0 && w[i] == tstar);
            uint64_t before = cta_exclusive_scan(eq, nullptr);
            uint64_t kept = 0;
            for (int i = i0; i < i1; i++) {
                const int64_t v = w[i];
                bool keep = tstar == 0 ? v > 0 : (v > tstar || (v == tstar && (int64_t)before++ < j));
                w[i] = keep ? v : 0;
                kept += keep ? (uint64_t)v : 0;
            }
            const int64_t sum = (int64_t)(uint64_t)cta_sum_i128((i128)(u128)kept, red);
            __syncthreads();
            if (sum > 0)
                for (int i = threadIdx.x; i < V; i += blockDim.x)
                    if (w[i] > 0) w[i] = d_div(w[i], sum);
            __syncthreads();
        }
        // draw: one generator step (rng_next, llama_int.c:2921-2929)
        __shared__ int64_t r_s;
        if (threadIdx.x == 0) {
            const uint64_t s0 = S->s0;
            uint64_t s1 = S->s1;
            const uint64_t res = s0 + s1;
            s1 ^= s0;
            S->s0 = ((s0 << 55) | (s0 >> 9)) ^ s1 ^ (s1 << 14);
            S->s1 = (s1 << 36) | (s1 >> 28);
            r_s = (int64_t)(res >> 16);
            sel_s = 0x7fffffff;
        }
        __syncthreads();
        const int64_t r = r_s;
        const int C = (V + blockDim.x - 1) / blockDim.x, i0 = threadIdx.x * C, i1 = min(V, i0 + C);
        uint64_t part = 0;
        for (int i = i0; i < i1; i++) part += (uint64_t)w[i];
        uint64_t run = cta_exclusive_scan(part, nullptr);
        for (int i = i0; i < i1; i++) {
            run += (uint64_t)w[i];
            if ((int64_t)run > r) { atomicMin(&sel_s, i); break; }
        }
        __syncthreads();
        sel = sel_s;
        if (sel == 0x7fffffff) sel = cta_argmax(w, V);
    }
    if (threadIdx.x == 0) {
        result[b] = sel;
        if (tokens) tokens[b] = sel;
        if (pos_arr) {
            const int np1 = pos_arr[b] + 1;
            if (hist) hist[(size_t)b * hist_stride + np1] = sel;
            pos_arr[b] = np1;
        }
    }
}

// After a prefill: the argmax of the sequence's last prompt row becomes its
// next token at position L, recorded in the history (llama_int.c:3087-3089).
__global__ void k_prefill_done(const int *__restrict__ arg, int *__restrict__ tokens, int *__restrict__ pos_arr,
                               int *__restrict__ hist, int hist_stride, int seq, int L) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        tokens[seq] = arg[0];
        pos_arr[seq] = L;
        hist[(size_t)seq * hist_stride + L] = arg[0];
    }
}

}  // namespace iq
