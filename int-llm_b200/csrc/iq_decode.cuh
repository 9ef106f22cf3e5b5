// iq_decode.cuh -- the whole decode step of one sequence (llama_forward for one
// token, llama_int.c:2807-2886, then argmax, llama_int.c:2888-2893) as ONE
// persistent kernel: every SM stays resident for the token and the phases of
// each layer (transformer_layer_forward, llama_int.c:1326-1569) follow each
// other behind grid-wide barriers instead of kernel launches:
//   QKV (rmsnorm fused) | attention (RoPE, KV write, exact softmax, PV) |
//   O (+ residual) | gate|up (rmsnorm, SwiGLU fused) | down (+ residual)
// then the LM head (final rmsnorm fused) and a two-level first-max argmax.
// At the start of each matvec phase every CTA asks L2 to prefetch its own
// slice of the NEXT phase's weights (the stream-K split is static, so each
// CTA knows its byte range), so HBM keeps streaming across the barriers.
// The arithmetic is the per-kernel path's, bit for bit: the same stream-K
// matvec device code (mv_stream), the same integer attention formulas.
// Every grid barrier wait is bounded; on time-out the kernel records
// IQ_ERR_TIMEOUT, flags the barrier as abandoned and every CTA returns.
#pragma once
#include "iq_sync.cuh"
#include "iq_planes.cuh"

namespace iq {

// One matrix in the bf16 form, as the persistent kernel reads it.
struct MvView {
    const uint4 *planes;
    PackedRes R;
    int M, N, Kp;
};
struct DecLayer {
    MvView qkv, o, gu, down;
    const int64_t *n1, *n2;   // input / post-attention rmsnorm weights
    int64_t *kc, *vc;         // this layer's [max_seq][kvd] cache of sequence 0
};
// Grid barrier state: arrival count, generation word and abandon flag, each
// on its own 128-byte line.
struct GridBar {
    unsigned int count, pad0[31];
    unsigned int gen, pad1[31];
    unsigned int abort, pad2[31];
};
struct DecParams {
    int L, d, nh, nkv, hd, inter, V, max_seq, att_short, hist_stride;
    int64_t scale;                 // fp_inv_sqrt(fp_from_int(hd)) (llama_int.c:1433)
    const DecLayer *layers;        // device array [L]
    MvView lm;
    const int64_t *embed, *fnorm, *rcos, *rsin;
    int64_t *hidden, *qkv, *att, *act, *logits;
    RowAcc *racc;
    int64_t *asc, *amx;            // [nh][max_seq] scores / numerators, [nh] maxima
    unsigned long long *asum;      // [nh] wrapping int64 sums
    unsigned long long *argv;      // [gridDim.x][2] per-CTA (value, index)
    int *d_tok, *d_pos, *d_arg, *d_hist;
    GridBar *bar;
    unsigned long long *stamps;    // optional: %globaltimer after each barrier (CTA 0), for profiling
    int prefetch;                  // 1 = L2 prefetch of the next phase's weights
};

#define IQ_DEC_THREADS 256
#define IQ_GRID_WAIT_NS 1000000000ull   // healthy barrier waits last microseconds

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u32(unsigned int *p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// Profiling aid: CTA 0 thread 0 appends (tag, %globaltimer) to the stamp log.
__device__ unsigned long long *g_dec_stamps;
__device__ __forceinline__ void dec_mark(int tag) {
    unsigned long long *st = g_dec_stamps;
    if (st && blockIdx.x == 0 && threadIdx.x == 0) {
        const unsigned long long i = st[0]++;
        if (i < 1022) st[2 + i] = ((unsigned long long)tag << 56) | (global_ns() & ((1ull << 56) - 1));
    }
}

__shared__ unsigned int s_dec_phase;  // this CTA's matvec phase count in the step
__device__ __forceinline__ void mv_mark(int tag) {
    dec_mark(tag);
    unsigned long long *st = g_dec_stamps;
    if (tag == 7 && st && (threadIdx.x & 31) == 0) {   // latest loop end over every warp of the grid
        const unsigned int ph = s_dec_phase;
        if (ph < 300) atomicMax(&st[700 + ph], global_ns() & ((1ull << 56) - 1));
    }
    if (tag == 6 && st && (threadIdx.x & 31) == 0) {   // latest staging end
        const unsigned int ph = s_dec_phase;
        if (ph < 300) atomicMax(&st[400 + ph], global_ns() & ((1ull << 56) - 1));
    }
}

__device__ __forceinline__ unsigned int ld_relaxed_u32(const unsigned int *p) {
    unsigned int v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier: the CTA's writes are ordered before its arrival
// (bar.sync + gpu-scope fence), the last CTA to arrive resets the count and
// releases the next generation; the others poll the generation with relaxed
// loads and fence once it moved. Measured on B200: ~2.3 us at 148 CTAs, ~2.9
// at 296 (a two-level count and per-CTA arrival flags were both slower).
// Returns false when the barrier was abandoned.
__device__ __forceinline__ bool grid_sync(GridBar *b, unsigned long long *stamps = nullptr) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        int good = 1;
        const unsigned int g = ld_relaxed_u32(&b->gen);
        __threadfence();
        if (atomicAdd(&b->count, 1u) == gridDim.x - 1) {
            b->count = 0;
            __threadfence();
            st_release_u32(&b->gen, g + 1);
        } else {
            const uint64_t t0 = global_ns();
            unsigned int it = 0;
            while (ld_relaxed_u32(&b->gen) == g) {
                if ((++it & 63u) == 0) {
                    if (ld_relaxed_u32(&b->abort)) { good = 0; break; }
                    if (global_ns() - t0 > IQ_GRID_WAIT_NS) {
                        atomicExch(&b->abort, 1u);
                        atomicExch(&g_iq_err, (int)IQ_ERR_TIMEOUT);
                        good = 0;
                        break;
                    }
                }
            }
            __threadfence();   // acquire side: what the releasing CTA saw is visible
        }
        ok = good;
        if (stamps && blockIdx.x == 0) {   // [0] = count, [1] = start, [2..] = (tag 0, time)
            const unsigned long long i = stamps[0]++;
            if (i < 1022) stamps[2 + i] = global_ns() & ((1ull << 56) - 1);
        }
    }
    __syncthreads();
    return ok != 0;
}

// Barrier cost probe: iters barriers with no work between them.
__global__ void k_bar_bench(GridBar *b, int iters) {
    for (int i = 0; i < iters; i++)
        if (!grid_sync(b)) return;
}

// The stream-K matvec of one phase over every warp of the grid (one out-of-line
// copy: it keeps the standalone kernel's register budget without spills).
__device__ __noinline__ void dec_mv(const MvView &W, const int64_t *x, const int64_t *nrm, int64_t *out, int add,
                                       RowAcc *racc, unsigned char *xd) {
    dec_mark(5);
    if (threadIdx.x == 0) s_dec_phase++;
    __syncthreads();
    mv_stream<3, true, true, false>(out, W.planes, W.R, x, W.M, W.N, W.Kp, add, racc, nrm, xd,
                                    (int64_t)blockIdx.x * (IQ_DEC_THREADS / 32) + (threadIdx.x >> 5),
                                    (int64_t)gridDim.x * (IQ_DEC_THREADS / 32));
}

// Asks L2 to prefetch the weight tiles this CTA's warps will read in W's
// stream-K split (1 KB per 16 x 32 tile in the bf16 form), 32 KB per request.
__device__ __forceinline__ void l2_prefetch_slice(const MvView &W, int on) {
    if (!on || threadIdx.x >= 32) return;
    const int64_t total = (int64_t)((W.M + 15) / 16) * (W.Kp / 32);
    const int64_t nw = (int64_t)gridDim.x * (IQ_DEC_THREADS / 32), w0 = (int64_t)blockIdx.x * (IQ_DEC_THREADS / 32);
    const int64_t u0 = total * w0 / nw, u1 = total * (w0 + IQ_DEC_THREADS / 32) / nw;
    const char *base = reinterpret_cast<const char *>(W.planes) + u0 * 1024;
    const int64_t len = (u1 - u0) * 1024;
    for (int64_t off = (int64_t)threadIdx.x * 32768; off < len; off += 32 * 32768) {
        const uint32_t n = (uint32_t)min((int64_t)32768, len - off);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(base + off), "r"(n) : "memory");
    }
}

// RoPE of one head vector (rope_apply, llama_int.c:997-1008) into dst.
__device__ __forceinline__ void rope_head(int64_t *dst, const int64_t *src, const int64_t *c, const int64_t *s,
                                          int hd) {
    const int half = hd / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const int64_t x0 = src[i], x1 = src[i + half];
        dst[i] = d_mul(x0, c[i]) - d_mul(x1, s[i]);
        dst[i + half] = d_mul(x1, c[i]) + d_mul(x0, s[i]);
    }
}

// Exact score of positions t (the current one from the CTA's own roped key,
// earlier ones from the cache): fp_mul((int64)(sum_d (i128)q k >> 48), scale).
// Groups of 8 lanes split the dims of one position (coalesced 64-byte pieces).
__device__ __forceinline__ void scores_range(int64_t *sc_out, int t0, int nt, int pos, const int64_t *qs,
                                             const int64_t *ks, const int64_t *kcache, int kvd, int hd,
                                             int64_t scale) {
    const int sl = threadIdx.x & 7, nsg = blockDim.x >> 3;
    for (int tb = 0; tb < nt; tb += nsg) {  // uniform trip count: every lane shuffles
        const int tt = tb + (threadIdx.x >> 3), t = t0 + tt;
        const bool live = tt < nt;
        const int64_t *kr = (live && t == pos) ? ks : kcache + (size_t)(live ? t : 0) * kvd;
        i128 dot = 0;
        for (int d = sl; d < hd; d += 8) dot += d_mul128(qs[d], live ? kr[d] : 0);
#pragma unroll
        for (int m = 4; m >= 1; m >>= 1) dot += shfl_xor_i128(dot, m);
        if (live && sl == 0) sc_out[tt] = d_mul((int64_t)(dot >> 48), scale);
    }
}

// Attention with one CTA per query head (contexts up to att_short): RoPE,
// KV write at pos (by the first query head of each kv group), scores, integer
// softmax, PV -- k_attention's arithmetic (llama_int.c:1432-1529).
__device__ __noinline__ void dec_attn_short(const DecParams &p, const DecLayer &Ly, int pos, int64_t *sm) {
    __shared__ uint64_t red[64];
    const int hd = p.hd, grp = p.nh / p.nkv, kvd = p.nkv * hd, T = pos + 1, half = hd / 2;
    const int64_t *c = p.rcos + (size_t)pos * half, *sn = p.rsin + (size_t)pos * half;
    for (int h = blockIdx.x; h < p.nh; h += gridDim.x) {
        const int g = h / grp;
        int64_t *qs = sm, *ks = sm + hd, *vs = sm + 2 * hd, *sc = sm + 3 * hd;   // sc: [T], then [groups][hd]
        rope_head(qs, p.qkv + (size_t)h * hd, c, sn, hd);
        rope_head(ks, p.qkv + p.d + (size_t)g * hd, c, sn, hd);
        for (int i = threadIdx.x; i < hd; i += blockDim.x) vs[i] = p.qkv[p.d + kvd + g * hd + i];
        __syncthreads();
        dec_mark(1);
        if (h % grp == 0)   // the cache row at pos, once per kv head (llama_int.c:1415-1416)
            for (int i = threadIdx.x; i < hd; i += blockDim.x) {
                Ly.kc[(size_t)pos * kvd + g * hd + i] = ks[i];
                Ly.vc[(size_t)pos * kvd + g * hd + i] = vs[i];
            }
        scores_range(sc, 0, T, pos, qs, ks, Ly.kc + g * hd, kvd, hd, p.scale);
        __syncthreads();
        dec_mark(2);
        cta_softmax(sc, T, red);
        __syncthreads();
        dec_mark(3);
        const int groups = blockDim.x / hd, gi = threadIdx.x / hd, d = threadIdx.x % hd;
        uint64_t acc = 0;
        if (gi < groups)
            for (int t = gi; t < T; t += groups)
                acc += (uint64_t)d_mul(sc[t], t == pos ? vs[d] : Ly.vc[(size_t)t * kvd + g * hd + d]);
        __syncthreads();
        int64_t *part = sc;   // reuse: [groups][hd]
        if (gi < groups) part[gi * hd + d] = (int64_t)acc;
        __syncthreads();
        for (int dd = threadIdx.x; dd < hd; dd += blockDim.x) {
            uint64_t s = 0;
            for (int gg = 0; gg < groups; gg++) s += (uint64_t)part[gg * hd + dd];
            p.att[(size_t)h * hd + dd] = (int64_t)s;
        }
        __syncthreads();
        dec_mark(4);
    }
}

#define DEC_TILE 64
// Long contexts, step 1 of 3, units (query head, 64-position tile) over the
// grid: scores into asc and the tile maximum into amx (atomic max). The unit
// holding pos ropes k and, for the first query head of its group, writes the
// cache row (k and v) at pos.
__device__ __noinline__ void dec_attn_scores(const DecParams &p, const DecLayer &Ly, int pos, int64_t *sm) {
    const int hd = p.hd, grp = p.nh / p.nkv, kvd = p.nkv * hd, T = pos + 1, half = hd / 2;
    const int ntile = (T + DEC_TILE - 1) / DEC_TILE;
    const int64_t *c = p.rcos + (size_t)pos * half, *sn = p.rsin + (size_t)pos * half;
    for (int u = blockIdx.x; u < p.nh * ntile; u += gridDim.x) {
        const int h = u / ntile, tile = u % ntile, g = h / grp, t0 = tile * DEC_TILE;
        const int nt = min(DEC_TILE, T - t0);
        int64_t *qs = sm, *ks = sm + hd, *sc = sm + 2 * hd;
        rope_head(qs, p.qkv + (size_t)h * hd, c, sn, hd);
        const bool has_pos = pos >= t0 && pos < t0 + nt;
        if (has_pos) rope_head(ks, p.qkv + p.d + (size_t)g * hd, c, sn, hd);
        __syncthreads();
        if (has_pos && h % grp == 0)
            for (int i = threadIdx.x; i < hd; i += blockDim.x) {
                Ly.kc[(size_t)pos * kvd + g * hd + i] = ks[i];
                Ly.vc[(size_t)pos * kvd + g * hd + i] = p.qkv[p.d + kvd + g * hd + i];
            }
        scores_range(sc, t0, nt, pos, qs, ks, Ly.kc + g * hd, kvd, hd, p.scale);
        __syncthreads();
        if (threadIdx.x < 32) {
            int64_t m = INT64_MIN;
            for (int i = threadIdx.x; i < nt; i += 32) {
                m = max(m, sc[i]);
                p.asc[(size_t)h * p.max_seq + t0 + i] = sc[i];
            }
            for (int k = 16; k >= 1; k >>= 1) m = max(m, (int64_t)__shfl_xor_sync(0xffffffffu, m, k));
            if (threadIdx.x == 0) atomicMax((long long *)&p.amx[h], (long long)m);
        }
        __syncthreads();
    }
}

// Step 2: e_t = fp_safe_exp(s_t - max) in place; S = wrapping int64 sum.
__device__ __noinline__ void dec_attn_exp(const DecParams &p, int pos) {
    const int T = pos + 1, ntile = (T + DEC_TILE - 1) / DEC_TILE;
    for (int u = blockIdx.x; u < p.nh * ntile; u += gridDim.x) {
        const int h = u / ntile, t0 = (u % ntile) * DEC_TILE;
        const int nt = min(DEC_TILE, T - t0);
        if (threadIdx.x < 64) {
            uint64_t e = 0;
            if ((int)threadIdx.x < nt) {
                int64_t *s = p.asc + (size_t)h * p.max_seq + t0 + threadIdx.x;
                const int64_t v = d_safe_exp((int64_t)((uint64_t)*s - (uint64_t)p.amx[h]));
                *s = v;
                e = (uint64_t)v;
            }
            for (int k = 16; k >= 1; k >>= 1) e += __shfl_xor_sync(0xffffffffu, e, k);
            if ((threadIdx.x & 31) == 0) atomicAdd(&p.asum[h], (unsigned long long)e);
        }
    }
}

// Step 3: p_t = fp_div(e_t, S) (if S > 0), partial sums of fp_mul(p_t, v_t[d])
// over the tile, added into att (wrapping int64: exact in any order).
__device__ __noinline__ void dec_attn_pv(const DecParams &p, const DecLayer &Ly, int pos, int64_t *sm) {
    const int hd = p.hd, grp = p.nh / p.nkv, kvd = p.nkv * hd, T = pos + 1;
    const int ntile = (T + DEC_TILE - 1) / DEC_TILE;
    for (int u = blockIdx.x; u < p.nh * ntile; u += gridDim.x) {
        const int h = u / ntile, g = h / grp, t0 = (u % ntile) * DEC_TILE;
        const int nt = min(DEC_TILE, T - t0);
        int64_t *ps = sm;   // [DEC_TILE] then [groups][hd]
        const int64_t S = (int64_t)p.asum[h];
        for (int i = threadIdx.x; i < nt; i += blockDim.x) {
            int64_t v = p.asc[(size_t)h * p.max_seq + t0 + i];
            ps[i] = S > 0 ? d_div(v, S) : v;
        }
        __syncthreads();
        const int groups = blockDim.x / hd, gi = threadIdx.x / hd, d = threadIdx.x % hd;
        uint64_t acc = 0;
        if (gi < groups)
            for (int i = gi; i < nt; i += groups)
                acc += (uint64_t)d_mul(ps[i], Ly.vc[(size_t)(t0 + i) * kvd + g * hd + d]);
        if (gi < groups) atomicAdd((unsigned long long *)&p.att[(size_t)h * hd + d], (unsigned long long)acc);
        __syncthreads();
    }
}

// One decode step of sequence 0: token d_tok[0] at position d_pos[0]; on exit
// d_arg[0] = d_tok[0] = argmax, d_pos[0] += 1 and d_hist records the token.
__global__ void __launch_bounds__(IQ_DEC_THREADS, 2) k_decode_token(const __grid_constant__ DecParams p) {
    extern __shared__ __align__(16) unsigned char dsm[];
    int64_t *sm64 = reinterpret_cast<int64_t *>(dsm);
    if (ld_acquire_u32(&p.bar->abort)) return;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        g_dec_stamps = p.stamps;
        if (p.stamps) {
            p.stamps[0] = 0;
            p.stamps[1] = global_ns() & ((1ull << 56) - 1);
            for (int i = 400; i < 1024; i++) p.stamps[i] = 0;
        }
    }
    if (threadIdx.x == 0) s_dec_phase = 0;
    const int tok = p.d_tok[0], pos = p.d_pos[0];
    const bool chunked = pos + 1 > p.att_short;
    const int64_t *erow = p.embed + (size_t)tok * p.d;   // hidden = embed[token] (llama_int.c:2822-2824)
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < p.d; i += blockDim.x) p.hidden[i] = erow[i];
    for (int l = 0; l < p.L; l++) {
        const DecLayer &Ly = p.layers[l];
        if (blockIdx.x == gridDim.x - 1) {   // nothing reads these before the next barrier
            for (int i = threadIdx.x; i < p.nh * p.hd; i += blockDim.x) p.att[i] = 0;
            for (int i = threadIdx.x; i < p.nh; i += blockDim.x) { p.amx[i] = INT64_MIN; p.asum[i] = 0; }
        }
        l2_prefetch_slice(Ly.o, p.prefetch);
        dec_mv(Ly.qkv, l == 0 ? erow : p.hidden, Ly.n1, p.qkv, IQ_EPI_STORE, p.racc, dsm);
        if (!grid_sync(p.bar, p.stamps)) return;
        l2_prefetch_slice(Ly.gu, p.prefetch);
        if (!chunked) {
            dec_attn_short(p, Ly, pos, sm64);
        } else {
            dec_attn_scores(p, Ly, pos, sm64);
            if (!grid_sync(p.bar, p.stamps)) return;
            dec_attn_exp(p, pos);
            if (!grid_sync(p.bar, p.stamps)) return;
            dec_attn_pv(p, Ly, pos, sm64);
        }
        if (!grid_sync(p.bar, p.stamps)) return;
        l2_prefetch_slice(Ly.down, p.prefetch);
        dec_mv(Ly.o, p.att, nullptr, p.hidden, IQ_EPI_ADD, p.racc, dsm);
        if (!grid_sync(p.bar, p.stamps)) return;
        l2_prefetch_slice(l + 1 < p.L ? p.layers[l + 1].qkv : p.lm, p.prefetch);
        dec_mv(Ly.gu, p.hidden, Ly.n2, p.act, IQ_EPI_SWIGLU, p.racc, dsm);
        if (!grid_sync(p.bar, p.stamps)) return;
        dec_mv(Ly.down, p.act, nullptr, p.hidden, IQ_EPI_ADD, p.racc, dsm);
        if (!grid_sync(p.bar, p.stamps)) return;
    }
    dec_mv(p.lm, p.hidden, p.fnorm, p.logits, IQ_EPI_STORE, p.racc, dsm);
    if (!grid_sync(p.bar, p.stamps)) return;
    {   // first maximum of this CTA's slice (strict >, llama_int.c:2888-2893)
        __shared__ int64_t bv[IQ_DEC_THREADS / 32];
        __shared__ int bi[IQ_DEC_THREADS / 32];
        const int lo = (int)((int64_t)p.V * blockIdx.x / gridDim.x), hi = (int)((int64_t)p.V * (blockIdx.x + 1) / gridDim.x);
        int64_t best = INT64_MIN;
        int idx = 0x7fffffff;
        for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            const int64_t v = p.logits[i];
            if (v > best) { best = v; idx = i; }
        }
        for (int m = 16; m >= 1; m >>= 1) {
            const int64_t ov = __shfl_xor_sync(0xffffffffu, best, m);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, m);
            if (ov > best || (ov == best && oi < idx)) { best = ov; idx = oi; }
        }
        if ((threadIdx.x & 31) == 0) { bv[threadIdx.x >> 5] = best; bi[threadIdx.x >> 5] = idx; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < IQ_DEC_THREADS / 32; w++)
                if (bv[w] > best || (bv[w] == best && bi[w] < idx)) { best = bv[w]; idx = bi[w]; }
            p.argv[2 * blockIdx.x] = (unsigned long long)best;
            p.argv[2 * blockIdx.x + 1] = (unsigned long long)(unsigned)idx;
        }
    }
    if (!grid_sync(p.bar, p.stamps)) return;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        int64_t best = INT64_MIN;
        int idx = 0x7fffffff;
        for (unsigned int b = 0; b < gridDim.x; b++) {
            const int64_t v = (int64_t)p.argv[2 * b];
            const int i = (int)p.argv[2 * b + 1];
            if (v > best || (v == best && i < idx)) { best = v; idx = i; }
        }
        p.d_arg[0] = idx;
        p.d_tok[0] = idx;
        const int np1 = pos + 1;
        p.d_pos[0] = np1;
        if (p.d_hist) p.d_hist[np1] = idx;
    }
}

}  // namespace iq
