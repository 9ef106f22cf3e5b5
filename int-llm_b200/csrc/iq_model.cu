// iq_model.cu -- device-resident integer Llama model: weights, RoPE tables,
// exact int64 KV cache and the decode step (llama_forward, llama_int.c:2807-2886)
// built from the kernels in iq_layer.cuh, captured once into a CUDA graph and
// replayed per token; greedy generate (llama_int.c:3067-3135) on top.
//
// Tensor parallelism (output rows): rank r of P owns a contiguous block of q
// heads, the kv heads they read (a kv head is replicated on every rank whose q
// heads use it when P > n_kv), rows [r*d/P, (r+1)*d/P) of O and down,
// rows [r*inter/P, ...) of gate and of up, and rows [r*V/P, ...) of the LM
// head. Every projection output is all-gathered (NCCL, int64, a pure copy), so
// no partial sum ever crosses a GPU and the result is bit-identical at every P.
// Per layer: rmsnorm -> QKV (local heads) -> RoPE + KV write -> attention
// (local heads) -> gather -> O rows -> gather -> += residual -> rmsnorm ->
// gate|up rows -> SwiGLU -> gather -> down rows -> gather -> += residual;
// then final rmsnorm, LM-head rows, gather of the logits, first-max argmax.
// With P = 1 the gathers vanish and the residual adds fuse into the O and
// down projections' epilogues.
#include <cstring>
#include <thread>
#include <atomic>
#include <string>
#include <algorithm>
#include <cstdio>
#include <vector>
#include <chrono>
#include <nccl.h>
#include "iq_common.cuh"
#include "iq_layer.cuh"
#include "iq_decode.cuh"

using namespace iq;

struct Shard {
    int P = 1, r = 0;
    int nh_l = 0, nkv_l = 0;         // local q / kv heads
    int q_lo = 0, kv_lo = 0;         // first local q / kv head (global index)
    int d_l = 0, it_l = 0, v_l = 0;  // local rows of O/down, of gate (and of up), of the LM head
};

// Row ownership of rank r among P; IQ_ERR_ARG where the shapes do not divide.
static int make_shard(const iq_config &c, int P, int r, Shard *s) {
    if (P < 1 || r < 0 || r >= P) return IQ_ERR_ARG;
    if (c.num_heads % P || c.hidden_dim % P || c.intermediate_dim % P || c.vocab_size % P) return IQ_ERR_ARG;
    const int grp = c.num_heads / c.num_kv_heads;
    s->P = P; s->r = r;
    s->nh_l = c.num_heads / P;
    s->q_lo = r * s->nh_l;
    const int kv_first = s->q_lo / grp, kv_last = (s->q_lo + s->nh_l - 1) / grp;
    s->kv_lo = kv_first;
    s->nkv_l = kv_last - kv_first + 1;
    // local head h_l must read local kv head h_l / (nh_l / nkv_l), the same map as globally
    if (s->nh_l % s->nkv_l || s->nh_l / s->nkv_l != std::min(grp, s->nh_l)) return IQ_ERR_ARG;
    if (grp < s->nh_l && s->nh_l % grp) return IQ_ERR_ARG;
    s->d_l = c.hidden_dim / P;
    s->it_l = c.intermediate_dim / P;
    s->v_l = c.vocab_size / P;
    return IQ_OK;
}

struct iq_model {
    iq_config c;
    Shard sh;
    int dev = 0;
    int max_batch = 1;
    int kvd_l = 0, qkv_rows = 0;  // local kv width, local fused QKV rows
    cudaStream_t s = nullptr;
    ncclComm_t comm = nullptr;
    // weights (local rows)
    int64_t *embed = nullptr, *fnorm = nullptr, *lm = nullptr;
    std::vector<int64_t *> norm1, wqkv, wo, norm2, wgu, wdown;
    std::vector<int64_t *> kc, vc;  // per layer [B][max_seq][kvd_l]
    int64_t *rcos = nullptr, *rsin = nullptr;
    // byte-plane packed copies of every projection (M=1 decode path)
    std::vector<Packed> pqkv, po, pgu, pdown;
    Packed plm;
    // tcgen05 row-plane copies (rows >= 2: batched decode, prefill)
    std::vector<PackedTC> tqkv, to, tgu, tdown;
    PackedTC tlm;
    uint8_t *digits = nullptr;  // x-digit scratch of the tcgen05 GEMM
    int64_t *gpart = nullptr;   // split-K partial scratch of the tcgen05 GEMM
    size_t gpart_bytes = 0;
    int rmax = 1;               // row capacity of the activation buffers
    int *d_seq = nullptr;       // sequence of each decode row (identity)
    int *d_ptok = nullptr, *d_ppos = nullptr, *d_pseq = nullptr;  // prefill rows
    RowAcc *racc = nullptr;  // split-row scratch of the packed matvec (self-resetting)
    // activations (device)
    int64_t *hidden = nullptr, *normed = nullptr, *qkv = nullptr, *att = nullptr, *gu = nullptr,
            *act = nullptr, *logits = nullptr;
    // tensor-parallel buffers: local pieces and gather staging (P > 1)
    int64_t *att_l = nullptr, *proj_l = nullptr, *act_l = nullptr, *logits_l = nullptr, *gath = nullptr,
            *proj_full = nullptr;
    int *d_tok = nullptr, *d_pos = nullptr, *d_arg = nullptr, *d_hist = nullptr;
    int *h_pin = nullptr;  // pinned host scratch: tokens / pos / argmax
    int *h_rows = nullptr; // pinned host scratch: prefill rows (token, pos, seq) x max_seq
    int64_t *h_logits = nullptr;
    size_t attn_smem = 0;
    size_t gqa_smem = 0;  // k_attention_gqa shared memory (0 = use k_attention)
    int hpc = 1;          // query heads per attention CTA
    int att_pv_tc = 0;       // phase 3 on the tensor cores (k_attn_pv_tc<att_pv_tc>), 0: off
    size_t att_s3tc = 0;
    int att_scores_tc = 0;   // scores on the int8 tensor cores (k_attn_scores_tc)
    int att_pv_spt = 0;   // k_attn_pv instance (att_pv_spt())
    int att_phased = 1;   // phased attention (k_attn_*), else one CTA per (row, head)
    int64_t *asc = nullptr, *amx = nullptr;  // phased-attention scratch: scores, maxima
    uint64_t *asum = nullptr;                // and sums
    size_t att_s1 = 0, att_s3 = 0;           // its shared-memory sizes
    cudaGraphExec_t graph = nullptr;    // one decode step at batch max_batch (phased attention)
    cudaGraphExec_t graph_s = nullptr;  // the same step with single-kernel attention
    int att_short = 0;  // steps whose positions all lie below this use k_attention
    int64_t att_scale = 0;  // fp_inv_sqrt(fp_from_int(head_dim))
    bool loaded_globals = false;
    std::vector<bool> loaded_layer;
    // persistent decode kernel (k_decode_token) for batch 1 without tensor
    // parallelism: requested mode, and its state once prepared
    bool failed = false;        // the communicator was aborted or a peer left: the model is unusable
    int (*peer_check)(void *) = nullptr;   // host-side liveness of the other ranks (nonzero: one left)
    void *peer_ctx = nullptr;
    int64_t timeout_ms = 60000; // bounded host waits under tensor parallelism
    bool want_logits = false;   // decode steps also gather the full logits (TP; hashing callers)
    int kv_kbits = 0, kv_vbits = 0;   // packed KV cache (K and V code widths); 0 = exact
    std::vector<uint8_t *> kq;        // per layer [B][max_seq][kvd] K codes
    std::vector<uint16_t *> vq;       // per layer V codes
    std::vector<int64_t *> kmag, vmag; // per layer [B][max_seq][nkv] magnitudes
    bool sampling = false;      // steps draw with sample_token instead of argmax
    SampleState *d_samp = nullptr;   // [max_batch] sampling parameters and generator states
    int64_t *swork = nullptr;        // [rmax][vocab] sampling scratch
    int prefill_seq = 0;             // sequence of the prefill chunk being enqueued
    int64_t *pairs_l = nullptr, *pairs_g = nullptr;   // TP argmax: local pair, gathered pairs
    int dec_mode = 0;           // 1 = use it where it applies, 0 = per-kernel path (default: faster today)
    bool dec_ready = false;     // prepared for the current weights
    DecParams dec{};
    DecLayer *d_layers = nullptr;
    GridBar *bar = nullptr;
    unsigned long long *argv = nullptr;
    int dec_grid = 0;
    size_t dec_smem = 0;
};

static const void *att_pv_kernel(int spt) {
    switch (spt) {
        case 1: return (const void *)k_attn_pv<1>;
        case 2: return (const void *)k_attn_pv<2>;
        case 4: return (const void *)k_attn_pv<4>;
        case 8: return (const void *)k_attn_pv<8>;
        default: return (const void *)k_attn_pv<0>;
    }
}

static const void *att_pv_tc_kernel(int hb) {
    return hb == 2 ? (const void *)k_attn_pv_tc<2> : (const void *)k_attn_pv_tc<1>;
}

static int dalloc(void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes ? bytes : 8);
    if (e != cudaSuccess) return cuda_fail(e);
    return IQ_OK;
}
#define DALLOC(p, bytes) do { int _r = dalloc((void **)&(p), (bytes)); if (_r) return _r; } while (0)

// RoPE tables computed on the device with the fp_math ports (rope_init, llama_int.c:960-986)
__global__ void k_rope_init(int64_t *cs, int64_t *sn, int hd, int max_seq, int theta) {
    const CordicTables &ct = g_cordic;
    int half = hd / 2;
    int64_t lt = d_log(d_from_int(theta));
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < max_seq * half; e += gridDim.x * blockDim.x) {
        int p = e / half, i = e % half;
        int64_t nf = -d_div(d_from_int(2 * i), d_from_int(hd));
        int64_t th = d_exp(d_mul(nf, lt));
        int64_t c, s;
        d_sincos(ct, d_mul(d_from_int(p), th), &c, &s);
        cs[e] = c;
        sn[e] = s;
    }
}

// x[i] += y[i] (int64 wrap): the residual adds of llama_int.c:1535, 1556
__global__ void k_add(int64_t *__restrict__ x, const int64_t *__restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] = (int64_t)((uint64_t)x[i] + (uint64_t)y[i]);
}

// all-gather output [P][B][w] -> [B][P*w]
__global__ void k_unshard(int64_t *__restrict__ out, const int64_t *__restrict__ g, int P, int B, int w) {
    const int64_t n = (int64_t)P * B * w;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        int64_t p = e / ((int64_t)B * w), rem = e % ((int64_t)B * w);
        int64_t b = rem / w, i = rem % w;
        out[b * (int64_t)P * w + p * w + i] = g[e];
    }
}

// raw int64 weights live on the device only while a layer is being packed
static int alloc_raw_layer(iq_model *m, int l) {
    const iq_config &c = m->c;
    const Shard &S = m->sh;
    const size_t d = c.hidden_dim;
    if (!m->norm1[l]) DALLOC(m->norm1[l], d * 8);
    if (!m->norm2[l]) DALLOC(m->norm2[l], d * 8);
    if (!m->wqkv[l]) DALLOC(m->wqkv[l], (size_t)m->qkv_rows * d * 8);
    if (!m->wo[l]) DALLOC(m->wo[l], (size_t)S.d_l * d * 8);
    if (!m->wgu[l]) DALLOC(m->wgu[l], (size_t)2 * S.it_l * d * 8);
    if (!m->wdown[l]) DALLOC(m->wdown[l], (size_t)S.d_l * c.intermediate_dim * 8);
    return IQ_OK;
}
static void free_raw_layer(iq_model *m, int l) {
    for (int64_t **p : {&m->wqkv[l], &m->wo[l], &m->wgu[l], &m->wdown[l]})
        if (*p) { cudaFree(*p); *p = nullptr; }
}

static int model_alloc(iq_model *m) {
    const iq_config &c = m->c;
    const Shard &S = m->sh;
    const int B = m->rmax, d = c.hidden_dim, L = c.num_layers, hd = c.head_dim;
    m->kvd_l = S.nkv_l * hd;
    m->qkv_rows = S.nh_l * hd + 2 * m->kvd_l;
    DALLOC(m->embed, (size_t)c.vocab_size * d * 8);
    DALLOC(m->fnorm, (size_t)d * 8);
    m->norm1.resize(L); m->wqkv.resize(L); m->wo.resize(L); m->norm2.resize(L);
    m->wgu.resize(L); m->wdown.resize(L); m->kc.resize(L); m->vc.resize(L);
    m->pqkv.resize(L); m->po.resize(L); m->pgu.resize(L); m->pdown.resize(L);
    m->tqkv.resize(L); m->to.resize(L); m->tgu.resize(L); m->tdown.resize(L);
    m->loaded_layer.assign(L, false);
    for (int l = 0; l < L; l++) {
        DALLOC(m->norm1[l], (size_t)d * 8);
        DALLOC(m->norm2[l], (size_t)d * 8);
        size_t kvb = (size_t)m->max_batch * c.max_seq_len * m->kvd_l * 8;
        DALLOC(m->kc[l], kvb);
        DALLOC(m->vc[l], kvb);
    }
    size_t rows = std::max(std::max((size_t)S.v_l, (size_t)m->qkv_rows),
                           std::max((size_t)2 * S.it_l, (size_t)d)) + 16;
    DALLOC(m->racc, rows * sizeof(RowAcc));
    IQ_CUDA(cudaMemset(m->racc, 0, rows * sizeof(RowAcc)));
    size_t half = hd / 2;
    DALLOC(m->rcos, (size_t)c.max_seq_len * half * 8);
    DALLOC(m->rsin, (size_t)c.max_seq_len * half * 8);
    DALLOC(m->hidden, (size_t)B * d * 8);
    DALLOC(m->normed, (size_t)B * d * 8);
    DALLOC(m->qkv, (size_t)B * m->qkv_rows * 8);
    DALLOC(m->att, (size_t)B * d * 8);
    DALLOC(m->gu, (size_t)B * 2 * S.it_l * 8);
    DALLOC(m->act, (size_t)B * c.intermediate_dim * 8);
    DALLOC(m->logits, (size_t)B * c.vocab_size * 8);
    if (S.P > 1) {
        size_t wmax = std::max(std::max((size_t)d, (size_t)c.intermediate_dim), (size_t)c.vocab_size);
        DALLOC(m->att_l, (size_t)B * S.nh_l * hd * 8);
        DALLOC(m->proj_l, (size_t)B * S.d_l * 8);
        DALLOC(m->act_l, (size_t)B * S.it_l * 8);
        DALLOC(m->logits_l, (size_t)B * S.v_l * 8);
        DALLOC(m->gath, (size_t)B * wmax * 8);
        DALLOC(m->proj_full, (size_t)B * d * 8);
        DALLOC(m->pairs_l, (size_t)B * 2 * 8);
        DALLOC(m->pairs_g, (size_t)S.P * B * 2 * 8);
    }
    const int NB = m->max_batch;
    DALLOC(m->d_tok, (size_t)NB * 4);
    DALLOC(m->d_pos, (size_t)NB * 4);
    DALLOC(m->d_seq, (size_t)NB * 4);
    DALLOC(m->d_arg, (size_t)B * 4);
    DALLOC(m->d_hist, (size_t)NB * (c.max_seq_len + 1) * 4);
    DALLOC(m->d_samp, (size_t)NB * sizeof(SampleState));
    DALLOC(m->swork, (size_t)NB * c.vocab_size * 8);
    DALLOC(m->d_ptok, (size_t)B * 4);
    DALLOC(m->d_ppos, (size_t)B * 4);
    DALLOC(m->d_pseq, (size_t)B * 4);
    {
        std::vector<int> ident(NB);
        for (int i = 0; i < NB; i++) ident[i] = i;
        IQ_CUDA(cudaMemcpy(m->d_seq, ident.data(), (size_t)NB * 4, cudaMemcpyHostToDevice));
    }
    {
        size_t kmax = std::max((size_t)d, (size_t)c.intermediate_dim);
        size_t kpad = (kmax + TC_BK - 1) / TC_BK * TC_BK, rpad = ((size_t)B + TC_BR - 1) / TC_BR * TC_BR;
        DALLOC(m->digits, rpad * 8 * kpad);
        // split-K partials: KS * Rpad * Mpad * 16 with KS * tiles <= 2 * SMs + tiles
        m->gpart_bytes = (size_t)(8 * dev_info().sms + 8) * TC_BM * TC_BR * 16;
        DALLOC(m->gpart, m->gpart_bytes);
    }
    // pinned ints: [0, B) results, then (max_seq + 2) slots of 2*NB (token, pos)
    IQ_CUDA(cudaMallocHost(&m->h_pin, ((size_t)B + 16 + (size_t)2 * NB * (c.max_seq_len + 2)) * 4));
    IQ_CUDA(cudaMallocHost(&m->h_logits, (size_t)c.vocab_size * 8));
    IQ_CUDA(cudaMallocHost(&m->h_rows, (size_t)3 * (c.max_seq_len + 1) * 4));
    int groups_area = 256;  // attention block size (PV partials reuse the score area)
    m->attn_smem = (size_t)(hd + (c.max_seq_len > groups_area ? c.max_seq_len : groups_area)) * 8;
    return IQ_OK;
}

// ---------------------------------------------------------------- the step

static int nccl_fail(ncclResult_t r) { return r == ncclSuccess ? IQ_OK : IQ_ERR_NCCL; }
#define IQ_NCCL(call) do { ncclResult_t _r = (call); if (_r != ncclSuccess) return nccl_fail(_r); } while (0)

// all-gather of a [B][w] local piece into out [B][P*w] (rank-major columns)
static int gather_rows(iq_model *m, const int64_t *local, int64_t *out, int B, int w) {
    const int P = m->sh.P;
    if (B == 1) {
        IQ_NCCL(ncclAllGather(local, out, (size_t)w, ncclInt64, m->comm, m->s));
        return IQ_OK;
    }
    IQ_NCCL(ncclAllGather(local, m->gath, (size_t)B * w, ncclInt64, m->comm, m->s));
    int64_t n = (int64_t)P * B * w;
    k_unshard<<<(int)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, m->s>>>(out, m->gath, P, B, w);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

static int add_into(iq_model *m, int64_t *x, const int64_t *y, int64_t n) {
    k_add<<<(int)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, m->s>>>(x, y, n);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

// Enqueues one forward pass over R rows: row r is token tok[r] of sequence
// seq[r] at position pos[r] (device arrays). Decode: R = B rows, one per
// sequence. Prefill: R = L rows of one sequence at positions 0..L-1 -- each
// row computes exactly what the reference's sequential llama_forward call at
// that position computes (causal attention per row).
// lm: 0 = LM head on every row (logits [R][V]); 1 = only the last row (prefill
// sampling, logits [1][V]); 2 = no LM head (an inner prefill chunk). decode != 0: argmax advances d_tok / d_pos and
// records the token in d_hist.
// tmax: a host-known bound on pos[r] + 1 over the rows (0 = unknown); short
// contexts (tmax <= att_short) take the single-kernel attention.
static int enqueue_rows(iq_model *m, int R, const int *tok, const int *pos, const int *seq, int lm, int decode,
                        int tmax = 0) {
    const iq_config &c = m->c;
    const Shard &S = m->sh;
    const bool tp = S.P > 1;
    const int d = c.hidden_dim, hd = c.head_dim;
    cudaStream_t s = m->s;
    int rc;
    auto proj = [&](int64_t *out, const Packed &P, const PackedTC &T, const int64_t *x, int rows,
                    int add) -> int {
        if (rows == 1) return launch_matvec_planes(out, P, x, s, add, m->racc);
        return launch_gemm_tc(out, T, x, rows, s, add, m->digits,
                              gemm_tc_part_bytes(T, rows) <= m->gpart_bytes ? m->gpart : nullptr);
    };
    // rmsnorm(x, nw) followed by a projection. A single row goes through the
    // packed matvec with the norm fused into its digit staging (each CTA
    // normalises x itself); several rows are normalised once into m->normed.
    auto norm_proj = [&](int64_t *out, const Packed &P, const PackedTC &T, const int64_t *x, const int64_t *nw,
                         int rows) -> int {
        if (rows == 1 && (size_t)8 * (P.Kp + 16) <= 100 * 1024)
            return launch_matvec_planes(out, P, x, s, 0, m->racc, nw);
        k_rmsnorm<<<rows, 256, 0, s>>>(m->normed, x, nw, d);
        IQ_CHECK_LAUNCH();
        return proj(out, P, T, m->normed, rows, 0);
    };
    // rmsnorm -> gate|up -> SwiGLU into act. One row: the matvec over the
    // pair-interleaved gate|up rows forms SwiGLU in its epilogue (no gu
    // round trip, one launch); several rows: GEMM into m->gu, then k_swiglu.
    auto norm_gu_swiglu = [&](int64_t *act, int l, const int64_t *x, const int64_t *nw, int rows) -> int {
        if (rows == 1 && S.it_l % 8 == 0) {
            if ((size_t)8 * (m->pgu[l].Kp + 16) <= 100 * 1024)
                return launch_matvec_planes(act, m->pgu[l], x, s, IQ_EPI_SWIGLU, m->racc, nw);
            k_rmsnorm<<<1, 256, 0, s>>>(m->normed, x, nw, d);
            IQ_CHECK_LAUNCH();
            return launch_matvec_planes(act, m->pgu[l], m->normed, s, IQ_EPI_SWIGLU, m->racc);
        }
        k_rmsnorm<<<rows, 256, 0, s>>>(m->normed, x, nw, d);
        IQ_CHECK_LAUNCH();
        int rc = proj(m->gu, m->pgu[l], m->tgu[l], m->normed, rows, 0);
        if (rc) return rc;
        k_swiglu<<<(rows * S.it_l + 255) / 256, 256, 0, s>>>(act, m->gu, S.it_l, rows);
        IQ_CHECK_LAUNCH();
        return IQ_OK;
    };
    k_embed<<<dim3((d + 255) / 256, R), 256, 0, s>>>(m->hidden, m->embed, tok, d);
    IQ_CHECK_LAUNCH();
    const int pairs = (S.nh_l + S.nkv_l) * (hd / 2) + m->kvd_l;
    int64_t *att_out = tp ? m->att_l : m->att;
    int64_t *act_out = tp ? m->act_l : m->act;
    for (int l = 0; l < c.num_layers; l++) {
        if ((rc = norm_proj(m->qkv, m->pqkv[l], m->tqkv[l], m->hidden, m->norm1[l], R))) return rc;
        const bool packed = m->kv_kbits > 0;
        // decode rows with short contexts: RoPE and the cache write happen inside
        // k_attention (one launch fewer per layer)
        const bool fused_rope = decode && !packed && tmax > 0 && tmax <= m->att_short;
        if (!fused_rope) {
            k_rope_kv<<<dim3((pairs + 255) / 256, R), 256, 0, s>>>(m->qkv, m->kc[l], m->vc[l], m->rcos, m->rsin,
                                                                   pos, seq, S.nh_l, S.nkv_l, hd, c.max_seq_len);
            IQ_CHECK_LAUNCH();
        }
        if (packed) {   // kv_pack_vector of the rows' K and V (the exact values stay unread)
            const int nwarp = R * S.nkv_l;
            k_kv_pack<<<(nwarp + 7) / 8, 256, 0, s>>>(m->kq[l], m->vq[l], m->kmag[l], m->vmag[l], m->kc[l], m->vc[l],
                                                     pos, seq, R, S.nkv_l, hd, c.max_seq_len, m->kv_kbits,
                                                     m->kv_vbits);
            IQ_CHECK_LAUNCH();
        }
        const KVView kview{m->kc[l], packed ? m->kq[l] : nullptr, nullptr, packed ? m->kmag[l] : nullptr,
                           m->kv_kbits, S.nkv_l, hd};
        const KVView vview{m->vc[l], nullptr, packed ? m->vq[l] : nullptr, packed ? m->vmag[l] : nullptr,
                           m->kv_vbits, S.nkv_l, hd};
        const bool att_short = !packed && tmax > 0 && tmax <= m->att_short;
        if (packed || (m->att_phased && !att_short)) {
            const int grid_t = (c.max_seq_len + ATT_TILE - 1) / ATT_TILE;
            int64_t n = (int64_t)R * S.nh_l * hd;
            k_attn_init<<<(int)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s>>>(att_out, m->amx, m->asum, R,
                                                                                   S.nh_l, hd);
            IQ_CHECK_LAUNCH();
            if (m->att_scores_tc)
                k_attn_scores_tc<<<dim3((c.max_seq_len + ATT_TC_POS - 1) / ATT_TC_POS, S.nkv_l, R), 256, 0, s>>>(
                    m->asc, m->amx, m->qkv, kview, pos, seq, S.nh_l, S.nkv_l, hd, c.max_seq_len, c.max_seq_len,
                    m->att_scale);
            else
                k_attn_scores<<<dim3(grid_t, S.nkv_l, R), 256, m->att_s1, s>>>(m->asc, m->amx, m->qkv, kview, pos,
                                                                                seq, S.nh_l, S.nkv_l, hd,
                                                                                c.max_seq_len, c.max_seq_len,
                                                                                m->att_scale);
            IQ_CHECK_LAUNCH();
            k_attn_exp<<<dim3((c.max_seq_len + 255) / 256, S.nh_l, R), 256, 0, s>>>(m->asc, m->amx, m->asum, pos,
                                                                                   S.nh_l, c.max_seq_len);
            IQ_CHECK_LAUNCH();
            const dim3 gpv(grid_t, S.nkv_l, R);
#define IQ_PV(SPT) k_attn_pv<SPT><<<gpv, 256, m->att_s3, s>>>(att_out, m->asc, m->asum, vview, pos, seq, S.nh_l, \
                                                          S.nkv_l, hd, c.max_seq_len, c.max_seq_len)
            const dim3 gtc((c.max_seq_len + PV_CH - 1) / PV_CH, S.nkv_l, R);
#define IQ_PVTC(SPT) k_attn_pv_tc<SPT><<<gtc, 256, m->att_s3tc, s>>>(att_out, m->asc, m->asum, vview, pos, seq, \
                                                                   S.nh_l, S.nkv_l, hd, c.max_seq_len, c.max_seq_len)
            if (m->att_pv_tc == 2) IQ_PVTC(2);
            else if (m->att_pv_tc == 1) IQ_PVTC(1);
#undef IQ_PVTC
            else switch (m->att_pv_spt) {
                case 1: IQ_PV(1); break;
                case 2: IQ_PV(2); break;
                case 4: IQ_PV(4); break;
                case 8: IQ_PV(8); break;
                default: IQ_PV(0);
            }
#undef IQ_PV
        } else if (m->gqa_smem && !att_short)
            k_attention_gqa<<<dim3(S.nh_l / m->hpc, R), 256, m->gqa_smem, s>>>(
                att_out, m->qkv, m->kc[l], m->vc[l], pos, seq, S.nh_l, S.nkv_l, hd, c.max_seq_len, c.max_seq_len,
                m->hpc);
        else if (fused_rope)
            k_attention<true><<<dim3(S.nh_l, R), 256, m->attn_smem, s>>>(att_out, m->qkv, m->kc[l], m->vc[l], pos,
                                                                         seq, S.nh_l, S.nkv_l, hd, c.max_seq_len,
                                                                         m->att_scale, m->rcos, m->rsin);
        else
            k_attention<false><<<dim3(S.nh_l, R), 256, m->attn_smem, s>>>(att_out, m->qkv, m->kc[l], m->vc[l], pos,
                                                                          seq, S.nh_l, S.nkv_l, hd, c.max_seq_len,
                                                                          m->att_scale, nullptr, nullptr);
        IQ_CHECK_LAUNCH();
        if (tp) {
            if ((rc = gather_rows(m, m->att_l, m->att, R, S.nh_l * hd))) return rc;
            if ((rc = proj(m->proj_l, m->po[l], m->to[l], m->att, R, 0))) return rc;
            if ((rc = gather_rows(m, m->proj_l, m->proj_full, R, S.d_l))) return rc;
            if ((rc = add_into(m, m->hidden, m->proj_full, (int64_t)R * d))) return rc;
        } else if ((rc = proj(m->hidden, m->po[l], m->to[l], m->att, R, 1))) {
            return rc;
        }
        if ((rc = norm_gu_swiglu(act_out, l, m->hidden, m->norm2[l], R))) return rc;
        if (tp) {
            if ((rc = gather_rows(m, m->act_l, m->act, R, S.it_l))) return rc;
            if ((rc = proj(m->proj_l, m->pdown[l], m->tdown[l], m->act, R, 0))) return rc;
            if ((rc = gather_rows(m, m->proj_l, m->proj_full, R, S.d_l))) return rc;
            if ((rc = add_into(m, m->hidden, m->proj_full, (int64_t)R * d))) return rc;
        } else if ((rc = proj(m->hidden, m->pdown[l], m->tdown[l], m->act, R, 1))) {
            return rc;
        }
    }
    if (lm == 2) return IQ_OK;                                  // no LM head wanted
    const int LR = lm ? 1 : R;                                  // rows through the LM head
    const int64_t *fin = m->hidden + (size_t)(R - LR) * d;   // the rows the LM head reads
    if (tp) {
        if ((rc = norm_proj(m->logits_l, m->plm, m->tlm, fin, m->fnorm, LR))) return rc;
        if (decode && !m->want_logits && !m->sampling) {
            // sharded argmax: each rank's first maximum, then (value, index) pairs
            k_argmax_local<<<LR, 1024, 0, s>>>(m->pairs_l, m->logits_l, S.v_l, S.r * S.v_l);
            IQ_CHECK_LAUNCH();
            IQ_NCCL(ncclAllGather(m->pairs_l, m->pairs_g, (size_t)LR * 2, ncclInt64, m->comm, s));
            k_argmax_pairs<<<(LR + 127) / 128, 128, 0, s>>>(m->d_arg, m->pairs_g, S.P, LR, m->d_tok, m->d_pos,
                                                          m->d_hist, c.max_seq_len + 1);
            IQ_CHECK_LAUNCH();
            return IQ_OK;
        }
        if ((rc = gather_rows(m, m->logits_l, m->logits, LR, S.v_l))) return rc;
    } else if ((rc = norm_proj(m->logits, m->plm, m->tlm, fin, m->fnorm, LR))) {
        return rc;
    }
    if (m->sampling) {   // sample_token with each sequence's parameters and generator
        if (decode)
            k_sample<<<LR, IQ_SAMPLE_THREADS, 0, s>>>(m->d_arg, m->logits, c.vocab_size, m->d_samp, 1, m->swork,
                                                      m->d_tok, m->d_pos, m->d_hist, c.max_seq_len + 1);
        else
            k_sample<<<1, IQ_SAMPLE_THREADS, 0, s>>>(m->d_arg, m->logits + (size_t)(LR - 1) * c.vocab_size,
                                                     c.vocab_size, m->d_samp + m->prefill_seq, 1, m->swork,
                                                     nullptr, nullptr, nullptr, 0);
    } else if (decode) {
        k_argmax<<<LR, 1024, 0, s>>>(m->d_arg, m->logits, c.vocab_size, m->d_tok, m->d_pos, m->d_hist,
                                     c.max_seq_len + 1);
    } else {
        k_argmax<<<1, 1024, 0, s>>>(m->d_arg, m->logits + (size_t)(LR - 1) * c.vocab_size, c.vocab_size,
                                    nullptr, nullptr, nullptr, 0);
    }
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

static void invalidate_exec(iq_model *m);

static int64_t ms_now() {
    return std::chrono::duration_cast<std::chrono::milliseconds>(
               std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Bounded wait: polls done() (1 finished, 0 pending, < 0 failed) and
// async_err() (a communicator error) until done, calling abort() on an
// asynchronous error or after timeout_ms without completion. Pure host logic
// (the callables are the CUDA / NCCL queries), so it is testable without a
// GPU (iq_selftest_watchdog).
template <class Done, class AsyncErr, class Abort, class Now>
static int watch_wait(Done done, AsyncErr async_err, Abort abort, Now now_ms, int64_t timeout_ms, int *polls) {
    const int64_t t0 = now_ms();
    for (int n = 1;; n++) {
        if (polls) *polls = n;
        const int d = done();
        if (d > 0) return IQ_OK;
        if (d < 0) return IQ_ERR_CUDA;
        if (async_err()) { abort(); return IQ_ERR_NCCL; }
        if (now_ms() - t0 > timeout_ms) { abort(); return IQ_ERR_TIMEOUT; }
        if (n > 64) std::this_thread::yield();
    }
}

// Host wait for the model's stream. Without tensor parallelism a plain
// synchronise. With it, a peer that stopped posting its half of a collective
// would block the NCCL kernels (and a plain synchronise) forever: the stream is
// polled together with NCCL's asynchronous error state, and an error or a wait
// beyond the model's timeout aborts the communicator (ncclCommAbort), which
// ends the pending collectives; the model is then marked failed and every
// later call returns IQ_ERR_STATE.
static int wait_stream(iq_model *m) {
    if (m->failed) return IQ_ERR_STATE;
    if (m->sh.P == 1 || !m->comm) {
        IQ_CUDA(cudaStreamSynchronize(m->s));
        return IQ_OK;
    }
    return watch_wait(
        [&]() {
            const cudaError_t e = cudaStreamQuery(m->s);
            if (e == cudaSuccess) return 1;
            if (e == cudaErrorNotReady) return 0;
            cuda_fail(e);
            return -1;
        },
        [&]() {
            ncclResult_t r = ncclSuccess;
            if (ncclCommGetAsyncError(m->comm, &r) != ncclSuccess) return true;
            return r != ncclSuccess && r != ncclInProgress;
        },
        [&]() {
            ncclCommAbort(m->comm);
            m->comm = nullptr;
            m->failed = true;
        },
        ms_now, m->timeout_ms, nullptr);
}
#define IQ_WAIT(m) do { int _w = wait_stream(m); if (_w) return _w; } while (0)

// Whether decode steps must leave the full logits in m->logits (only hashing
// callers need them under tensor parallelism; otherwise ranks exchange argmax
// pairs). Captured step graphs bake the choice in, so a change drops them.
static int set_want_logits(iq_model *m, bool want) {
    if (m->sh.P == 1 || m->want_logits == want) return IQ_OK;
    invalidate_exec(m);
    m->want_logits = want;
    return IQ_OK;
}

static MvView mv_view(const Packed &P) {
    return MvView{(const uint4 *)P.planes, packed_res(P), P.M, P.N, P.Kp};
}

// Prepares the persistent decode kernel when it applies: batch 1, no tensor
// parallelism, every decode matrix in the bf16 form (so one instantiation of
// the matvec serves all), SwiGLU fused (pair-interleaved gate|up) and the
// phased-attention scratch present. Must run outside stream capture.
static int dec_prepare(iq_model *m) {
    if (m->dec_ready || m->dec_mode == 0) return IQ_OK;
    const iq_config &c = m->c;
    const Shard &S = m->sh;
    if (m->max_batch != 1 || S.P != 1 || !m->att_phased || S.it_l % 8 || c.head_dim > 256 || m->kv_kbits)
        return IQ_OK;
    auto bf = [](const Packed &P) { return P.fmt == IQ_FMT_BF16 && (size_t)8 * (P.Kp + 16) <= 100 * 1024; };
    if (!bf(m->plm)) return IQ_OK;
    for (int l = 0; l < c.num_layers; l++)
        if (!bf(m->pqkv[l]) || !bf(m->po[l]) || !bf(m->pgu[l]) || !bf(m->pdown[l])) return IQ_OK;
    std::vector<DecLayer> hl(c.num_layers);
    size_t kmax = m->plm.Kp;
    for (int l = 0; l < c.num_layers; l++) {
        hl[l] = DecLayer{mv_view(m->pqkv[l]), mv_view(m->po[l]), mv_view(m->pgu[l]), mv_view(m->pdown[l]),
                         m->norm1[l], m->norm2[l], m->kc[l], m->vc[l]};
        for (const Packed *P : {&m->pqkv[l], &m->po[l], &m->pgu[l], &m->pdown[l]}) kmax = std::max(kmax, (size_t)P->Kp);
    }
    const int att_short = 256;
    const size_t hd = c.head_dim;
    m->dec_smem = std::max({(size_t)8 * (kmax + 16), (3 * hd + std::max<size_t>(att_short, IQ_DEC_THREADS)) * 8,
                            (2 * hd + DEC_TILE) * 8});
    IQ_CUDA(cudaFuncSetAttribute(k_decode_token, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->dec_smem));
    int occ = 0;
    IQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_decode_token, IQ_DEC_THREADS, m->dec_smem));
    if (occ < 1) return IQ_OK;
    static const int per_sm = getenv("IQ_DEC_PER_SM") ? atoi(getenv("IQ_DEC_PER_SM")) : 2;
    const int grid = dev_info().sms * std::max(1, std::min(occ, per_sm));
    if (!m->d_layers) DALLOC(m->d_layers, (size_t)c.num_layers * sizeof(DecLayer));
    IQ_CUDA(cudaMemcpy(m->d_layers, hl.data(), hl.size() * sizeof(DecLayer), cudaMemcpyHostToDevice));
    if (!m->bar) DALLOC(m->bar, sizeof(GridBar));
    IQ_CUDA(cudaMemset(m->bar, 0, sizeof(GridBar)));
    if (m->dec_grid < grid) {
        if (m->argv) cudaFree(m->argv);
        m->argv = nullptr;
        DALLOC(m->argv, (size_t)grid * 2 * sizeof(unsigned long long));
    }
    m->dec_grid = grid;
    DecParams &p = m->dec;
    p.L = c.num_layers; p.d = c.hidden_dim; p.nh = c.num_heads; p.nkv = c.num_kv_heads; p.hd = c.head_dim;
    p.inter = c.intermediate_dim; p.V = c.vocab_size; p.max_seq = c.max_seq_len; p.att_short = att_short;
    p.hist_stride = c.max_seq_len + 1;
    p.scale = m->att_scale;
    p.layers = m->d_layers;
    p.lm = mv_view(m->plm);
    p.embed = m->embed; p.fnorm = m->fnorm; p.rcos = m->rcos; p.rsin = m->rsin;
    p.hidden = m->hidden; p.qkv = m->qkv; p.att = m->att; p.act = m->act; p.logits = m->logits;
    p.racc = m->racc;
    p.asc = m->asc; p.amx = m->amx; p.asum = (unsigned long long *)m->asum; p.argv = m->argv;
    p.d_tok = m->d_tok; p.d_pos = m->d_pos; p.d_arg = m->d_arg; p.d_hist = m->d_hist;
    p.bar = m->bar;
    p.stamps = nullptr;
    p.prefetch = getenv("IQ_DEC_PREFETCH") ? atoi(getenv("IQ_DEC_PREFETCH")) : 1;
    if (getenv("IQ_DEC_STAMPS")) {   // profiling aid: barrier exit times of the last step
        static unsigned long long *st = nullptr;
        if (!st) DALLOC(st, 1024 * 8);
        p.stamps = st;
    }
    m->dec_ready = true;
    return IQ_OK;
}

static int enqueue_step(iq_model *m, int B, int tmax) {
    if (B == 1 && m->dec_ready && m->dec_mode) {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.gridDim = dim3((unsigned)m->dec_grid);
        cfg.blockDim = dim3(IQ_DEC_THREADS);
        cfg.dynamicSmemBytes = m->dec_smem;
        cfg.stream = m->s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        IQ_CUDA(cudaLaunchKernelEx(&cfg, k_decode_token, m->dec));
        return IQ_OK;
    }
    return enqueue_rows(m, B, m->d_tok, m->d_pos, m->d_seq, 0, 1, tmax);
}

// the decode-step graph for contexts up to tmax (0 = any length)
static cudaGraphExec_t &step_graph(iq_model *m, int tmax) {
    return tmax > 0 && tmax <= m->att_short ? m->graph_s : m->graph;
}
static int ensure_graph(iq_model *m, int tmax) {
    cudaGraphExec_t &gx = step_graph(m, tmax);
    if (gx) return IQ_OK;
    int prc = dec_prepare(m);   // outside the capture: it allocates and copies
    if (prc) return prc;
    const int tcap = tmax > 0 && tmax <= m->att_short ? m->att_short : 0;
    cudaGraph_t g;
    IQ_CUDA(cudaStreamBeginCapture(m->s, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m, m->max_batch, tcap);
    cudaError_t e = cudaStreamEndCapture(m->s, &g);
    if (rc) { if (e == cudaSuccess) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return cuda_fail(e);
    e = cudaGraphInstantiate(&gx, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e);
    return IQ_OK;
}

static bool model_ready(iq_model *m) {
    if (!m || !m->loaded_globals || m->failed) return false;
    for (bool b : m->loaded_layer) if (!b) return false;
    return true;
}

// Entry gate of every call that launches work: IQ_ERR_ARG / IQ_ERR_STATE as
// model_ready, and, under tensor parallelism, the host-side peer check before
// anything is enqueued: a rank that left between steps is found here, so no
// collective is ever launched towards it (IQ_ERR_NCCL; the model is failed).
static int model_gate(iq_model *m) {
    if (!m) return IQ_ERR_ARG;
    if (!model_ready(m)) return IQ_ERR_STATE;
    if (m->sh.P > 1 && m->peer_check && m->peer_check(m->peer_ctx)) {
        m->failed = true;
        return IQ_ERR_NCCL;
    }
    return IQ_OK;
}

// ----------------------------------------------------------- host helpers

static int h2d(void *dst, const void *src, size_t bytes) {
    IQ_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    return IQ_OK;
}

// Weights are about to change: captured step graphs and the persistent decode
// kernel's parameters hold pointers to the packed copies, so drop them.
static void invalidate_exec(iq_model *m) {
    cudaStreamSynchronize(m->s);
    if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }
    if (m->graph_s) { cudaGraphExecDestroy(m->graph_s); m->graph_s = nullptr; }
    m->dec_ready = false;
}

static int repack(iq_model *m, Packed *P, const int64_t *W, int M, int N) {
    if (P->planes) { IQ_CUDA(cudaStreamSynchronize(m->s)); free_packed(P); }
    int rc = pack_weights(W, M, N, m->s, P);
    if (rc) return rc;
    IQ_CUDA(cudaStreamSynchronize(m->s));
    return IQ_OK;
}
static int repack_tc(iq_model *m, PackedTC *P, const int64_t *W, int M, int N) {
    if (P->planes) { IQ_CUDA(cudaStreamSynchronize(m->s)); free_packed_tc(P); }
    int rc = pack_weights_tc(W, M, N, m->s, P);
    if (rc) return rc;
    IQ_CUDA(cudaStreamSynchronize(m->s));
    return IQ_OK;
}
// Packs layer l's projections in both formats, then frees its raw int64 copies.
static int repack_layer(iq_model *m, int l) {
    invalidate_exec(m);
    const iq_config &c = m->c;
    const Shard &S = m->sh;
    int rc, d = c.hidden_dim, it = c.intermediate_dim;
    if ((rc = repack(m, &m->pqkv[l], m->wqkv[l], m->qkv_rows, d))) return rc;
    if ((rc = repack(m, &m->po[l], m->wo[l], S.d_l, d))) return rc;
    if (S.it_l % 8) {  // no pair interleave: SwiGLU stays a separate kernel
        if ((rc = repack(m, &m->pgu[l], m->wgu[l], 2 * S.it_l, d))) return rc;
    } else {
        // the matvec form of gate|up is packed pair-interleaved (see k_interleave_pairs)
        int64_t *tmp = nullptr;
        const int64_t n = (int64_t)2 * S.it_l * d;
        IQ_CUDA(cudaMalloc(&tmp, (size_t)n * 8));
        k_interleave_pairs<<<(int)std::min<int64_t>((n + 255) / 256, 65535), 256, 0, m->s>>>(tmp, m->wgu[l], S.it_l,
                                                                                            d);
        cudaError_t e = cudaGetLastError();
        rc = e == cudaSuccess ? repack(m, &m->pgu[l], tmp, 2 * S.it_l, d) : cuda_fail(e);
        cudaStreamSynchronize(m->s);
        cudaFree(tmp);
        if (rc) return rc;
    }
    if ((rc = repack(m, &m->pdown[l], m->wdown[l], S.d_l, it))) return rc;
    if ((rc = repack_tc(m, &m->tqkv[l], m->wqkv[l], m->qkv_rows, d))) return rc;
    if ((rc = repack_tc(m, &m->to[l], m->wo[l], S.d_l, d))) return rc;
    if ((rc = repack_tc(m, &m->tgu[l], m->wgu[l], 2 * S.it_l, d))) return rc;
    if ((rc = repack_tc(m, &m->tdown[l], m->wdown[l], S.d_l, it))) return rc;
    free_raw_layer(m, l);
    return IQ_OK;
}
static int repack_lm(iq_model *m) {
    int rc;
    if ((rc = repack(m, &m->plm, m->lm, m->sh.v_l, m->c.hidden_dim))) return rc;
    if ((rc = repack_tc(m, &m->tlm, m->lm, m->sh.v_l, m->c.hidden_dim))) return rc;
    cudaFree(m->lm);
    m->lm = nullptr;
    return IQ_OK;
}

// Where each full host tensor's rows land on this rank: (first row, row count,
// device destination) pieces; the tensor has `cols` columns.
struct Piece { size_t row0, nrows; int64_t *dst; };
struct TensorPlan { std::string name; size_t rows, cols; bool ones; std::vector<Piece> pieces; };

static std::vector<TensorPlan> tensor_plan(iq_model *m) {
    const iq_config &c = m->c;
    const Shard &S = m->sh;
    const size_t d = c.hidden_dim, hd = c.head_dim, kvd = (size_t)c.num_kv_heads * hd, it = c.intermediate_dim,
                 V = c.vocab_size;
    std::vector<TensorPlan> t;
    t.push_back({"model.embed_tokens.weight", V, d, false, {{0, V, m->embed}}});
    t.push_back({"lm_head.weight", V, d, false, {{(size_t)S.r * S.v_l, (size_t)S.v_l, m->lm}}});
    t.push_back({"model.norm.weight", 1, d, true, {{0, 1, m->fnorm}}});
    char nm[160];
    for (int l = 0; l < c.num_layers; l++) {
        auto name = [&](const char *x) { snprintf(nm, sizeof nm, "model.layers.%d.%s.weight", l, x); return std::string(nm); };
        const size_t qr = (size_t)S.nh_l * hd, kr = (size_t)S.nkv_l * hd;
        int64_t *q = m->wqkv[l], *k = q + qr * d, *v = k + kr * d;
        t.push_back({name("input_layernorm"), 1, d, true, {{0, 1, m->norm1[l]}}});
        t.push_back({name("self_attn.q_proj"), d, d, false, {{(size_t)S.q_lo * hd, qr, q}}});
        t.push_back({name("self_attn.k_proj"), kvd, d, false, {{(size_t)S.kv_lo * hd, kr, k}}});
        t.push_back({name("self_attn.v_proj"), kvd, d, false, {{(size_t)S.kv_lo * hd, kr, v}}});
        t.push_back({name("self_attn.o_proj"), d, d, false, {{(size_t)S.r * S.d_l, (size_t)S.d_l, m->wo[l]}}});
        t.push_back({name("post_attention_layernorm"), 1, d, true, {{0, 1, m->norm2[l]}}});
        t.push_back({name("mlp.gate_proj"), it, d, false, {{(size_t)S.r * S.it_l, (size_t)S.it_l, m->wgu[l]}}});
        t.push_back({name("mlp.up_proj"), it, d, false,
                     {{(size_t)S.r * S.it_l, (size_t)S.it_l, m->wgu[l] + (size_t)S.it_l * d}}});
        t.push_back({name("mlp.down_proj"), d, it, false, {{(size_t)S.r * S.d_l, (size_t)S.d_l, m->wdown[l]}}});
    }
    return t;
}

static int upload_pieces(const TensorPlan &tp, const int64_t *full) {
    for (const Piece &p : tp.pieces) {
        int rc = h2d(p.dst, full + p.row0 * tp.cols, p.nrows * tp.cols * 8);
        if (rc) return rc;
    }
    return IQ_OK;
}


extern "C" {

IQ_API int iq_tp_shard_info(const iq_config *cfg, int tp_size, int tp_rank, int info[8]) {
    if (!cfg || !info) return IQ_ERR_ARG;
    Shard s;
    int rc = make_shard(*cfg, tp_size, tp_rank, &s);
    if (rc) return rc;
    int v[8] = {s.q_lo, s.nh_l, s.kv_lo, s.nkv_l, s.r * s.d_l, s.d_l, s.r * s.it_l, s.it_l};
    memcpy(info, v, sizeof v);
    return IQ_OK;
}

IQ_API int iq_nccl_unique_id(void *id_out) {
    if (!id_out) return IQ_ERR_ARG;
    ncclUniqueId id;
    IQ_NCCL(ncclGetUniqueId(&id));
    memcpy(id_out, &id, sizeof(id));
    return IQ_OK;
}

IQ_API int iq_model_create_tp(const iq_config *cfg, int max_batch, int device, int tp_rank, int tp_size,
                              const void *nccl_id, iq_model **out) {
    if (!cfg || !out || max_batch < 1 || tp_size < 1 || (tp_size > 1 && !nccl_id)) return IQ_ERR_ARG;
    *out = nullptr;
    const iq_config &c = *cfg;
    if (c.hidden_dim <= 0 || c.num_heads <= 0 || c.num_kv_heads <= 0 || c.head_dim <= 1 ||
        c.num_layers <= 0 || c.intermediate_dim <= 0 || c.vocab_size <= 0 || c.max_seq_len <= 0 ||
        c.num_heads % c.num_kv_heads != 0 || c.hidden_dim != c.num_heads * c.head_dim ||
        (c.head_dim & 1) || c.head_dim > 256)
        return IQ_ERR_ARG;
    Shard sh;
    int rc = make_shard(c, tp_size, tp_rank, &sh);
    if (rc) return rc;
    IQ_CUDA(cudaSetDevice(device));
    if ((rc = ensure_device_pub(device))) return rc;
    iq_model *m = new iq_model();
    m->c = c;
    m->sh = sh;
    m->dev = device;
    m->max_batch = max_batch;
    // activation rows: the decode batch, or a prefill chunk of up to 1024 positions
    m->rmax = std::max(max_batch, std::min(c.max_seq_len, 1024));
    cudaError_t e = cudaStreamCreateWithFlags(&m->s, cudaStreamNonBlocking);
    if (e != cudaSuccess) { delete m; return cuda_fail(e); }
    if ((rc = model_alloc(m))) { iq_model_destroy(m); return rc; }
    if (tp_size > 1) {
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof(id));
        if (ncclCommInitRank(&m->comm, tp_size, id, tp_rank) != ncclSuccess) {
            m->comm = nullptr;
            iq_model_destroy(m);
            return IQ_ERR_NCCL;
        }
    }
    {
        static int hpc_env = getenv("IQ_ATT_HPC") ? atoi(getenv("IQ_ATT_HPC")) : 1;
        int grpl = sh.nh_l / sh.nkv_l;
        m->hpc = (hpc_env >= 1 && grpl % hpc_env == 0) ? hpc_env : 1;
        const size_t grp = (size_t)m->hpc;
        size_t g = (grp * c.head_dim + grp * (size_t)c.max_seq_len + (size_t)ATT_TT * (c.head_dim + 1)) * 8;
        if (hpc_env >= 1 && g <= 200 * 1024) {
            e = cudaFuncSetAttribute(k_attention_gqa, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g);
            if (e != cudaSuccess) { iq_model_destroy(m); return cuda_fail(e); }
            m->gqa_smem = g;
        }
    }
    {
        static int att_env = getenv("IQ_ATT") ? atoi(getenv("IQ_ATT")) : 1;
        const size_t grp = (size_t)sh.nh_l / sh.nkv_l, hd = c.head_dim;
        m->att_s1 = att_scores_smem((int)grp, (int)hd);
        m->att_s3 = att_pv_smem((int)grp, (int)hd);
        m->att_pv_spt = getenv("IQ_PV_DIRECT") ? 0 : att_pv_spt((int)grp, (int)hd);
        m->att_scores_tc = !getenv("IQ_SCORES_DIRECT") && hd % 32 == 0 && hd <= 256;
        m->att_s3tc = att_pv_tc_smem((int)grp, (int)hd);
        m->att_pv_tc = getenv("IQ_PV_NOTC") || m->att_s3tc > 200 * 1024 ? 0 : att_pv_tc_hb((int)grp, (int)hd);
        // the phased scores use 32-bit limb dots, exact for head_dim <= 256
        m->att_phased = att_env == 1 && hd <= 256 && m->att_s1 <= 200 * 1024 && m->att_s3 <= 200 * 1024;
        if (m->att_phased) {
            size_t n = (size_t)m->rmax * sh.nh_l;
            if ((rc = dalloc((void **)&m->asc, n * c.max_seq_len * 8)) || (rc = dalloc((void **)&m->amx, n * 8)) ||
                (rc = dalloc((void **)&m->asum, n * 8))) { iq_model_destroy(m); return rc; }
            e = cudaFuncSetAttribute(k_attn_scores, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->att_s1);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(att_pv_kernel(m->att_pv_spt), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)m->att_s3);
            if (e == cudaSuccess && m->att_pv_tc)
                e = cudaFuncSetAttribute(att_pv_tc_kernel(m->att_pv_tc), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)m->att_s3tc);
            if (e != cudaSuccess) { iq_model_destroy(m); return cuda_fail(e); }
        }
    }
    if (!m->att_phased && !m->gqa_smem && m->attn_smem > 200 * 1024) { iq_model_destroy(m); return IQ_ERR_UNSUPPORTED; }
    if (m->attn_smem > 48 * 1024 && m->attn_smem <= 200 * 1024) {
        e = cudaFuncSetAttribute(k_attention<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->attn_smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attention<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->attn_smem);
        if (e != cudaSuccess) { iq_model_destroy(m); return cuda_fail(e); }
    }
    {
        // contexts up to this length use one CTA per (row, head): fewer launches
        // than the phased kernels and enough parallelism while T is short
        static int short_env = getenv("IQ_ATT_SHORT") ? atoi(getenv("IQ_ATT_SHORT")) : 384;
        m->att_short = m->attn_smem <= 200 * 1024 ? short_env : 0;
    }
    k_rope_init<<<256, 128, 0, m->s>>>(m->rcos, m->rsin, c.head_dim, c.max_seq_len, c.rope_theta);
    k_att_scale<<<1, 1, 0, m->s>>>(m->hidden, c.head_dim);  // hidden is scratch until reset
    e = cudaMemcpyAsync(&m->att_scale, m->hidden, 8, cudaMemcpyDeviceToHost, m->s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->s);
    if (e != cudaSuccess) { iq_model_destroy(m); return cuda_fail(e); }
    if ((rc = iq_model_reset(m))) { iq_model_destroy(m); return rc; }
    *out = m;
    return IQ_OK;
}

IQ_API int iq_model_config(const iq_model *m, iq_config *cfg) {
    if (!m || !cfg) return IQ_ERR_ARG;
    *cfg = m->c;
    return IQ_OK;
}

IQ_API int iq_model_create(const iq_config *cfg, int max_batch, int device, iq_model **out) {
    return iq_model_create_tp(cfg, max_batch, device, 0, 1, nullptr, out);
}

IQ_API int iq_model_destroy(iq_model *m) {
    if (!m) return IQ_ERR_ARG;
    cudaSetDevice(m->dev);
    if (m->failed && m->s) {
        // an aborted collective may still hold the stream: wait a bounded time;
        // if it never drains, the device buffers are left to the process exit
        // (cudaFree would wait for the device, i.e. forever)
        const int64_t t0 = ms_now();
        while (cudaStreamQuery(m->s) == cudaErrorNotReady && ms_now() - t0 < 10000)
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
        if (cudaStreamQuery(m->s) == cudaErrorNotReady) {
            delete m;
            return IQ_ERR_TIMEOUT;
        }
    }
    if (m->s) cudaStreamSynchronize(m->s);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    if (m->graph_s) cudaGraphExecDestroy(m->graph_s);
    if (m->comm) {
        if (m->failed) ncclCommAbort(m->comm);   // a peer left: no collective to complete
        else ncclCommDestroy(m->comm);
    }
    void *bufs[] = {m->embed, m->fnorm, m->lm, m->rcos, m->rsin, m->hidden, m->normed, m->qkv, m->att,
                    m->gu, m->act, m->logits, m->att_l, m->proj_l, m->act_l, m->logits_l, m->gath,
                    m->proj_full, m->d_tok, m->d_pos, m->d_arg, m->d_hist, m->racc, m->digits, m->gpart, m->asc, m->amx, m->asum, m->d_seq,
                    m->d_ptok, m->d_ppos, m->d_pseq, m->d_layers, m->bar, m->argv, m->pairs_l, m->pairs_g,
                    m->d_samp, m->swork};
    for (void *p : bufs) if (p) cudaFree(p);
    for (auto *v : {&m->norm1, &m->wqkv, &m->wo, &m->norm2, &m->wgu, &m->wdown, &m->kc, &m->vc, &m->kmag, &m->vmag})
        for (int64_t *p : *v) if (p) cudaFree(p);
    for (uint8_t *p : m->kq) if (p) cudaFree(p);
    for (uint16_t *p : m->vq) if (p) cudaFree(p);
    for (auto *v : {&m->pqkv, &m->po, &m->pgu, &m->pdown})
        for (Packed &P : *v) free_packed(&P);
    free_packed(&m->plm);
    for (auto *v : {&m->tqkv, &m->to, &m->tgu, &m->tdown})
        for (PackedTC &P : *v) free_packed_tc(&P);
    free_packed_tc(&m->tlm);
    if (m->h_pin) cudaFreeHost(m->h_pin);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->h_rows) cudaFreeHost(m->h_rows);
    if (m->s) cudaStreamDestroy(m->s);
    delete m;
    return IQ_OK;
}

IQ_API int iq_model_load_globals(iq_model *m, const int64_t *embed, const int64_t *final_norm,
                                 const int64_t *lm_head) {
    if (!m || !embed || !final_norm || !lm_head) return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(m->dev));
    invalidate_exec(m);
    if (!m->lm) DALLOC(m->lm, (size_t)m->sh.v_l * m->c.hidden_dim * 8);
    std::vector<TensorPlan> plan = tensor_plan(m);
    const int64_t *src[3] = {embed, lm_head, final_norm};
    int rc;
    for (int i = 0; i < 3; i++)
        if ((rc = upload_pieces(plan[i], src[i]))) return rc;
    if ((rc = repack_lm(m))) return rc;
    m->loaded_globals = true;
    return IQ_OK;
}

IQ_API int iq_model_load_layer(iq_model *m, int l, const int64_t *const w[9]) {
    if (!m || !w || l < 0 || l >= m->c.num_layers) return IQ_ERR_ARG;
    for (int i = 0; i < 9; i++) if (!w[i]) return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(m->dev));
    int rc;
    if ((rc = alloc_raw_layer(m, l))) return rc;
    std::vector<TensorPlan> plan = tensor_plan(m);
    for (int i = 0; i < 9; i++)
        if ((rc = upload_pieces(plan[3 + 9 * l + i], w[i]))) return rc;
    if ((rc = repack_layer(m, l))) return rc;
    m->loaded_layer[l] = true;
    return IQ_OK;
}

IQ_API int iq_model_reset(iq_model *m) {
    if (!m) return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(m->dev));
    size_t kvb = (size_t)m->max_batch * m->c.max_seq_len * m->kvd_l * 8;
    for (int l = 0; l < m->c.num_layers; l++) {
        IQ_CUDA(cudaMemsetAsync(m->kc[l], 0, kvb, m->s));
        IQ_CUDA(cudaMemsetAsync(m->vc[l], 0, kvb, m->s));
    }
    if (m->kv_kbits) {   // kv_cache_reset also clears the packed arrays (llama_int.c:1160-1172)
        const size_t ne = (size_t)m->max_batch * m->c.max_seq_len * m->kvd_l;
        const size_t nv = (size_t)m->max_batch * m->c.max_seq_len * m->sh.nkv_l;
        for (int l = 0; l < m->c.num_layers; l++) {
            IQ_CUDA(cudaMemsetAsync(m->kq[l], 0, ne, m->s));
            IQ_CUDA(cudaMemsetAsync(m->vq[l], 0, ne * 2, m->s));
            IQ_CUDA(cudaMemsetAsync(m->kmag[l], 0, nv * 8, m->s));
            IQ_CUDA(cudaMemsetAsync(m->vmag[l], 0, nv * 8, m->s));
        }
    }
    // a persistent decode kernel that gave up on a barrier left it abandoned
    if (m->bar) IQ_CUDA(cudaMemsetAsync(m->bar, 0, sizeof(GridBar), m->s));
    IQ_CUDA(cudaStreamSynchronize(m->s));
    return IQ_OK;
}

// Synthetic weights: the global tensors, then layer by layer (generate on host
// threads, upload this rank's rows, pack, free the raw copies), so the device
// never holds more than one layer of raw int64 weights.
static int synth_jobs(iq_model *m, const std::vector<TensorPlan> &plan, size_t j0, size_t j1, int config_index,
                      int threads) {
    std::atomic<size_t> next(j0);
    std::atomic<int> status(IQ_OK);
    auto worker = [&]() {
        cudaSetDevice(m->dev);
        std::vector<int64_t> buf;
        for (;;) {
            size_t j = next.fetch_add(1);
            if (j >= j1 || status.load() != IQ_OK) return;
            const TensorPlan &tp = plan[j];
            size_t n = tp.rows * tp.cols;
            buf.resize(n);
            if (tp.ones) std::fill(buf.begin(), buf.end(), IQ_ONE);
            else iq_synth_weights(iq_tensor_seed(config_index, tp.name.c_str()), buf.data(), (int64_t)n);
            int rc = upload_pieces(tp, buf.data());
            if (rc) status.store(rc);
        }
    };
    int nt = (int)std::min<size_t>((size_t)threads, j1 - j0);
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; t++) pool.emplace_back(worker);
    for (auto &t : pool) t.join();
    return status.load();
}

IQ_API int iq_model_synth(iq_model *m, int config_index, int threads) {
    if (!m) return IQ_ERR_ARG;
    if (threads < 1) threads = 1;
    IQ_CUDA(cudaSetDevice(m->dev));
    if (!m->lm) DALLOC(m->lm, (size_t)m->sh.v_l * m->c.hidden_dim * 8);
    int rc;
    for (int l = 0; l < m->c.num_layers; l++)
        if (!m->norm1[l] && (rc = alloc_raw_layer(m, l))) return rc;
    std::vector<TensorPlan> plan = tensor_plan(m);  // norms and globals are stable pointers
    if ((rc = synth_jobs(m, plan, 0, 3, config_index, threads))) return rc;
    if ((rc = repack_lm(m))) return rc;
    for (int l = 0; l < m->c.num_layers; l++) {
        if ((rc = alloc_raw_layer(m, l))) return rc;
        plan = tensor_plan(m);
        if ((rc = synth_jobs(m, plan, 3 + 9 * (size_t)l, 3 + 9 * (size_t)(l + 1), config_index, threads))) return rc;
        if ((rc = repack_layer(m, l))) return rc;
    }
    m->loaded_globals = true;
    m->loaded_layer.assign(m->c.num_layers, true);
    return IQ_OK;
}

// ------------------------------------------------------------- forward

static int set_tok_pos(iq_model *m, const int *tok, const int *pos, int B, int slot) {
    // distinct pinned slots so that queued copies never see a later overwrite
    int *h = m->h_pin + m->max_batch + 16 + (size_t)slot * 2 * m->max_batch;
    for (int b = 0; b < B; b++) { h[b] = tok[b]; h[m->max_batch + b] = pos[b]; }
    IQ_CUDA(cudaMemcpyAsync(m->d_tok, h, (size_t)B * 4, cudaMemcpyHostToDevice, m->s));
    IQ_CUDA(cudaMemcpyAsync(m->d_pos, h + m->max_batch, (size_t)B * 4, cudaMemcpyHostToDevice, m->s));
    return IQ_OK;
}

// Enqueues the prefill of sequence sq: prompt positions 0..L-1 in chunks of up
// to rmax rows. hash_logits: LM head on every row and the logits of every
// position appended to *hv in order; otherwise only the last row's logits.
// Ends with the sequence's decode state at position L (k_prefill_done).
static int enqueue_prefill(iq_model *m, int sq, const int *prompt, int L, std::vector<int64_t> *hv) {
    int *h = m->h_rows;
    m->prefill_seq = sq;
    for (int p = 0; p < L; p++) { h[p] = prompt[p]; h[L + p] = p; h[2 * L + p] = sq; }
    int rc;
    for (int p0 = 0; p0 < L; p0 += m->rmax) {
        const int n = std::min(m->rmax, L - p0);
        const bool last = p0 + n == L;
        IQ_CUDA(cudaMemcpyAsync(m->d_ptok, h + p0, (size_t)n * 4, cudaMemcpyHostToDevice, m->s));
        IQ_CUDA(cudaMemcpyAsync(m->d_ppos, h + L + p0, (size_t)n * 4, cudaMemcpyHostToDevice, m->s));
        IQ_CUDA(cudaMemcpyAsync(m->d_pseq, h + 2 * L + p0, (size_t)n * 4, cudaMemcpyHostToDevice, m->s));
        if ((rc = enqueue_rows(m, n, m->d_ptok, m->d_ppos, m->d_pseq, hv ? 0 : (last ? 1 : 2), 0))) return rc;
        if (hv) {
            size_t old = hv->size(), cnt = (size_t)n * m->c.vocab_size;
            hv->resize(old + cnt);
            IQ_CUDA(cudaMemcpyAsync(hv->data() + old, m->logits, cnt * 8, cudaMemcpyDeviceToHost, m->s));
        }
        // the pinned row arrays are reused by the next chunk only after these copies ran
        IQ_WAIT(m);
    }
    k_prefill_done<<<1, 32, 0, m->s>>>(m->d_arg, m->d_tok, m->d_pos, m->d_hist, m->c.max_seq_len + 1, sq, L);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

IQ_API int iq_forward(iq_model *m, int token, int pos, int64_t *logits, int *argmax_out) {
    if (int g_ = model_gate(m)) return g_;
    if (token < 0 || token >= m->c.vocab_size || pos < 0 || pos >= m->c.max_seq_len) return IQ_ERR_RANGE;
    IQ_CUDA(cudaSetDevice(m->dev));
    IQ_WAIT(m);
    int rc;
    int *h = m->h_rows;
    h[0] = token; h[1] = pos; h[2] = 0;
    IQ_CUDA(cudaMemcpyAsync(m->d_ptok, h, 4, cudaMemcpyHostToDevice, m->s));
    IQ_CUDA(cudaMemcpyAsync(m->d_ppos, h + 1, 4, cudaMemcpyHostToDevice, m->s));
    IQ_CUDA(cudaMemcpyAsync(m->d_pseq, h + 2, 4, cudaMemcpyHostToDevice, m->s));
    if ((rc = enqueue_rows(m, 1, m->d_ptok, m->d_ppos, m->d_pseq, 0, 0, pos + 1))) return rc;
    if (logits) IQ_CUDA(cudaMemcpyAsync(m->h_logits, m->logits, (size_t)m->c.vocab_size * 8, cudaMemcpyDeviceToHost, m->s));
    IQ_CUDA(cudaMemcpyAsync(m->h_pin, m->d_arg, 4, cudaMemcpyDeviceToHost, m->s));
    IQ_WAIT(m);
    if (logits) memcpy(logits, m->h_logits, (size_t)m->c.vocab_size * 8);
    if (argmax_out) *argmax_out = m->h_pin[0];
    return take_dev_error();
}

static uint64_t fnv_mix(uint64_t h, const int64_t *v, size_t n) {
    for (size_t i = 0; i < n; i++) {
        uint64_t u = (uint64_t)v[i];
        for (int b = 0; b < 8; b++) { h ^= u & 0xff; h *= 1099511628211ULL; u >>= 8; }
    }
    return h;
}

// one step for B sequences whose positions are all below tmax: a captured
// graph when B == max_batch
static int run_step(iq_model *m, int B, int tmax) {
    if (B == m->max_batch) {
        int rc = ensure_graph(m, tmax);
        if (rc) return rc;
        IQ_CUDA(cudaGraphLaunch(step_graph(m, tmax), m->s));
        return IQ_OK;
    }
    return enqueue_step(m, B, tmax);
}

IQ_API int iq_generate(iq_model *m, const int *prompt, int plen, int max_new, int *out, int *n_out,
                       uint64_t *logit_hash) {
    if (!m || !prompt || !out || !n_out || plen < 1 || max_new < 1) return IQ_ERR_ARG;
    if (int g_ = model_gate(m)) return g_;
    const iq_config &c = m->c;
    *n_out = -1;
    for (int i = 0; i < plen; i++)
        if (prompt[i] < 0 || prompt[i] >= c.vocab_size) return IQ_ERR_RANGE;  // llama_int.c:2813
    if (plen > c.max_seq_len) return IQ_ERR_RANGE;                          // llama_int.c:2817
    int rc;
    if ((rc = iq_model_reset(m))) return rc;
    const bool hash = logit_hash != nullptr;
    const int V = c.vocab_size;
    uint64_t h = 1469598103934665603ULL;
    if ((rc = set_want_logits(m, hash || m->sampling))) return rc;
    memcpy(out, prompt, (size_t)plen * sizeof(int));
    // prefill: every prompt position in batched rows (== the M=1 loop of llama_int.c:3081-3092)
    std::vector<int64_t> hv;
    if ((rc = enqueue_prefill(m, 0, prompt, plen, hash ? &hv : nullptr))) return rc;
    if (hash) h = fnv_mix(h, hv.data(), hv.size());
    int total = plen;
    // decode positions plen .. ; the reference stops when pos reaches max_seq_len
    const int steps = std::min(max_new - 1, c.max_seq_len - plen);
    if (hash) {
        IQ_CUDA(cudaMemcpyAsync(m->h_pin, m->d_tok, 4, cudaMemcpyDeviceToHost, m->s));
        IQ_WAIT(m);
        out[total++] = m->h_pin[0];  // prefill's sample is appended unconditionally
        for (int i = 1; i <= steps; i++) {
            if ((rc = run_step(m, 1, plen + i))) return rc;  // d_tok / d_pos advanced on the device
            IQ_CUDA(cudaMemcpyAsync(m->h_logits, m->logits, (size_t)V * 8, cudaMemcpyDeviceToHost, m->s));
            IQ_CUDA(cudaMemcpyAsync(m->h_pin, m->d_arg, 4, cudaMemcpyDeviceToHost, m->s));
            IQ_WAIT(m);
            h = fnv_mix(h, m->h_logits, V);
            const int nx = m->h_pin[0];
            if (nx == 2) break;  // LLAMA_EOS (llama_int.c:3046, 3110)
            out[total++] = nx;
        }
        *logit_hash = h;
    } else {
        for (int i = 1; i <= steps; i++)
            if ((rc = run_step(m, 1, plen + i))) return rc;
        std::vector<int> hist(steps + 1);
        IQ_CUDA(cudaMemcpyAsync(hist.data(), m->d_hist + plen, (size_t)(steps + 1) * 4, cudaMemcpyDeviceToHost, m->s));
        IQ_WAIT(m);
        out[total++] = hist[0];
        for (int i = 1; i <= steps; i++) {
            if (hist[i] == 2) break;
            out[total++] = hist[i];
        }
    }
    *n_out = total;
    return take_dev_error();
}

IQ_API int iq_generate_sampled(iq_model *m, const int *prompt, int plen, int max_new, int64_t temperature,
                               int top_k, int64_t top_p, uint64_t seed, int *out, int *n_out, uint64_t *logit_hash) {
    if (int g_ = model_gate(m)) return g_;
    IQ_CUDA(cudaSetDevice(m->dev));
    SampleState st{};
    st.temperature = temperature;
    st.top_k = top_k;
    st.top_p = top_p;
    uint64_t rs[2];
    iq_rng_seed(seed, rs);   // rng_seed once per generation (llama_int.c:4783-4789)
    st.s0 = rs[0];
    st.s1 = rs[1];
    IQ_WAIT(m);
    IQ_CUDA(cudaMemcpy(m->d_samp, &st, sizeof(st), cudaMemcpyHostToDevice));
    invalidate_exec(m);   // the step graphs bake in argmax or sampling
    m->sampling = true;
    int rc = iq_generate(m, prompt, plen, max_new, out, n_out, logit_hash);
    invalidate_exec(m);
    m->sampling = false;
    return rc;
}

IQ_API int iq_generate_batch(iq_model *m, const int *prompts, int plen, int max_new, int *out, int *n_out,
                             uint64_t *logit_hashes) {
    if (!m || !prompts || !out || !n_out || plen < 1 || max_new < 1) return IQ_ERR_ARG;
    if (int g_ = model_gate(m)) return g_;
    const iq_config &c = m->c;
    const int B = m->max_batch;
    for (int i = 0; i < B * plen; i++)
        if (prompts[i] < 0 || prompts[i] >= c.vocab_size) return IQ_ERR_RANGE;
    if (plen > c.max_seq_len) return IQ_ERR_RANGE;
    int rc;
    if ((rc = iq_model_reset(m))) return rc;
    const bool hash = logit_hashes != nullptr;
    const int V = c.vocab_size;
    std::vector<int64_t> hv;
    if ((rc = set_want_logits(m, hash))) return rc;
    for (int b = 0; b < B; b++) {  // each sequence's prompt as batched rows
        if ((rc = enqueue_prefill(m, b, prompts + (size_t)b * plen, plen, hash ? &hv : nullptr))) return rc;
        if (hash) {
            logit_hashes[b] = fnv_mix(1469598103934665603ULL, hv.data(), hv.size());
            hv.clear();
        }
    }
    const int steps = std::min(max_new - 1, c.max_seq_len - plen);
    std::vector<int64_t> lg;
    std::vector<int> argm, live(B, 1);
    if (hash) { lg.resize((size_t)B * V); argm.resize(B); }
    for (int i = 1; i <= steps; i++) {
        if ((rc = run_step(m, B, plen + i))) return rc;
        if (!hash) continue;
        // every sequence's logits of this step enter its hash until (and
        // including) the step that samples EOS, as the reference's loop forwards
        IQ_CUDA(cudaMemcpyAsync(lg.data(), m->logits, lg.size() * 8, cudaMemcpyDeviceToHost, m->s));
        IQ_CUDA(cudaMemcpyAsync(argm.data(), m->d_arg, (size_t)B * 4, cudaMemcpyDeviceToHost, m->s));
        IQ_WAIT(m);
        for (int b = 0; b < B; b++) {
            if (!live[b]) continue;
            logit_hashes[b] = fnv_mix(logit_hashes[b], lg.data() + (size_t)b * V, V);
            if (argm[b] == 2) live[b] = 0;
        }
    }
    const int stride = c.max_seq_len + 1;
    std::vector<int> hist((size_t)B * stride);
    IQ_CUDA(cudaMemcpyAsync(hist.data(), m->d_hist, hist.size() * 4, cudaMemcpyDeviceToHost, m->s));
    IQ_WAIT(m);
    const int ow = plen + max_new;
    for (int b = 0; b < B; b++) {
        int *o = out + (size_t)b * ow;
        memcpy(o, prompts + (size_t)b * plen, (size_t)plen * 4);
        int total = plen;
        o[total++] = hist[(size_t)b * stride + plen];
        for (int i = 1; i <= steps; i++) {
            int t = hist[(size_t)b * stride + plen + i];
            if (t == 2) break;
            o[total++] = t;
        }
        n_out[b] = total;
    }
    return take_dev_error();
}

IQ_API int iq_model_set_attention(iq_model *m, int short_max) {
    if (!m || short_max < 0) return IQ_ERR_ARG;
    if (short_max > 0 && m->attn_smem > 200 * 1024) return IQ_ERR_UNSUPPORTED;
    IQ_CUDA(cudaSetDevice(m->dev));
    IQ_CUDA(cudaStreamSynchronize(m->s));
    if (m->graph_s) { cudaGraphExecDestroy(m->graph_s); m->graph_s = nullptr; }
    m->att_short = short_max;
    return IQ_OK;
}

IQ_API int iq_sample_dev(const int64_t *d_logits, int rows, int V, int64_t temperature, int top_k, int64_t top_p,
                         uint64_t *rng, int *out) {
    if (!d_logits || rows < 1 || V < 1 || !rng || !out) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    std::vector<SampleState> h(rows);
    for (int r = 0; r < rows; r++) {
        h[r].temperature = temperature;
        h[r].top_k = top_k;
        h[r].top_p = top_p;
        h[r].s0 = rng[2 * r];
        h[r].s1 = rng[2 * r + 1];
    }
    SampleState *d_st = nullptr;
    int64_t *work = nullptr;
    int *d_out = nullptr;
    cudaStream_t s = lib_stream();
    cudaError_t e = cudaMalloc(&d_st, rows * sizeof(SampleState));
    if (e == cudaSuccess) e = cudaMalloc(&work, (size_t)rows * V * 8);
    if (e == cudaSuccess) e = cudaMalloc(&d_out, rows * sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_st, h.data(), rows * sizeof(SampleState), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        k_sample<<<rows, IQ_SAMPLE_THREADS, 0, s>>>(d_out, d_logits, V, d_st, 1, work, nullptr, nullptr, nullptr, 0);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, d_out, rows * sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h.data(), d_st, rows * sizeof(SampleState), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(d_st);
    cudaFree(work);
    cudaFree(d_out);
    if (e != cudaSuccess) return cuda_fail(e);
    for (int r = 0; r < rows; r++) { rng[2 * r] = h[r].s0; rng[2 * r + 1] = h[r].s1; }
    return IQ_OK;
}

IQ_API int iq_model_set_kv_packed(iq_model *m, int k_bits, int v_bits) {
    if (!m) return IQ_ERR_ARG;
    const bool off = k_bits == 0 && v_bits == 0;
    if (!off && (k_bits < 1 || k_bits > 8 || v_bits < 1 || v_bits > 16)) return IQ_ERR_ARG;  // llama_int.c:4742-4747
    if (!off && !m->att_phased) return IQ_ERR_UNSUPPORTED;
    IQ_CUDA(cudaSetDevice(m->dev));
    invalidate_exec(m);
    if (!off && m->kq.empty()) {
        const size_t ne = (size_t)m->max_batch * m->c.max_seq_len * m->kvd_l;
        const size_t nv = (size_t)m->max_batch * m->c.max_seq_len * m->sh.nkv_l;
        const int L = m->c.num_layers;
        m->kq.assign(L, nullptr);
        m->vq.assign(L, nullptr);
        m->kmag.assign(L, nullptr);
        m->vmag.assign(L, nullptr);
        for (int l = 0; l < L; l++) {
            DALLOC(m->kq[l], ne);
            DALLOC(m->vq[l], ne * 2);
            DALLOC(m->kmag[l], nv * 8);
            DALLOC(m->vmag[l], nv * 8);
        }
    }
    m->kv_kbits = k_bits;
    m->kv_vbits = v_bits;
    return iq_model_reset(m);
}

IQ_API int iq_model_set_peer_check(iq_model *m, int (*fn)(void *ctx), void *ctx) {
    if (!m) return IQ_ERR_ARG;
    m->peer_check = fn;
    m->peer_ctx = ctx;
    return IQ_OK;
}

IQ_API int iq_model_set_timeout(iq_model *m, int64_t ms) {
    if (!m || ms < 1) return IQ_ERR_ARG;
    m->timeout_ms = ms;
    return IQ_OK;
}

// The bounded-wait logic of tensor-parallel steps on scripted events (no GPU):
// scenario 0 completes at the third poll; 1 reports a communicator error at
// the second; 2 never completes (a simulated clock advances 10 ms per poll,
// limit 100 ms); 3 fails the stream query.
IQ_API int iq_selftest_watchdog(int scenario, int *aborted, int *polls) {
    if (!aborted || !polls || scenario < 0 || scenario > 3) return IQ_ERR_ARG;
    int n = 0;
    int64_t clock = 0;
    *aborted = 0;
    return watch_wait(
        [&]() { n++; return scenario == 3 ? -1 : (scenario == 0 && n >= 3) ? 1 : 0; },
        [&]() { return scenario == 1 && n >= 2; },
        [&]() { (*aborted)++; },
        [&]() { clock += 10; return clock; }, 100, polls);
}

IQ_API int iq_model_set_decode(iq_model *m, int mode) {
    if (!m || mode < 0 || mode > 1) return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(m->dev));
    invalidate_exec(m);
    m->dec_mode = mode;
    return IQ_OK;
}

// Diagnostic: microseconds per grid barrier of the persistent decode kernel
// (k_bar_bench) with `grid` co-resident CTAs of 256 threads (mode must be 0).
IQ_API int iq_bench_grid_sync(int grid, int iters, int mode, float *us) {
    if (grid < 1 || iters < 1 || mode != 0 || !us) return IQ_ERR_ARG;
    int dev, rc;
    if ((rc = cur_device(&dev))) return rc;
    GridBar *b = nullptr;
    IQ_CUDA(cudaMalloc(&b, sizeof(GridBar)));
    cudaMemset(b, 0, sizeof(GridBar));
    void (*k)(GridBar *, int) = k_bar_bench;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.stream = lib_stream();
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaError_t e = cudaLaunchKernelEx(&cfg, k, b, 10);
    if (e == cudaSuccess) e = cudaEventRecord(e0, lib_stream());
    if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, k, b, iters);
    if (e == cudaSuccess) e = cudaEventRecord(e1, lib_stream());
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFree(b);
    if (e != cudaSuccess) return cuda_fail(e);
    *us = ms * 1000.0f / iters;
    return take_dev_error();
}

// Profiling aid (IQ_DEC_STAMPS set): copies the last persistent step's barrier
// exit times (ns since its start) into out[n], returns the count.
IQ_API int iq_model_decode_stamps(iq_model *m, int64_t *out, int n) {
    if (!m || !out || n < 1 || !m->dec_ready || !m->dec.stamps) return IQ_ERR_STATE;
    unsigned long long h[1024];
    IQ_CUDA(cudaStreamSynchronize(m->s));
    IQ_CUDA(cudaMemcpy(h, m->dec.stamps, sizeof(h), cudaMemcpyDeviceToHost));
    const int cnt = (int)std::min<unsigned long long>(h[0], std::min(n, 1022));
    const unsigned long long mask = (1ull << 56) - 1;
    for (int i = 0; i < cnt; i++) out[i] = (int64_t)(((h[2 + i] >> 56) << 56) | ((h[2 + i] & mask) - h[1]));
    // slots 400.. / 700..: per matvec phase, the latest staging end / loop end over all warps
    if (n >= 1024)
        for (int i = 400; i < 1000; i++) out[i] = h[i] ? (int64_t)((h[i] & mask) - h[1]) : 0;
    return cnt;
}

IQ_API int iq_model_decode_info(iq_model *m, int *persistent, int *grid) {
    if (!m || !persistent || !grid) return IQ_ERR_ARG;
    if (int g_ = model_gate(m)) return g_;
    IQ_CUDA(cudaSetDevice(m->dev));
    int rc = dec_prepare(m);
    if (rc) return rc;
    *persistent = m->dec_ready && m->dec_mode ? 1 : 0;
    *grid = *persistent ? m->dec_grid : 0;
    return IQ_OK;
}

IQ_API int iq_model_weight_bytes(iq_model *m, int64_t *decode_bytes, int64_t *gemm_bytes) {
    if (!m || !decode_bytes || !gemm_bytes) return IQ_ERR_ARG;
    if (int g_ = model_gate(m)) return g_;
    int64_t d = packed_bytes(m->plm), g = 0;
    for (const std::vector<Packed> *v : {&m->pqkv, &m->po, &m->pgu, &m->pdown})
        for (const Packed &P : *v) d += packed_bytes(P);
    for (const std::vector<PackedTC> *v : {&m->tqkv, &m->to, &m->tgu, &m->tdown})
        for (const PackedTC &P : *v) g += (int64_t)P.np * P.Mpad * P.Kpad + 16 * (int64_t)P.Mpad;
    g += (int64_t)m->tlm.np * m->tlm.Mpad * m->tlm.Kpad + 16 * (int64_t)m->tlm.Mpad;
    *decode_bytes = d;
    *gemm_bytes = g;
    return IQ_OK;
}

IQ_API int iq_decode_steps_timed(iq_model *m, int pos0, int steps, float *ms) {
    if (!m || !ms || steps < 1 || pos0 < 0 || pos0 + steps > m->c.max_seq_len) return IQ_ERR_ARG;
    if (int g_ = model_gate(m)) return g_;
    IQ_CUDA(cudaSetDevice(m->dev));
    int rc;
    std::vector<int> tok(m->max_batch), pos(m->max_batch, pos0);
    IQ_WAIT(m);
    IQ_CUDA(cudaMemcpy(tok.data(), m->d_tok, tok.size() * 4, cudaMemcpyDeviceToHost));
    if ((rc = set_tok_pos(m, tok.data(), pos.data(), m->max_batch, 0))) return rc;
    if ((rc = ensure_graph(m, pos0 + 1)) || (rc = ensure_graph(m, pos0 + steps))) return rc;
    cudaEvent_t e0, e1;
    IQ_CUDA(cudaEventCreate(&e0));
    IQ_CUDA(cudaEventCreate(&e1));
    IQ_CUDA(cudaEventRecord(e0, m->s));
    for (int i = 0; i < steps; i++) IQ_CUDA(cudaGraphLaunch(step_graph(m, pos0 + i + 1), m->s));
    IQ_CUDA(cudaEventRecord(e1, m->s));
    IQ_WAIT(m);
    IQ_CUDA(cudaEventElapsedTime(ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return IQ_OK;
}

}  // extern "C"
