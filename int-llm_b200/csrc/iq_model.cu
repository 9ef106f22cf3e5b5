// iq_model.cu -- device-resident integer Llama model: weights, RoPE tables,
// exact int64 KV cache and the decode step (llama_forward, llama_int.c:2807-2886)
// built from the kernels in iq_layer.cuh, captured once into a CUDA graph and
// replayed per token; greedy generate (llama_int.c:3067-3135) on top.
//
// Per layer the step is 7 launches:
//   rmsnorm -> QKV matvec (q|k|v rows fused, exact: rows are independent)
//   -> RoPE + KV write -> attention -> O matvec (+= residual)
//   -> rmsnorm -> gate|up matvec (fused rows) -> SwiGLU -> down matvec (+= residual)
// then final rmsnorm, LM head matvec and argmax.
#include <cstring>
#include <thread>
#include <atomic>
#include <string>
#include <algorithm>
#include <cstdio>
#include <vector>
#include "iq_common.cuh"
#include "iq_layer.cuh"


using namespace iq;

struct iq_model {
    iq_config c;
    int dev = 0;
    int max_batch = 1;
    int kvd = 0, qkv_rows = 0;
    cudaStream_t s = nullptr;
    // weights
    int64_t *embed = nullptr, *fnorm = nullptr, *lm = nullptr;
    std::vector<int64_t *> norm1, wqkv, wo, norm2, wgu, wdown;
    std::vector<int64_t *> kc, vc;  // per layer [B][max_seq][kvd]
    int64_t *rcos = nullptr, *rsin = nullptr;
    // activations (device)
    int64_t *hidden = nullptr, *normed = nullptr, *qkv = nullptr, *att = nullptr, *gu = nullptr,
            *act = nullptr, *logits = nullptr;
    int *d_tok = nullptr, *d_pos = nullptr, *d_arg = nullptr, *d_hist = nullptr;
    // byte-plane packed copies of every projection (M=1 decode path)
    std::vector<Packed> pqkv, po, pgu, pdown;
    Packed plm;
    RowAcc *racc = nullptr;  // split-row scratch of the packed matvec (self-resetting)
    int *h_pin = nullptr;  // pinned host scratch: tokens / pos / argmax
    int64_t *h_logits = nullptr;
    size_t attn_smem = 0;
    // graph of one decode step at batch max_batch
    cudaGraphExec_t graph = nullptr;
    bool loaded_globals = false;
    std::vector<bool> loaded_layer;
};

static int dalloc(void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes);
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

static int model_alloc(iq_model *m) {
    const iq_config &c = m->c;
    const int B = m->max_batch, d = c.hidden_dim, L = c.num_layers;
    m->kvd = c.num_kv_heads * c.head_dim;
    m->qkv_rows = d + 2 * m->kvd;
    DALLOC(m->embed, (size_t)c.vocab_size * d * 8);
    DALLOC(m->fnorm, (size_t)d * 8);
    DALLOC(m->lm, (size_t)c.vocab_size * d * 8);
    m->norm1.resize(L); m->wqkv.resize(L); m->wo.resize(L); m->norm2.resize(L);
    m->wgu.resize(L); m->wdown.resize(L); m->kc.resize(L); m->vc.resize(L);
    m->loaded_layer.assign(L, false);
    m->pqkv.resize(L); m->po.resize(L); m->pgu.resize(L); m->pdown.resize(L);
    {
        size_t rows = std::max(std::max((size_t)c.vocab_size, (size_t)m->qkv_rows),
                               std::max((size_t)2 * c.intermediate_dim, (size_t)d)) + 16;
        DALLOC(m->racc, rows * sizeof(RowAcc));
        IQ_CUDA(cudaMemset(m->racc, 0, rows * sizeof(RowAcc)));
    }
    for (int l = 0; l < L; l++) {
        DALLOC(m->norm1[l], (size_t)d * 8);
        DALLOC(m->wqkv[l], (size_t)m->qkv_rows * d * 8);
        DALLOC(m->wo[l], (size_t)d * d * 8);
        DALLOC(m->norm2[l], (size_t)d * 8);
        DALLOC(m->wgu[l], (size_t)2 * c.intermediate_dim * d * 8);
        DALLOC(m->wdown[l], (size_t)d * c.intermediate_dim * 8);
        size_t kvb = (size_t)B * c.max_seq_len * m->kvd * 8;
        DALLOC(m->kc[l], kvb);
        DALLOC(m->vc[l], kvb);
    }
    size_t half = c.head_dim / 2;
    DALLOC(m->rcos, (size_t)c.max_seq_len * half * 8);
    DALLOC(m->rsin, (size_t)c.max_seq_len * half * 8);
    DALLOC(m->hidden, (size_t)B * d * 8);
    DALLOC(m->normed, (size_t)B * d * 8);
    DALLOC(m->qkv, (size_t)B * m->qkv_rows * 8);
    DALLOC(m->att, (size_t)B * d * 8);
    DALLOC(m->gu, (size_t)B * 2 * c.intermediate_dim * 8);
    DALLOC(m->act, (size_t)B * c.intermediate_dim * 8);
    DALLOC(m->logits, (size_t)B * c.vocab_size * 8);
    DALLOC(m->d_tok, (size_t)B * 4);
    DALLOC(m->d_pos, (size_t)B * 4);
    DALLOC(m->d_arg, (size_t)B * 4);
    DALLOC(m->d_hist, (size_t)B * (c.max_seq_len + 1) * 4);
    // pinned ints: [0, B) results, then (max_seq + 2) slots of 2*B (token, pos)
    IQ_CUDA(cudaMallocHost(&m->h_pin, ((size_t)B + 16 + (size_t)2 * B * (c.max_seq_len + 2)) * 4));
    IQ_CUDA(cudaMallocHost(&m->h_logits, (size_t)c.vocab_size * 8));
    int groups_area = 256;  // attention block size (PV partials reuse the score area)
    m->attn_smem = (size_t)(c.head_dim + (c.max_seq_len > groups_area ? c.max_seq_len : groups_area)) * 8;
    return IQ_OK;
}

// ---------------------------------------------------------------- the step

// Enqueues one forward step for sequences [0, B): tokens in d_tok, positions in
// d_pos (both device), logits -> m->logits, argmax -> d_arg; the argmax kernel
// then advances d_tok / d_pos and records the token in d_hist.
static int enqueue_step(iq_model *m, int B) {
    const iq_config &c = m->c;
    const int d = c.hidden_dim, inter = c.intermediate_dim, hd = c.head_dim;
    cudaStream_t s = m->s;
    int rc;
    auto proj = [&](int64_t *out, const int64_t *W, const Packed &P, const int64_t *x, int M, int N,
                    int add) -> int {
        if (B == 1) return launch_matvec_planes(out, P, x, s, add, m->racc);
        return launch_gemm_add(out, W, x, B, M, N, s, add);
    };
    k_embed<<<dim3((d + 255) / 256, B), 256, 0, s>>>(m->hidden, m->embed, m->d_tok, d);
    IQ_CHECK_LAUNCH();
    const int pairs = (c.num_heads + c.num_kv_heads) * (hd / 2) + m->kvd;
    for (int l = 0; l < c.num_layers; l++) {
        k_rmsnorm<<<B, 256, 0, s>>>(m->normed, m->hidden, m->norm1[l], d);
        IQ_CHECK_LAUNCH();
        if ((rc = proj(m->qkv, m->wqkv[l], m->pqkv[l], m->normed, m->qkv_rows, d, 0))) return rc;
        k_rope_kv<<<dim3((pairs + 255) / 256, B), 256, 0, s>>>(m->qkv, m->kc[l], m->vc[l], m->rcos, m->rsin,
                                                               m->d_pos, c.num_heads, c.num_kv_heads, hd,
                                                               c.max_seq_len);
        IQ_CHECK_LAUNCH();
        k_attention<<<dim3(c.num_heads, B), 256, m->attn_smem, s>>>(m->att, m->qkv, m->kc[l], m->vc[l], m->d_pos,
                                                                    c.num_heads, c.num_kv_heads, hd,
                                                                    c.max_seq_len);
        IQ_CHECK_LAUNCH();
        if ((rc = proj(m->hidden, m->wo[l], m->po[l], m->att, d, d, 1))) return rc;
        k_rmsnorm<<<B, 256, 0, s>>>(m->normed, m->hidden, m->norm2[l], d);
        IQ_CHECK_LAUNCH();
        if ((rc = proj(m->gu, m->wgu[l], m->pgu[l], m->normed, 2 * inter, d, 0))) return rc;
        k_swiglu<<<(B * inter + 255) / 256, 256, 0, s>>>(m->act, m->gu, inter, B);
        IQ_CHECK_LAUNCH();
        if ((rc = proj(m->hidden, m->wdown[l], m->pdown[l], m->act, d, inter, 1))) return rc;
    }
    k_rmsnorm<<<B, 256, 0, s>>>(m->normed, m->hidden, m->fnorm, d);
    IQ_CHECK_LAUNCH();
    if ((rc = proj(m->logits, m->lm, m->plm, m->normed, c.vocab_size, d, 0))) return rc;
    k_argmax<<<B, 1024, 0, s>>>(m->d_arg, m->logits, c.vocab_size, m->d_tok, m->d_pos, m->d_hist,
                                c.max_seq_len + 1);
    IQ_CHECK_LAUNCH();
    return IQ_OK;
}

static int ensure_graph(iq_model *m) {
    if (m->graph) return IQ_OK;
    cudaGraph_t g;
    IQ_CUDA(cudaStreamBeginCapture(m->s, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m, m->max_batch);
    cudaError_t e = cudaStreamEndCapture(m->s, &g);
    if (rc) { if (e == cudaSuccess) cudaGraphDestroy(g); return rc; }
    if (e != cudaSuccess) return cuda_fail(e);
    e = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e);
    return IQ_OK;
}

static bool model_ready(iq_model *m) {
    if (!m || !m->loaded_globals) return false;
    for (bool b : m->loaded_layer) if (!b) return false;
    return true;
}

// ----------------------------------------------------------- host helpers

static int h2d(void *dst, const void *src, size_t bytes) {
    IQ_CUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    return IQ_OK;
}

static int fill_const(int64_t *dst, int64_t v, size_t n) {
    std::vector<int64_t> h(n, v);
    return h2d(dst, h.data(), n * 8);
}

static int repack(iq_model *m, Packed *P, const int64_t *W, int M, int N) {
    if (P->planes) { IQ_CUDA(cudaStreamSynchronize(m->s)); free_packed(P); }
    int rc = pack_weights(W, M, N, m->s, P);
    if (rc) return rc;
    IQ_CUDA(cudaStreamSynchronize(m->s));
    return IQ_OK;
}
static int repack_layer(iq_model *m, int l) {
    const iq_config &c = m->c;
    int rc, d = c.hidden_dim, it = c.intermediate_dim;
    if ((rc = repack(m, &m->pqkv[l], m->wqkv[l], m->qkv_rows, d))) return rc;
    if ((rc = repack(m, &m->po[l], m->wo[l], d, d))) return rc;
    if ((rc = repack(m, &m->pgu[l], m->wgu[l], 2 * it, d))) return rc;
    return repack(m, &m->pdown[l], m->wdown[l], d, it);
}

extern "C" {

IQ_API int iq_model_create(const iq_config *cfg, int max_batch, int device, iq_model **out) {
    if (!cfg || !out || max_batch < 1) return IQ_ERR_ARG;
    *out = nullptr;
    const iq_config &c = *cfg;
    if (c.hidden_dim <= 0 || c.num_heads <= 0 || c.num_kv_heads <= 0 || c.head_dim <= 1 ||
        c.num_layers <= 0 || c.intermediate_dim <= 0 || c.vocab_size <= 0 || c.max_seq_len <= 0 ||
        c.num_heads % c.num_kv_heads != 0 || c.hidden_dim != c.num_heads * c.head_dim ||
        (c.head_dim & 1) || c.head_dim > 256)
        return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(device));
    int rc = ensure_device_pub(device);
    if (rc) return rc;
    iq_model *m = new iq_model();
    m->c = c;
    m->dev = device;
    m->max_batch = max_batch;
    cudaError_t e = cudaStreamCreateWithFlags(&m->s, cudaStreamNonBlocking);
    if (e != cudaSuccess) { delete m; return cuda_fail(e); }
    if ((rc = model_alloc(m))) { iq_model_destroy(m); return rc; }
    if (m->attn_smem > 200 * 1024) { iq_model_destroy(m); return IQ_ERR_UNSUPPORTED; }
    if (m->attn_smem > 48 * 1024) {
        e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->attn_smem);
        if (e != cudaSuccess) { iq_model_destroy(m); return cuda_fail(e); }
    }
    k_rope_init<<<256, 128, 0, m->s>>>(m->rcos, m->rsin, c.head_dim, c.max_seq_len, c.rope_theta);
    e = cudaStreamSynchronize(m->s);
    if (e != cudaSuccess) { iq_model_destroy(m); return cuda_fail(e); }
    if ((rc = iq_model_reset(m))) { iq_model_destroy(m); return rc; }
    *out = m;
    return IQ_OK;
}

IQ_API int iq_model_destroy(iq_model *m) {
    if (!m) return IQ_ERR_ARG;
    cudaSetDevice(m->dev);
    if (m->s) cudaStreamSynchronize(m->s);
    if (m->graph) cudaGraphExecDestroy(m->graph);
    void *bufs[] = {m->embed, m->fnorm, m->lm, m->rcos, m->rsin, m->hidden, m->normed, m->qkv, m->att,
                    m->gu, m->act, m->logits, m->d_tok, m->d_pos, m->d_arg, m->d_hist};
    for (void *p : bufs) if (p) cudaFree(p);
    for (auto *v : {&m->norm1, &m->wqkv, &m->wo, &m->norm2, &m->wgu, &m->wdown, &m->kc, &m->vc})
        for (int64_t *p : *v) if (p) cudaFree(p);
    for (auto *v : {&m->pqkv, &m->po, &m->pgu, &m->pdown})
        for (Packed &P : *v) free_packed(&P);
    free_packed(&m->plm);
    if (m->racc) cudaFree(m->racc);
    if (m->h_pin) cudaFreeHost(m->h_pin);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->s) cudaStreamDestroy(m->s);
    delete m;
    return IQ_OK;
}

IQ_API int iq_model_load_globals(iq_model *m, const int64_t *embed, const int64_t *final_norm,
                                 const int64_t *lm_head) {
    if (!m || !embed || !final_norm || !lm_head) return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(m->dev));
    const iq_config &c = m->c;
    int rc;
    if ((rc = h2d(m->embed, embed, (size_t)c.vocab_size * c.hidden_dim * 8))) return rc;
    if ((rc = h2d(m->fnorm, final_norm, (size_t)c.hidden_dim * 8))) return rc;
    if ((rc = h2d(m->lm, lm_head, (size_t)c.vocab_size * c.hidden_dim * 8))) return rc;
    if ((rc = repack(m, &m->plm, m->lm, c.vocab_size, c.hidden_dim))) return rc;
    m->loaded_globals = true;
    return IQ_OK;
}

IQ_API int iq_model_load_layer(iq_model *m, int l, const int64_t *const w[9]) {
    if (!m || !w || l < 0 || l >= m->c.num_layers) return IQ_ERR_ARG;
    for (int i = 0; i < 9; i++) if (!w[i]) return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(m->dev));
    const size_t d = m->c.hidden_dim, kvd = m->kvd, it = m->c.intermediate_dim;
    int rc;
    if ((rc = h2d(m->norm1[l], w[0], d * 8))) return rc;
    if ((rc = h2d(m->wqkv[l], w[1], d * d * 8))) return rc;
    if ((rc = h2d(m->wqkv[l] + d * d, w[2], kvd * d * 8))) return rc;
    if ((rc = h2d(m->wqkv[l] + (d + kvd) * d, w[3], kvd * d * 8))) return rc;
    if ((rc = h2d(m->wo[l], w[4], d * d * 8))) return rc;
    if ((rc = h2d(m->norm2[l], w[5], d * 8))) return rc;
    if ((rc = h2d(m->wgu[l], w[6], it * d * 8))) return rc;
    if ((rc = h2d(m->wgu[l] + it * d, w[7], it * d * 8))) return rc;
    if ((rc = h2d(m->wdown[l], w[8], d * it * 8))) return rc;
    if ((rc = repack_layer(m, l))) return rc;
    m->loaded_layer[l] = true;
    return IQ_OK;
}

IQ_API int iq_model_reset(iq_model *m) {
    if (!m) return IQ_ERR_ARG;
    IQ_CUDA(cudaSetDevice(m->dev));
    size_t kvb = (size_t)m->max_batch * m->c.max_seq_len * m->kvd * 8;
    for (int l = 0; l < m->c.num_layers; l++) {
        IQ_CUDA(cudaMemsetAsync(m->kc[l], 0, kvb, m->s));
        IQ_CUDA(cudaMemsetAsync(m->vc[l], 0, kvb, m->s));
    }
    IQ_CUDA(cudaStreamSynchronize(m->s));
    return IQ_OK;
}

// ------------------------------------------------------------- synthetic

struct SynthJob { std::string name; int64_t *dst; size_t n; bool ones; };

IQ_API int iq_model_synth(iq_model *m, int config_index, int threads) {
    if (!m) return IQ_ERR_ARG;
    const iq_config &c = m->c;
    const size_t d = c.hidden_dim, kvd = m->kvd, it = c.intermediate_dim, V = c.vocab_size;
    std::vector<SynthJob> jobs;
    jobs.push_back({"model.embed_tokens.weight", m->embed, V * d, false});
    jobs.push_back({"lm_head.weight", m->lm, V * d, false});
    jobs.push_back({"model.norm.weight", m->fnorm, d, true});
    char nm[160];
    for (int l = 0; l < c.num_layers; l++) {
        auto add = [&](const char *t, int64_t *dst, size_t n, bool ones) {
            snprintf(nm, sizeof nm, "model.layers.%d.%s.weight", l, t);
            jobs.push_back({nm, dst, n, ones});
        };
        add("input_layernorm", m->norm1[l], d, true);
        add("self_attn.q_proj", m->wqkv[l], d * d, false);
        add("self_attn.k_proj", m->wqkv[l] + d * d, kvd * d, false);
        add("self_attn.v_proj", m->wqkv[l] + (d + kvd) * d, kvd * d, false);
        add("self_attn.o_proj", m->wo[l], d * d, false);
        add("post_attention_layernorm", m->norm2[l], d, true);
        add("mlp.gate_proj", m->wgu[l], it * d, false);
        add("mlp.up_proj", m->wgu[l] + it * d, it * d, false);
        add("mlp.down_proj", m->wdown[l], d * it, false);
    }
    if (threads < 1) threads = 1;
    std::atomic<size_t> next(0);
    std::atomic<int> status(IQ_OK);
    auto worker = [&]() {
        cudaSetDevice(m->dev);
        std::vector<int64_t> buf;
        for (;;) {
            size_t j = next.fetch_add(1);
            if (j >= jobs.size() || status.load() != IQ_OK) return;
            const SynthJob &jb = jobs[j];
            buf.resize(jb.n);
            if (jb.ones) std::fill(buf.begin(), buf.end(), IQ_ONE);
            else iq_synth_weights(iq_tensor_seed(config_index, jb.name.c_str()), buf.data(), (int64_t)jb.n);
            cudaError_t e = cudaMemcpy(jb.dst, buf.data(), jb.n * 8, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) status.store(cuda_fail(e));
        }
    };
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; t++) pool.emplace_back(worker);
    for (auto &t : pool) t.join();
    if (status.load() != IQ_OK) return status.load();
    int rc;
    IQ_CUDA(cudaSetDevice(m->dev));
    if ((rc = repack(m, &m->plm, m->lm, c.vocab_size, c.hidden_dim))) return rc;
    for (int l = 0; l < c.num_layers; l++)
        if ((rc = repack_layer(m, l))) return rc;
    m->loaded_globals = true;
    m->loaded_layer.assign(c.num_layers, true);
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

IQ_API int iq_forward(iq_model *m, int token, int pos, int64_t *logits, int *argmax_out) {
    if (!model_ready(m)) return m ? IQ_ERR_STATE : IQ_ERR_ARG;
    if (token < 0 || token >= m->c.vocab_size || pos < 0 || pos >= m->c.max_seq_len) return IQ_ERR_RANGE;
    IQ_CUDA(cudaSetDevice(m->dev));
    IQ_CUDA(cudaStreamSynchronize(m->s));
    int rc;
    if ((rc = set_tok_pos(m, &token, &pos, 1, 0))) return rc;
    if ((rc = enqueue_step(m, 1))) return rc;
    if (logits) IQ_CUDA(cudaMemcpyAsync(m->h_logits, m->logits, (size_t)m->c.vocab_size * 8, cudaMemcpyDeviceToHost, m->s));
    IQ_CUDA(cudaMemcpyAsync(m->h_pin, m->d_arg, 4, cudaMemcpyDeviceToHost, m->s));
    IQ_CUDA(cudaStreamSynchronize(m->s));
    if (logits) memcpy(logits, m->h_logits, (size_t)m->c.vocab_size * 8);
    if (argmax_out) *argmax_out = m->h_pin[0];
    return IQ_OK;
}

static uint64_t fnv_mix(uint64_t h, const int64_t *v, size_t n) {
    for (size_t i = 0; i < n; i++) {
        uint64_t u = (uint64_t)v[i];
        for (int b = 0; b < 8; b++) { h ^= u & 0xff; h *= 1099511628211ULL; u >>= 8; }
    }
    return h;
}

// one step for B sequences: the captured graph when B == max_batch
static int run_step(iq_model *m, int B) {
    if (B == m->max_batch) {
        int rc = ensure_graph(m);
        if (rc) return rc;
        IQ_CUDA(cudaGraphLaunch(m->graph, m->s));
        return IQ_OK;
    }
    return enqueue_step(m, B);
}

IQ_API int iq_generate(iq_model *m, const int *prompt, int plen, int max_new, int *out, int *n_out,
                       uint64_t *logit_hash) {
    if (!m || !prompt || !out || !n_out || plen < 1 || max_new < 1) return IQ_ERR_ARG;
    if (!model_ready(m)) return IQ_ERR_STATE;
    const iq_config &c = m->c;
    *n_out = -1;
    for (int i = 0; i < plen; i++)
        if (prompt[i] < 0 || prompt[i] >= c.vocab_size) return IQ_ERR_RANGE;  // llama_int.c:2813
    if (plen > c.max_seq_len) return IQ_ERR_RANGE;                          // llama_int.c:2817
    int rc;
    if ((rc = iq_model_reset(m))) return rc;
    const bool hash = logit_hash != nullptr;
    uint64_t h = 1469598103934665603ULL;
    memcpy(out, prompt, (size_t)plen * sizeof(int));
    const int V = c.vocab_size;
    auto pull = [&]() -> int {  // sync, fold this step's logits into the hash, return argmax
        IQ_CUDA(cudaMemcpyAsync(m->h_logits, m->logits, (size_t)V * 8, cudaMemcpyDeviceToHost, m->s));
        IQ_CUDA(cudaMemcpyAsync(m->h_pin, m->d_arg, 4, cudaMemcpyDeviceToHost, m->s));
        IQ_CUDA(cudaStreamSynchronize(m->s));
        h = fnv_mix(h, m->h_logits, V);
        return IQ_OK;
    };
    // prefill: one M=1 forward per prompt position (llama_int.c:3081-3092)
    for (int p = 0; p < plen; p++) {
        if ((rc = set_tok_pos(m, &prompt[p], &p, 1, p))) return rc;
        if ((rc = run_step(m, 1))) return rc;
        if (hash && (rc = pull())) return rc;
    }
    int total = plen;
    // decode positions plen .. ; the reference stops when pos reaches max_seq_len
    int steps = std::min(max_new - 1, c.max_seq_len - plen);
    if (hash) {
        out[total++] = m->h_pin[0];  // prefill's sample is appended unconditionally
        for (int i = 1; i <= steps; i++) {
            if ((rc = run_step(m, 1))) return rc;  // d_tok / d_pos advanced on the device
            if ((rc = pull())) return rc;
            int nx = m->h_pin[0];
            if (nx == 2) break;  // LLAMA_EOS (llama_int.c:3046, 3110)
            out[total++] = nx;
        }
        *logit_hash = h;
    } else {
        for (int i = 1; i <= steps; i++)
            if ((rc = run_step(m, 1))) return rc;
        std::vector<int> hist(steps + 1);
        IQ_CUDA(cudaMemcpyAsync(hist.data(), m->d_hist + plen, (size_t)(steps + 1) * 4, cudaMemcpyDeviceToHost, m->s));
        IQ_CUDA(cudaStreamSynchronize(m->s));
        out[total++] = hist[0];
        for (int i = 1; i <= steps; i++) {
            if (hist[i] == 2) break;
            out[total++] = hist[i];
        }
    }
    *n_out = total;
    return IQ_OK;
}

IQ_API int iq_generate_batch(iq_model *m, const int *prompts, int plen, int max_new, int *out, int *n_out) {
    if (!m || !prompts || !out || !n_out || plen < 1 || max_new < 1) return IQ_ERR_ARG;
    if (!model_ready(m)) return IQ_ERR_STATE;
    const iq_config &c = m->c;
    const int B = m->max_batch;
    for (int i = 0; i < B * plen; i++)
        if (prompts[i] < 0 || prompts[i] >= c.vocab_size) return IQ_ERR_RANGE;
    if (plen > c.max_seq_len) return IQ_ERR_RANGE;
    int rc;
    if ((rc = iq_model_reset(m))) return rc;
    std::vector<int> tok(B), pos(B);
    for (int p = 0; p < plen; p++) {
        for (int b = 0; b < B; b++) { tok[b] = prompts[(size_t)b * plen + p]; pos[b] = p; }
        if ((rc = set_tok_pos(m, tok.data(), pos.data(), B, p))) return rc;
        if ((rc = run_step(m, B))) return rc;
    }
    int steps = std::min(max_new - 1, c.max_seq_len - plen);
    for (int i = 1; i <= steps; i++)
        if ((rc = run_step(m, B))) return rc;
    const int stride = c.max_seq_len + 1;
    std::vector<int> hist((size_t)B * stride);
    IQ_CUDA(cudaMemcpyAsync(hist.data(), m->d_hist, hist.size() * 4, cudaMemcpyDeviceToHost, m->s));
    IQ_CUDA(cudaStreamSynchronize(m->s));
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
    return IQ_OK;
}

IQ_API int iq_decode_steps_timed(iq_model *m, int pos0, int steps, float *ms) {
    if (!m || !ms || steps < 1 || pos0 < 0 || pos0 + steps > m->c.max_seq_len) return IQ_ERR_ARG;
    if (!model_ready(m)) return IQ_ERR_STATE;
    IQ_CUDA(cudaSetDevice(m->dev));
    int rc;
    std::vector<int> tok(m->max_batch), pos(m->max_batch, pos0);
    IQ_CUDA(cudaStreamSynchronize(m->s));
    IQ_CUDA(cudaMemcpy(tok.data(), m->d_tok, tok.size() * 4, cudaMemcpyDeviceToHost));
    if ((rc = set_tok_pos(m, tok.data(), pos.data(), m->max_batch, 0))) return rc;
    if ((rc = ensure_graph(m))) return rc;
    cudaEvent_t e0, e1;
    IQ_CUDA(cudaEventCreate(&e0));
    IQ_CUDA(cudaEventCreate(&e1));
    IQ_CUDA(cudaEventRecord(e0, m->s));
    for (int i = 0; i < steps; i++) IQ_CUDA(cudaGraphLaunch(m->graph, m->s));
    IQ_CUDA(cudaEventRecord(e1, m->s));
    IQ_CUDA(cudaEventSynchronize(e1));
    IQ_CUDA(cudaEventElapsedTime(ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return IQ_OK;
}

}  // extern "C"
