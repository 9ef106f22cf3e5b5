/*
 * ref_harness.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * Builds the reference int-llm CPU implementation, unmodified, into a shared
 * library so tests and the bench's CPU-baseline leg can call its static
 * functions. The reference sources are NOT copied: the recipe in
 * oracle/Makefile compiles this file with -I pointing at the read-only
 * reference checkout, and this file includes llama_int.c from there with
 * `main` renamed. Output goes to oracle/_ref/ (git-ignored).
 *
 * Exposed entry points (all thin wrappers over the reference's own code):
 *   ref_matmul_vec     -> matmul_vec            llama_int.c:1014-1046
 *   ref_rmsnorm        -> rmsnorm               llama_int.c:1048-1058
 *   ref_softmax        -> softmax               llama_int.c:1060-1072
 *   ref_fp             -> fp_math.h primitives  fp_math.h:491-921
 *   ref_rope_tables    -> rope_init             llama_int.c:960-986
 *   ref_model_*        -> llama_forward / generate on caller-owned weights
 *                         llama_int.c:2807-2886, 3067-3135
 *   ref_sample_token   -> sample_token with sample_params_t   llama_int.c:2958-3039
 *   ref_model_generate_sampled -> generate(..., sp)          llama_int.c:3067-3135
 *   ref_set_kv_packed  -> the --kv-packed switch g_kv_quant  llama_int.c:4740-4751
 *   ref_model_open_mgw -> mgw_load (mmap, layers cached) or mgw_load_streaming
 *                         (layers pread into fresh buffers and freed after
 *                         every layer), llama_int.c:2344-2803
 *
 * Built a second time against a copy of llama_int.c whose matmul_vec is
 * renamed and replaced by the libiq.so drop-in (include/iq_matmul_vec_shim.h):
 * oracle/_ref/libllamaref_iq.so, the integration test of that shim.
 */
#define main llama_int_main
#ifdef REF_SOURCE
#include REF_SOURCE   /* a patched copy of llama_int.c (the drop-in shim build) */
#else
#include "llama_int.c"
#endif
#undef main

#include <pthread.h>

#define REFAPI __attribute__((visibility("default")))

REFAPI void ref_matmul_vec(int64_t *out, const int64_t *w, const int64_t *in, int M, int N) {
    matmul_vec(out, w, in, M, N);
}

/* Row-partitioned multi-threaded call of the reference matmul_vec (rows are
 * independent, so each thread runs the unmodified function on its slice). */
typedef struct { int64_t *out; const int64_t *w; const int64_t *in; int r0, r1, N; } ref_mv_job;
static void *ref_mv_worker(void *p) {
    ref_mv_job *j = (ref_mv_job *)p;
    if (j->r1 > j->r0)
        matmul_vec(j->out + j->r0, j->w + (int64_t)j->r0 * j->N, j->in, j->r1 - j->r0, j->N);
    return NULL;
}
REFAPI void ref_matmul_vec_mt(int64_t *out, const int64_t *w, const int64_t *in, int M, int N, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    ref_mv_job jobs[256];
    for (int t = 0; t < threads; t++) {
        jobs[t].out = out; jobs[t].w = w; jobs[t].in = in; jobs[t].N = N;
        jobs[t].r0 = (int)((int64_t)M * t / threads);
        jobs[t].r1 = (int)((int64_t)M * (t + 1) / threads);
        pthread_create(&tid[t], NULL, ref_mv_worker, &jobs[t]);
    }
    for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
}

REFAPI void ref_rmsnorm(int64_t *out, const int64_t *x, const int64_t *w, int dim) {
    rmsnorm(out, x, w, dim);
}

REFAPI void ref_softmax(int64_t *x, int n) { softmax(x, n); }

REFAPI int64_t ref_bf16_to_q1648(uint16_t bits) { return bfloat16_to_q1648(bits); }

/* fn codes shared with oracle/iq_oracle.h and include/iq.h (IQ_FN_*) */
REFAPI int64_t ref_fp(int fn, int64_t x, int64_t y) {
    fp_math_init();
    fixed_t c, s;
    switch (fn) {
    case 0: return fp_mul(x, y);
    case 1: return fp_div(x, y);
    case 2: return fp_sqrt(x);
    case 3: return fp_sqrt_fast(x);
    case 4: return fp_inv_sqrt(x);
    case 5: return fp_exp(x);
    case 6: return fp_log(x);
    case 7: fp_sincos(x, &c, &s); return c;
    case 8: fp_sincos(x, &c, &s); return s;
    case 9: return fp_sigmoid(x);
    case 10: return fp_silu(x);
    case 11: return fp_safe_exp(x);
    case 12: return fp_exp_dyadic(x, (int)y);
    default: return 0;
    }
}

REFAPI void ref_rope_tables(int head_dim, int max_seq_len, int rope_theta, int64_t *cos_out, int64_t *sin_out) {
    llama_config_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.head_dim = head_dim;
    cfg.max_seq_len = max_seq_len;
    cfg.rope_theta = rope_theta;
    rope_table_t r;
    rope_init(&r, &cfg);
    size_t n = (size_t)max_seq_len * (head_dim / 2);
    memcpy(cos_out, r.cos_table, n * sizeof(int64_t));
    memcpy(sin_out, r.sin_table, n * sizeof(int64_t));
    rope_free(&r);
}

/* layer_ptrs: 9 pointers per layer in layer_weights_t order
 * (input_layernorm, q, k, v, o, post_attn_norm, gate, up, down). */
REFAPI void *ref_model_create(const int *cfg9, int64_t *embed, int64_t *final_norm,
                              int64_t *lm_head, int64_t **layer_ptrs) {
    llama_model_t *m = (llama_model_t *)calloc(1, sizeof(llama_model_t));
    if (!m) return NULL;
    m->cfg.hidden_dim = cfg9[0];
    m->cfg.num_heads = cfg9[1];
    m->cfg.num_kv_heads = cfg9[2];
    m->cfg.head_dim = cfg9[3];
    m->cfg.num_layers = cfg9[4];
    m->cfg.intermediate_dim = cfg9[5];
    m->cfg.vocab_size = cfg9[6];
    m->cfg.max_seq_len = cfg9[7];
    m->cfg.rope_theta = cfg9[8];
    m->embed_tokens = embed;
    m->final_norm = final_norm;
    m->lm_head = lm_head;
    m->native_stream_fd = -1;
    m->cached_layers = (layer_weights_t *)calloc((size_t)m->cfg.num_layers, sizeof(layer_weights_t));
    for (int l = 0; l < m->cfg.num_layers; l++) {
        int64_t **p = layer_ptrs + 9 * l;
        layer_weights_t *w = &m->cached_layers[l];
        w->input_layernorm = p[0]; w->q_proj = p[1]; w->k_proj = p[2]; w->v_proj = p[3];
        w->o_proj = p[4]; w->post_attn_norm = p[5]; w->gate_proj = p[6]; w->up_proj = p[7];
        w->down_proj = p[8];
    }
    m->layers_cached = 1;
    rope_init(&m->rope, &m->cfg);
    if (kv_cache_init(&m->kv, &m->cfg) != 0) return NULL;
    llama_init_scratch(m);
    return m;
}

REFAPI void ref_model_reset(void *h) { kv_cache_reset(&((llama_model_t *)h)->kv); }

/* Runs llama_forward once; copies the logits into logits_out when non-NULL.
 * Returns argmax, or -1 when llama_forward returned NULL. */
REFAPI int ref_model_forward(void *h, int token, int pos, int64_t *logits_out) {
    llama_model_t *m = (llama_model_t *)h;
    fixed_t *lg = llama_forward(m, token, pos);
    if (!lg) return -1;
    if (logits_out) memcpy(logits_out, lg, (size_t)m->cfg.vocab_size * sizeof(int64_t));
    int a = argmax(lg, m->cfg.vocab_size);
    free(lg);
    return a;
}

REFAPI int ref_model_generate(void *h, const int *prompt, int prompt_len, int max_new, int *out_tokens) {
    return generate((llama_model_t *)h, prompt, prompt_len, max_new, out_tokens, NULL);
}

REFAPI void ref_model_free(void *h) {
    llama_model_t *m = (llama_model_t *)h;
    if (!m) return;
    rope_free(&m->rope);
    kv_cache_free(&m->kv);
    free(m->scratch_buf);
    free(m->cached_layers);
    free(m);
}

/* Opens a .mgw model the way main() does for --native / --native-stream
 * (llama_int.c:4877-4910, 5048-5084). Returns NULL on any load error. */
REFAPI void *ref_model_open_mgw(const char *path, int streaming) {
    llama_model_t *m = (llama_model_t *)calloc(1, sizeof(llama_model_t));
    if (!m) return NULL;
    m->native_stream_fd = -1;
    int rc = streaming ? mgw_load_streaming(m, path) : mgw_load(m, path);
    if (rc != 0) { free(m); return NULL; }
    rope_init(&m->rope, &m->cfg);
    if (kv_cache_init(&m->kv, &m->cfg) != 0) return NULL;
    llama_init_scratch(m);
    return m;
}

REFAPI void ref_model_close_mgw(void *h) {
    llama_model_t *m = (llama_model_t *)h;
    if (!m) return;
    rope_free(&m->rope);
    kv_cache_free(&m->kv);
    free(m->scratch_buf);
    if (m->native_loaded) {
        free(m->cached_layers);
        munmap(m->native_mmap, m->native_mmap_size);
    } else if (m->native_stream) {
        if (!m->lm_head_tied) free(m->lm_head);
        free(m->embed_tokens);
        free(m->final_norm);
        free(m->ns_index);
        if (m->native_stream_fd >= 0) close(m->native_stream_fd);
    }
    free(m);
}

/* sample_token on caller logits with the given parameters and generator
 * state {s0, s1} (advanced in place). */
REFAPI int ref_sample_token(const int64_t *logits, int V, int64_t temp, int top_k, int64_t top_p, uint64_t *rng) {
    sample_params_t sp;
    sp.temperature = temp;
    sp.top_k = top_k;
    sp.top_p = top_p;
    sp.rng.s[0] = rng[0];
    sp.rng.s[1] = rng[1];
    int t = sample_token(logits, V, &sp);
    rng[0] = sp.rng.s[0];
    rng[1] = sp.rng.s[1];
    return t;
}

REFAPI void ref_rng_seed(uint64_t seed, uint64_t *rng) {
    rng_state_t r;
    rng_seed(&r, seed);
    rng[0] = r.s[0];
    rng[1] = r.s[1];
}

REFAPI int ref_model_generate_sampled(void *h, const int *prompt, int prompt_len, int max_new, int64_t temp,
                                      int top_k, int64_t top_p, uint64_t seed, int *out_tokens) {
    sample_params_t sp;
    sp.temperature = temp;
    sp.top_k = top_k;
    sp.top_p = top_p;
    rng_seed(&sp.rng, seed);
    return generate((llama_model_t *)h, prompt, prompt_len, max_new, out_tokens, &sp);
}

/* The reference's --kv-packed KbVb switch (llama_int.c:4740-4751): affects
 * models created afterwards (kv_cache_init reads it); (0, 0) turns it off. */
REFAPI void ref_set_kv_packed(int k_bits, int v_bits) {
    g_kv_quant.enabled = k_bits > 0;
    g_kv_quant.packed = k_bits > 0;
    g_kv_quant.k_bits = k_bits;
    g_kv_quant.v_bits = v_bits;
}
