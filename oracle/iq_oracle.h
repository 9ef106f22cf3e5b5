/*
 * iq_oracle.h -- CPU restatement of int-llm's Q16.48 hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker for the CUDA library
 * (libiq.so); only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it. The product never calls into it.
 *
 * Parity is pinned two ways: (1) the reference's determinism gate golden
 * (tests/determinism_golden.txt = c0d933ea340452ec, fp_determinism.c:162-200)
 * and its per-function sub-hashes, reproduced by iqo_det_hash(); (2) the
 * reference itself compiled from source into oracle/_ref (ref_harness.c),
 * whose outputs are compared with these functions in tests/ and frozen into
 * tests/golden/.
 */
#ifndef IQ_ORACLE_H
#define IQ_ORACLE_H
#include <stdint.h>

/* fp_math function codes (same numbering as ref_harness.c and IQ_FN_* in iq.h) */
enum {
    IQO_MUL = 0, IQO_DIV, IQO_SQRT, IQO_SQRT_FAST, IQO_INV_SQRT, IQO_EXP, IQO_LOG,
    IQO_COS, IQO_SIN, IQO_SIGMOID, IQO_SILU, IQO_SAFE_EXP, IQO_EXP_DYADIC
};

int64_t iqo_fp(int fn, int64_t x, int64_t y);
void iqo_fp_vec(int fn, const int64_t *x, const int64_t *y, int64_t *out, int64_t n);
uint64_t iqo_det_hash(uint64_t subs_out[12]);

void iqo_matmul_vec(int64_t *out, const int64_t *w, const int64_t *in, int M, int N);
void iqo_matmul_rows(int64_t *out, const int64_t *w, const int64_t *X, int rows, int M, int N);
void iqo_rmsnorm(int64_t *out, const int64_t *x, const int64_t *w, int dim);
void iqo_softmax(int64_t *x, int n);
void iqo_rope_tables(int head_dim, int max_seq_len, int rope_theta, int64_t *cos_out, int64_t *sin_out);

int64_t iqo_bf16_to_q1648(uint16_t bits);
uint16_t iqo_q1648_to_bf16_rne(int64_t w);
uint64_t iqo_fnv1a64(const char *s);
uint64_t iqo_fnv_mix_i64(uint64_t h, int64_t v);
uint64_t iqo_fnv_array(uint64_t h, const int64_t *v, int64_t n);
uint64_t iqo_tensor_seed(int config_index, const char *name);
void iqo_synth_weights(uint64_t seed, int64_t *out, int64_t n);
void iqo_synth_acts(uint64_t seed, int64_t *out, int64_t n);
void iqo_synth_tokens(uint64_t seed, int *out, int n, int vocab);

/* model: cfg9 = {dim, n_heads, n_kv_heads, head_dim, n_layers, inter, vocab, max_seq, rope_theta} */
void *iqo_model_create(const int *cfg9, const int64_t *embed, const int64_t *final_norm,
                       const int64_t *lm_head, const int64_t *const *layer_ptrs);
void iqo_model_reset(void *m);
int iqo_model_forward(void *m, int token, int pos, int64_t *logits_out);
int iqo_model_generate(void *m, const int *prompt, int prompt_len, int max_new, int *out_tokens,
                       uint64_t *logit_hash_out);
void iqo_model_free(void *m);
int iqo_sample_token(const int64_t *logits, int V, int64_t temp, int top_k, int64_t top_p, uint64_t rng[2]);
void iqo_rng_seed(uint64_t seed, uint64_t rng[2]);
int iqo_model_generate_sampled(void *h, const int *prompt, int plen, int max_new, int64_t temp, int top_k,
                               int64_t top_p, uint64_t seed, int *out, uint64_t *logit_hash_out);
#endif
