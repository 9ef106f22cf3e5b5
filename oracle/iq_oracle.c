/*
 * iq_oracle.c -- CPU restatement of int-llm's Q16.48 hot path (checker only).
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py. The product (libiq.so) never links it.
 *
 * Every function restates the reference algorithm in this file's own code and
 * cites the reference location it follows. Arithmetic is done in gcc's
 * __int128 with -fwrapv, matching the reference build flags (Makefile:38-39).
 * Pinned by: the determinism gate golden c0d933ea340452ec and its sub-hashes
 * (fp_determinism.c:162-200), and by direct comparison against the reference
 * compiled from source (oracle/_ref), see tests/test_oracle.py.
 */
#include "iq_oracle.h"
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

typedef __int128 i128;
typedef unsigned __int128 u128;

#define Q 48
#define ONE ((int64_t)1 << Q)

/* ---------------- fp_math.h primitives ---------------- */

/* fp_mul: floor((a*b) / 2^48), low 64 bits kept. fp_math.h:491-506 */
static inline int64_t o_mul(int64_t a, int64_t b) { return (int64_t)(((i128)a * b) >> Q); }

/* truncating signed 128-bit division with the b == -1 wrap rule. fp_math.h:258-265 */
static inline i128 o_divs128(i128 a, i128 b) {
    if (b == -1) return (i128)(0 - (u128)a);
    return a / b;
}

/* fp_div: sign-magnitude (|a| << 48), re-signed, truncating division. fp_math.h:508-524 */
static inline int64_t o_div(int64_t a, int64_t b) {
    if (b == 0) return 0; /* never reached on the path; the reference is undefined here */
    uint64_t mag = a < 0 ? (uint64_t)0 - (uint64_t)a : (uint64_t)a;
    i128 num = (i128)((u128)mag << Q);
    if (a < 0) num = (i128)(0 - (u128)num);
    return (int64_t)o_divs128(num, (i128)b);
}

static inline int64_t o_from_int(int x) {
    uint64_t mag = x < 0 ? (uint64_t)0 - (uint64_t)x : (uint64_t)x;
    u128 r = (u128)mag << Q;
    if (x < 0) r = 0 - r;
    return (int64_t)r;
}

static inline int o_bits128(u128 a) {
    uint64_t hi = (uint64_t)(a >> 64), lo = (uint64_t)a;
    if (hi) return 128 - __builtin_clzll(hi);
    return lo ? 64 - __builtin_clzll(lo) : 0;
}

/* fp_sqrt: Newton on isqrt(x << 48) from a CLZ guess, 7 rounds, then r^2 <= n fix-up.
 * fp_math.h:624-650 */
static int64_t o_sqrt(int64_t x) {
    if (x <= 0) return 0;
    i128 n = (i128)((u128)(uint64_t)x << Q);
    int bw = o_bits128((u128)n);
    uint64_t r = (uint64_t)1 << ((bw + 1) / 2);
    for (int it = 0; it < 7; it++) {
        if (r == 0) return 0;
        uint64_t q = (uint64_t)(int64_t)o_divs128(n, (i128)r);
        uint64_t nr = (r + q) >> 1;
        if (nr >= r) break;
        r = nr;
    }
    while ((i128)(int64_t)r * (int64_t)r > n) r--;
    return (int64_t)r;
}

/* fp_sqrt_fast: 64-bit Newton isqrt, result << 24. fp_math.h:605-620 */
static int64_t o_sqrt_fast(int64_t x) {
    if (x <= 0) return 0;
    uint64_t ux = (uint64_t)x;
    int bw = 64 - __builtin_clzll(ux);
    uint64_t r = (uint64_t)1 << ((bw + 1) / 2);
    for (int it = 0; it < 5; it++) {
        uint64_t nr = (r + ux / r) >> 1;
        if (nr >= r) break;
        r = nr;
    }
    return (int64_t)(r << 24);
}

/* fp_inv_sqrt: range-reduce to [2^48, 2^50), seed 1.0 or 0.5 by octave, 8 Newton
 * rounds y*(3 - x*y^2)/2 with early exit on y <= 0, rescale with saturation.
 * fp_math.h:658-707 */
static int64_t o_inv_sqrt(int64_t x) {
    if (x <= 0) return 0;
    int msb = 63 - __builtin_clzll((uint64_t)x);
    int k = (msb - Q) >> 1;
    int64_t xn = k >= 0 ? (x >> (2 * k)) : (int64_t)((uint64_t)x << (-2 * k));
    int msb_n = 63 - __builtin_clzll((uint64_t)xn);
    int64_t y = msb_n == Q ? ONE : (ONE >> 1);
    const int64_t three = 3 * ONE;
    for (int it = 0; it < 8; it++) {
        int64_t y2 = (int64_t)(((i128)y * y) >> Q);
        int64_t xy2 = (int64_t)(((i128)xn * y2) >> Q);
        int64_t f = three - xy2;
        y = (int64_t)(((i128)y * f) >> (Q + 1));
        if (y <= 0) { y = 1; break; }
    }
    if (k >= 0) {
        int64_t r = y >> k;
        return r < 0 ? 0 : r;
    }
    i128 r = (i128)((u128)(i128)y << (-k));
    if (r > (i128)INT64_MAX) return INT64_MAX;
    if (r < 0) return 0;
    return (int64_t)r;
}

/* fp_exp_dyadic: (1 + x/2^k)^(2^k) by k squarings. fp_math.h:714-720 */
static int64_t o_exp_dyadic(int64_t x, int k) {
    int64_t r = ONE + (x >> k);
    for (int i = 0; i < k; i++) r = o_mul(r, r);
    return r;
}

/* fp_exp: k = 14; negatives as 1 / exp(-x). fp_math.h:724-732 */
static int64_t o_exp(int64_t x) {
    if (x >= 0) return o_exp_dyadic(x, 14);
    int64_t p = o_exp_dyadic(-x, 14);
    if (p == 0) return 0;
    return o_div(ONE, p);
}

/* fp_safe_exp: clamp above at 10, zero below -10. fp_math.h:739-744 */
static int64_t o_safe_exp(int64_t x) {
    const int64_t ten = 10 * ONE;
    if (x > ten) x = ten;
    if (x < -ten) return 0;
    return o_exp(x);
}

/* fp_log: CLZ guess, up to 10 Newton rounds y - 1 + x/exp(y), stop when the step < 2 ulp
 * (the converged step is not applied). fp_math.h:752-771 */
static int64_t o_log(int64_t x) {
    if (x <= 0) return -50 * ONE;
    const int64_t ln2 = 195103586505167LL;
    int lz = __builtin_clzll((uint64_t)x);
    int64_t y = (int64_t)(63 - lz - Q) * ln2;
    for (int it = 0; it < 10; it++) {
        int64_t ey = o_exp(y);
        if (ey == 0) break;
        int64_t yn = y - ONE + o_div(x, ey);
        int64_t d = yn - y;
        if (d < 0) d = -d;
        if (d < 2) break;
        y = yn;
    }
    return y;
}

/* fp_atan_taylor. fp_math.h:785-795 */
static int64_t o_atan_taylor(int64_t x, int terms) {
    int64_t x2 = o_mul(x, x), t = x, s = x;
    for (int n = 1; n <= terms; n++) {
        t = -o_mul(t, x2);
        int64_t c = t / (2 * n + 1);
        if (c == 0) break;
        s += c;
    }
    return s;
}

/* CORDIC tables: pi by Machin, atan(2^-i) table, gain 1/sqrt(prod(1+2^-2i)).
 * fp_math.h:800-858 */
#define NCORDIC 48
static int64_t g_angles[NCORDIC], g_gain, g_pi;
static int g_init = 0;
static void o_init(void) {
    if (g_init) return;
    int64_t a5 = o_atan_taylor(ONE / 5, 40), a239 = o_atan_taylor(ONE / 239, 15);
    g_pi = (a5 << 4) - (a239 << 2);
    g_angles[0] = g_pi >> 2;
    for (int i = 1; i < NCORDIC; i++)
        g_angles[i] = i >= 25 ? (ONE >> i) : o_atan_taylor(ONE >> i, 40);
    int64_t ksq = ONE;
    for (int i = 0; i < NCORDIC; i++)
        ksq = o_mul(ksq, ONE + (2 * i < 63 ? (ONE >> (2 * i)) : 0));
    g_gain = o_div(ONE, o_sqrt(ksq));
    g_init = 1;
}

/* fp_sincos: reduce to [-pi, pi], fold to |a| <= pi/2, 48 CORDIC rotations. fp_math.h:861-902 */
static void o_sincos(int64_t a, int64_t *c, int64_t *s) {
    o_init();
    const int64_t two_pi = g_pi << 1, half_pi = g_pi >> 1;
    while (a > g_pi) a -= two_pi;
    while (a < -g_pi) a += two_pi;
    int neg = 0;
    if (a > half_pi) { a = g_pi - a; neg = 1; }
    else if (a < -half_pi) { a = -g_pi - a; neg = 1; }
    int64_t x = g_gain, y = 0, z = a;
    for (int i = 0; i < NCORDIC; i++) {
        int64_t xs = x >> i, ys = y >> i;
        if (z >= 0) { x -= ys; y += xs; z -= g_angles[i]; }
        else        { x += ys; y -= xs; z += g_angles[i]; }
    }
    *c = neg ? -x : x;
    *s = y;
}

/* fp_sigmoid / fp_silu. fp_math.h:911-921 */
static int64_t o_sigmoid(int64_t x) {
    const int64_t ten = 10 * ONE;
    if (x > ten) return ONE;
    if (x < -ten) return 0;
    return o_div(ONE, ONE + o_safe_exp(-x));
}
static int64_t o_silu(int64_t x) { return o_mul(x, o_sigmoid(x)); }

int64_t iqo_fp(int fn, int64_t x, int64_t y) {
    int64_t c, s;
    switch (fn) {
    case IQO_MUL: return o_mul(x, y);
    case IQO_DIV: return o_div(x, y);
    case IQO_SQRT: return o_sqrt(x);
    case IQO_SQRT_FAST: return o_sqrt_fast(x);
    case IQO_INV_SQRT: return o_inv_sqrt(x);
    case IQO_EXP: return o_exp(x);
    case IQO_LOG: return o_log(x);
    case IQO_COS: o_sincos(x, &c, &s); return c;
    case IQO_SIN: o_sincos(x, &c, &s); return s;
    case IQO_SIGMOID: return o_sigmoid(x);
    case IQO_SILU: return o_silu(x);
    case IQO_SAFE_EXP: return o_safe_exp(x);
    case IQO_EXP_DYADIC: return o_exp_dyadic(x, (int)y);
    default: return 0;
    }
}

void iqo_fp_vec(int fn, const int64_t *x, const int64_t *y, int64_t *out, int64_t n) {
    o_init();
    for (int64_t i = 0; i < n; i++) out[i] = iqo_fp(fn, x[i], y ? y[i] : 0);
}

/* ---------------- determinism gate restated (fp_determinism.c:43-200) ---------------- */

uint64_t iqo_fnv_mix_i64(uint64_t h, int64_t v) {
    uint64_t u = (uint64_t)v;
    for (int b = 0; b < 8; b++) { h ^= u & 0xff; h *= 1099511628211ULL; u >>= 8; }
    return h;
}

uint64_t iqo_det_hash(uint64_t subs_out[12]) {
    o_init();
    enum { CAP = 4096 + 256 };
    static int64_t grid[CAP];
    int n = 0;
    /* grid: specials, +-2^e for e in [-44, 14], 4096 xorshift values in [-32000, 32000]
     * (fp_determinism.c:101-137) */
    const int64_t sp[16] = { 0, ONE, -ONE, ONE / 2, -(ONE / 2), 1, -1, ONE + 1, ONE - 1,
                             (int64_t)32000 << Q, -((int64_t)32000 << Q), (int64_t)181 << Q,
                             7 * ONE, -7 * ONE, 2 * ONE, 10 * ONE };
    for (int i = 0; i < 16; i++) grid[n++] = sp[i];
    for (int e = -44; e <= 14; e++) {
        int64_t p = e >= 0 ? (ONE << e) : (ONE >> -e);
        grid[n++] = p; grid[n++] = -p;
    }
    uint64_t st = 0x9E3779B97F4A7C15ULL;
    const int64_t span = (int64_t)32000 << Q;
    for (int i = 0; i < 4096; i++) {
        st ^= st << 13; st ^= st >> 7; st ^= st << 17;
        int64_t mag = (int64_t)(st % (uint64_t)span);
        grid[n++] = (st & 1) ? mag : -mag;
    }
    const uint64_t H0 = 1469598103934665603ULL;
    uint64_t h[12];
    for (int i = 0; i < 12; i++) h[i] = H0;
    const int64_t forty = (int64_t)40 << Q, twenty = (int64_t)20 << Q;
    for (int i = 0; i < n; i++) {
        int64_t x = grid[i], y = grid[(i * 7 + 3) % n];
        h[0] = iqo_fnv_mix_i64(h[0], o_mul(x, y));
        if (y != 0) h[1] = iqo_fnv_mix_i64(h[1], o_div(x, y));
        int64_t xp = x < 0 ? -x : x;
        if (xp < 1024) xp += 1024;
        h[2] = iqo_fnv_mix_i64(h[2], o_sqrt(xp));
        h[3] = iqo_fnv_mix_i64(h[3], o_sqrt_fast(xp));
        h[4] = iqo_fnv_mix_i64(h[4], o_inv_sqrt(xp));
        h[6] = iqo_fnv_mix_i64(h[6], o_log(xp));
        int64_t ea = (int64_t)((uint64_t)x % (uint64_t)forty) - twenty;
        h[5] = iqo_fnv_mix_i64(h[5], o_exp(ea));
        int64_t c, s;
        o_sincos(x, &c, &s);
        h[7] = iqo_fnv_mix_i64(h[7], c);
        h[8] = iqo_fnv_mix_i64(h[8], s);
        h[9] = iqo_fnv_mix_i64(h[9], o_sigmoid(x));
        h[10] = iqo_fnv_mix_i64(h[10], o_silu(x));
    }
    /* fp_rng_next xorshift64 / fp_rng_uniform (top 48 bits). fp_math.h:928-940 */
    uint64_t rs = 0x123456789ABCDEFULL;
    for (int i = 0; i < 1024; i++) {
        rs ^= rs << 13; rs ^= rs >> 7; rs ^= rs << 17;
        h[11] = iqo_fnv_mix_i64(h[11], (int64_t)rs);
        rs ^= rs << 13; rs ^= rs >> 7; rs ^= rs << 17;
        h[11] = iqo_fnv_mix_i64(h[11], (int64_t)(rs >> 16));
    }
    uint64_t comb = H0;
    for (int i = 0; i < 12; i++) {
        comb = iqo_fnv_mix_i64(comb, (int64_t)h[i]);
        if (subs_out) subs_out[i] = h[i];
    }
    return comb;
}

/* ---------------- hot path: matmul_vec and the layer ops ---------------- */

/* Row-parallel helper: rows are independent, so splitting them across host
 * threads does not change any bit of the result. */
typedef struct { void (*fn)(void *, int, int); void *ctx; int r0, r1; } o_job;
static void *o_job_run(void *p) { o_job *j = (o_job *)p; j->fn(j->ctx, j->r0, j->r1); return NULL; }
static void o_parallel_rows(int rows, int64_t work, void (*fn)(void *, int, int), void *ctx) {
    int nt = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nt > 64) nt = 64;
    if (nt < 1 || work < (1 << 22) || rows < 2) nt = 1;
    if (nt > rows) nt = rows;
    if (nt == 1) { fn(ctx, 0, rows); return; }
    pthread_t t[64]; o_job j[64];
    for (int i = 0; i < nt; i++) {
        j[i].fn = fn; j[i].ctx = ctx;
        j[i].r0 = (int)((int64_t)rows * i / nt); j[i].r1 = (int)((int64_t)rows * (i + 1) / nt);
        pthread_create(&t[i], NULL, o_job_run, &j[i]);
    }
    for (int i = 0; i < nt; i++) pthread_join(t[i], NULL);
}

/* matmul_vec: out[i] = low64((sum_j (i128)in[j] * W[i][j]) >> 48), W row-major [M][N].
 * llama_int.c:1014-1046 (the 4-row unroll there does not change the result). */
typedef struct { int64_t *out; const int64_t *w, *in; int M, N, rows; } o_mv;
static void o_mv_rows(void *p, int r0, int r1) {
    o_mv *a = (o_mv *)p;
    for (int i = r0; i < r1; i++) {
        const int64_t *r = a->w + (int64_t)i * a->N;
        i128 acc = 0;
        for (int j = 0; j < a->N; j++) acc += (i128)a->in[j] * r[j];
        a->out[i] = (int64_t)(acc >> Q);
    }
}
void iqo_matmul_vec(int64_t *out, const int64_t *w, const int64_t *in, int M, int N) {
    o_mv a = { out, w, in, M, N, 0 };
    o_parallel_rows(M, (int64_t)M * N, o_mv_rows, &a);
}

/* rows x matmul_vec: the oracle for the batched extension (one matmul_vec per row). */
static void o_rows_rows(void *p, int r0, int r1) {
    o_mv *a = (o_mv *)p;
    for (int r = r0; r < r1; r++) {
        const int64_t *x = a->in + (int64_t)r * a->N;
        for (int i = 0; i < a->M; i++) {
            const int64_t *wr = a->w + (int64_t)i * a->N;
            i128 acc = 0;
            for (int j = 0; j < a->N; j++) acc += (i128)x[j] * wr[j];
            a->out[(int64_t)r * a->M + i] = (int64_t)(acc >> Q);
        }
    }
}
void iqo_matmul_rows(int64_t *out, const int64_t *w, const int64_t *X, int rows, int M, int N) {
    o_mv a = { out, w, X, M, N, rows };
    o_parallel_rows(rows, (int64_t)rows * M * N, o_rows_rows, &a);
}

/* rmsnorm: int128 sum of squares, (sum >> 48) / dim truncating, + eps 2814749767,
 * fp_inv_sqrt, out = fp_mul(fp_mul(x, inv), w). llama_int.c:1048-1058 */
void iqo_rmsnorm(int64_t *out, const int64_t *x, const int64_t *w, int dim) {
    i128 ss = 0;
    for (int i = 0; i < dim; i++) ss += (i128)x[i] * x[i];
    int64_t ms = (int64_t)((ss >> Q) / dim);
    ms += (int64_t)2814749767LL;
    int64_t inv = o_inv_sqrt(ms);
    for (int i = 0; i < dim; i++) out[i] = o_mul(o_mul(x[i], inv), w[i]);
}

/* softmax: max-subtract, fp_safe_exp, int64 sum, fp_div by the sum only if sum > 0.
 * llama_int.c:1060-1072 */
void iqo_softmax(int64_t *x, int n) {
    int64_t mx = x[0];
    for (int i = 1; i < n; i++) if (x[i] > mx) mx = x[i];
    int64_t sum = 0;
    for (int i = 0; i < n; i++) { x[i] = o_safe_exp(x[i] - mx); sum += x[i]; }
    if (sum > 0) for (int i = 0; i < n; i++) x[i] = o_div(x[i], sum);
}

/* rope_init: theta_i = exp(-(2i/hd) * ln(theta)), angle = pos * theta_i, CORDIC sincos;
 * table index pos*half + i. llama_int.c:960-986 */
void iqo_rope_tables(int hd, int max_seq, int theta, int64_t *cos_out, int64_t *sin_out) {
    o_init();
    int half = hd / 2;
    int64_t lt = o_log(o_from_int(theta));
    for (int i = 0; i < half; i++) {
        int64_t nf = -o_div(o_from_int(2 * i), o_from_int(hd));
        int64_t th = o_exp(o_mul(nf, lt));
        for (int p = 0; p < max_seq; p++) {
            int64_t c, s;
            o_sincos(o_mul(o_from_int(p), th), &c, &s);
            cos_out[(int64_t)p * half + i] = c;
            sin_out[(int64_t)p * half + i] = s;
        }
    }
}

/* rope_apply: half-split rotation. llama_int.c:997-1008 */
static void o_rope_apply(const int64_t *ct, const int64_t *st, int half, int64_t *v, int pos) {
    const int64_t *c = ct + (int64_t)pos * half, *s = st + (int64_t)pos * half;
    for (int i = 0; i < half; i++) {
        int64_t x0 = v[i], x1 = v[i + half];
        v[i] = o_mul(x0, c[i]) - o_mul(x1, s[i]);
        v[i + half] = o_mul(x1, c[i]) + o_mul(x0, s[i]);
    }
}

/* ---------------- model (forward / generate) ---------------- */

typedef struct {
    int dim, nh, nkv, hd, nl, inter, vocab, max_seq, theta;
    const int64_t *embed, *fnorm, *lm;
    const int64_t *const *lp; /* 9 per layer */
    int64_t *rc, *rs;         /* rope tables */
    int64_t *kc, *vc;         /* [layer][max_seq][nkv*hd] */
} omodel;

void *iqo_model_create(const int *c, const int64_t *embed, const int64_t *fnorm,
                       const int64_t *lm, const int64_t *const *lp) {
    omodel *m = (omodel *)calloc(1, sizeof(omodel));
    m->dim = c[0]; m->nh = c[1]; m->nkv = c[2]; m->hd = c[3]; m->nl = c[4];
    m->inter = c[5]; m->vocab = c[6]; m->max_seq = c[7]; m->theta = c[8];
    m->embed = embed; m->fnorm = fnorm; m->lm = lm;
    int64_t nlp = 9 * (int64_t)m->nl;
    const int64_t **cp = (const int64_t **)malloc(nlp * sizeof(*cp));
    memcpy(cp, lp, nlp * sizeof(*cp));
    m->lp = cp;
    size_t rn = (size_t)m->max_seq * (m->hd / 2);
    m->rc = (int64_t *)malloc(rn * 8); m->rs = (int64_t *)malloc(rn * 8);
    iqo_rope_tables(m->hd, m->max_seq, m->theta, m->rc, m->rs);
    size_t kn = (size_t)m->nl * m->max_seq * m->nkv * m->hd;
    m->kc = (int64_t *)calloc(kn, 8); m->vc = (int64_t *)calloc(kn, 8);
    return m;
}

void iqo_model_reset(void *h) {
    omodel *m = (omodel *)h;
    size_t kn = (size_t)m->nl * m->max_seq * m->nkv * m->hd;
    memset(m->kc, 0, kn * 8); memset(m->vc, 0, kn * 8);
}

/* transformer_layer_forward, exact KV path. llama_int.c:1326-1569 */
static void o_layer(omodel *m, int64_t *hid, int l, int pos, int64_t *sc) {
    const int64_t *const *w = m->lp + 9 * l;
    int dim = m->dim, hd = m->hd, nkv = m->nkv, kvd = nkv * hd, inter = m->inter;
    int grp = m->nh / nkv;
    int64_t *nrm = sc, *q = nrm + dim, *k = q + dim, *v = k + kvd, *att = v + kvd,
            *o = att + dim, *g = o + dim, *u = g + inter, *mlp = u + inter, *scr = mlp + dim;
    iqo_rmsnorm(nrm, hid, w[0], dim);
    iqo_matmul_vec(q, w[1], nrm, dim, dim);
    iqo_matmul_vec(k, w[2], nrm, kvd, dim);
    iqo_matmul_vec(v, w[3], nrm, kvd, dim);
    for (int h = 0; h < m->nh; h++) o_rope_apply(m->rc, m->rs, hd / 2, q + h * hd, pos);
    for (int h = 0; h < nkv; h++) o_rope_apply(m->rc, m->rs, hd / 2, k + h * hd, pos);
    size_t base = (size_t)l * m->max_seq;
    memcpy(m->kc + (base + pos) * kvd, k, kvd * 8);
    memcpy(m->vc + (base + pos) * kvd, v, kvd * 8);
    int64_t scale = o_inv_sqrt(o_from_int(hd));
    int T = pos + 1;
    for (int h = 0; h < m->nh; h++) {
        int kh = h / grp;
        const int64_t *qh = q + h * hd;
        for (int t = 0; t < T; t++) {
            const int64_t *kt = m->kc + (base + t) * kvd + kh * hd;
            i128 dot = 0;
            for (int d = 0; d < hd; d++) dot += (i128)qh[d] * kt[d];
            scr[t] = o_mul((int64_t)(dot >> Q), scale);
        }
        iqo_softmax(scr, T);
        int64_t *ah = att + h * hd;
        memset(ah, 0, hd * 8);
        for (int t = 0; t < T; t++) {
            const int64_t *vt = m->vc + (base + t) * kvd + kh * hd;
            for (int d = 0; d < hd; d++) ah[d] += o_mul(scr[t], vt[d]);
        }
    }
    iqo_matmul_vec(o, w[4], att, dim, dim);
    for (int i = 0; i < dim; i++) hid[i] += o[i];
    iqo_rmsnorm(nrm, hid, w[5], dim);
    iqo_matmul_vec(g, w[6], nrm, inter, dim);
    iqo_matmul_vec(u, w[7], nrm, inter, dim);
    for (int i = 0; i < inter; i++) g[i] = o_mul(o_silu(g[i]), u[i]);
    iqo_matmul_vec(mlp, w[8], g, dim, inter);
    for (int i = 0; i < dim; i++) hid[i] += mlp[i];
}

/* llama_forward: bounds checks, embedding row, layers, final norm, LM head.
 * Returns argmax (first max, llama_int.c:2888-2893) or -1 on a rejected token/pos.
 * llama_int.c:2807-2886 */
int iqo_model_forward(void *h, int token, int pos, int64_t *logits_out) {
    omodel *m = (omodel *)h;
    if (token < 0 || token >= m->vocab || pos < 0 || pos >= m->max_seq) return -1;
    int dim = m->dim, kvd = m->nkv * m->hd;
    size_t scn = (size_t)dim * 6 + 2 * (size_t)kvd + 2 * (size_t)m->inter + (size_t)m->max_seq;
    int64_t *sc = (int64_t *)malloc(scn * 8);
    int64_t *hid = (int64_t *)malloc((size_t)dim * 8);
    memcpy(hid, m->embed + (int64_t)token * dim, (size_t)dim * 8);
    for (int l = 0; l < m->nl; l++) o_layer(m, hid, l, pos, sc);
    int64_t *nrm = sc;
    iqo_rmsnorm(nrm, hid, m->fnorm, dim);
    int64_t *lg = logits_out ? logits_out : (int64_t *)malloc((size_t)m->vocab * 8);
    iqo_matmul_vec(lg, m->lm, nrm, m->vocab, dim);
    int best = 0;
    for (int i = 1; i < m->vocab; i++) if (lg[i] > lg[best]) best = i;
    if (!logits_out) free(lg);
    free(sc); free(hid);
    return best;
}

/* generate, greedy: reset KV, prefill every prompt position (sample only at the last),
 * decode i = 1..max_new-1, stop on EOS = 2. llama_int.c:3067-3135.
 * logit_hash_out: FNV-1a over every logit of every forward call, in call order. */
int iqo_model_generate(void *h, const int *prompt, int plen, int max_new, int *out,
                       uint64_t *logit_hash_out) {
    omodel *m = (omodel *)h;
    iqo_model_reset(m);
    int64_t *lg = (int64_t *)malloc((size_t)m->vocab * 8);
    uint64_t lh = 1469598103934665603ULL;
    memcpy(out, prompt, (size_t)plen * sizeof(int));
    int total = plen;
    for (int p = 0; p < plen; p++) {
        int a = iqo_model_forward(m, out[p], p, lg);
        if (a < 0) { free(lg); return -1; }
        for (int i = 0; i < m->vocab; i++) lh = iqo_fnv_mix_i64(lh, lg[i]);
        if (p == plen - 1) out[total++] = a;
    }
    for (int i = 1; i < max_new; i++) {
        int p = plen + i - 1;
        int a = iqo_model_forward(m, out[p], p, lg);
        if (a < 0) break;
        for (int j = 0; j < m->vocab; j++) lh = iqo_fnv_mix_i64(lh, lg[j]);
        if (a == 2) break;
        out[total++] = a;
    }
    free(lg);
    if (logit_hash_out) *logit_hash_out = lh;
    return total;
}

void iqo_model_free(void *h) {
    omodel *m = (omodel *)h;
    if (!m) return;
    free((void *)m->lp); free(m->rc); free(m->rs); free(m->kc); free(m->vc); free(m);
}

/* ---------------- synthetic inputs ---------------- */

/* bfloat16_to_q1648: +-(128 + mantissa) * 2^(e - 86), truncating right shifts,
 * exponent 0 -> 0, exponent 255 -> +-32000.0, shifts outside (-64, 64) -> 0.
 * safetensors.h:115-152 */
int64_t iqo_bf16_to_q1648(uint16_t b) {
    int sgn = (b >> 15) & 1, e = (b >> 7) & 0xFF, man = b & 0x7F;
    if (e == 0 && man == 0) return 0;
    if (e == 0xFF) return sgn ? -((int64_t)32000 << Q) : ((int64_t)32000 << Q);
    int64_t r;
    if (e == 0) r = 0;
    else {
        int sh = e - 86;
        int64_t sig = 128 + man;
        if (sh >= 0 && sh < 64) r = (int64_t)((uint64_t)sig << sh);
        else if (sh < 0 && sh > -64) r = sig >> -sh;
        else r = 0;
    }
    return sgn ? -r : r;
}

/* round-to-nearest-even of a Q16.48 value to bf16 bits (8 significant bits). */
uint16_t iqo_q1648_to_bf16_rne(int64_t w) {
    if (w == 0) return 0;
    uint16_t sgn = w < 0 ? 0x8000 : 0;
    uint64_t mag = w < 0 ? (uint64_t)0 - (uint64_t)w : (uint64_t)w;
    int p = 63 - __builtin_clzll(mag);
    uint64_t sig;
    if (p <= 7) sig = mag << (7 - p);
    else {
        int drop = p - 7;
        sig = mag >> drop;
        uint64_t rem = mag & (((uint64_t)1 << drop) - 1), half = (uint64_t)1 << (drop - 1);
        if (rem > half || (rem == half && (sig & 1))) sig++;
        if (sig == 256) { sig = 128; p++; }
    }
    return (uint16_t)(sgn | ((uint16_t)(p + 79) << 7) | (uint16_t)(sig - 128));
}

uint64_t iqo_fnv1a64(const char *s) {
    uint64_t h = 1469598103934665603ULL;
    for (; *s; s++) { h ^= (uint8_t)*s; h *= 1099511628211ULL; }
    return h;
}

uint64_t iqo_tensor_seed(int cfg, const char *name) {
    return 0x494E544C4C4D0000ULL ^ ((uint64_t)(uint32_t)cfg << 32) ^ iqo_fnv1a64(name);
}

/* xoroshiro128+ seeded by SplitMix64. llama_int.c:2909-2929 */
typedef struct { uint64_t s0, s1; } orng;
static void r_seed(orng *r, uint64_t seed) {
    uint64_t z = seed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    r->s0 = z ^ (z >> 31);
    z = seed + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    r->s1 = z ^ (z >> 31);
    if (!r->s0 && !r->s1) r->s0 = 1;
}
static inline uint64_t r_next(orng *r) {
    uint64_t a = r->s0, b = r->s1, res = a + b;
    b ^= a;
    r->s0 = ((a << 55) | (a >> 9)) ^ b ^ (b << 14);
    r->s1 = (b << 36) | (b >> 28);
    return res;
}

/* weights: CLT-12 Gaussian (fp_math.h:944-952 shape), sigma 0.02 via fp_mul,
 * RNE to bf16, exact bf16 -> Q16.48. */
void iqo_synth_weights(uint64_t seed, int64_t *out, int64_t n) {
    orng r; r_seed(&r, seed);
    for (int64_t i = 0; i < n; i++) {
        int64_t g = 0;
        for (int k = 0; k < 12; k++) g += (int64_t)(r_next(&r) >> 16);
        g -= 6 * ONE;
        out[i] = iqo_bf16_to_q1648(iqo_q1648_to_bf16_rne(o_mul(5629499534213LL, g)));
    }
}

/* activations: uniform [-8, 8) with full 48-bit fractions. */
void iqo_synth_acts(uint64_t seed, int64_t *out, int64_t n) {
    orng r; r_seed(&r, seed);
    for (int64_t i = 0; i < n; i++) out[i] = (int64_t)(r_next(&r) >> 12) - ((int64_t)1 << 51);
}

void iqo_synth_tokens(uint64_t seed, int *out, int n, int vocab) {
    orng r; r_seed(&r, seed);
    for (int i = 0; i < n; i++) out[i] = (int)(r_next(&r) % (uint64_t)vocab);
}

/* FNV-1a 64 continued over n little-endian int64 values (fp_determinism.c:43-56). */
uint64_t iqo_fnv_array(uint64_t h, const int64_t *v, int64_t n) {
    for (int64_t i = 0; i < n; i++) h = iqo_fnv_mix_i64(h, v[i]);
    return h;
}

/* ---------------- sampling ---------------- */

/* first maximum (strict >). llama_int.c:2888-2893 */
static int o_argmax(const int64_t *v, int n) {
    int b = 0;
    for (int i = 1; i < n; i++) if (v[i] > v[b]) b = i;
    return b;
}
static int o_cmp_desc(const void *a, const void *b) {
    int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return (y > x) - (y < x);
}

/* sample_token (llama_int.c:2958-3039): below a temperature of 0.01 the argmax;
 * else work = fp_div(logit, T); top-k keeps values >= the k-th largest (others
 * INT64_MIN / 2); softmax; top-p keeps the largest probabilities (first index
 * among equals) until their running int64 sum reaches p, zeroes the rest and
 * renormalises with fp_div; then the first index whose running sum exceeds
 * r = xoroshiro128+ >> 16, else the argmax of the probabilities.
 * rng: the generator state {s0, s1}, advanced once per sampled token. */
int iqo_sample_token(const int64_t *logits, int V, int64_t temp, int top_k, int64_t top_p, uint64_t rng[2]) {
    if (temp <= 0 || temp < ONE / 100) return o_argmax(logits, V);
    int64_t *w = (int64_t *)malloc((size_t)V * 8);
    for (int i = 0; i < V; i++) w[i] = o_div(logits[i], temp);
    if (top_k > 0 && top_k < V) {
        int64_t *srt = (int64_t *)malloc((size_t)V * 8);
        memcpy(srt, w, (size_t)V * 8);
        qsort(srt, (size_t)V, 8, o_cmp_desc);
        const int64_t thr = srt[top_k - 1];
        free(srt);
        for (int i = 0; i < V; i++) if (w[i] < thr) w[i] = INT64_MIN / 2;
    }
    iqo_softmax(w, V);
    if (top_p > 0 && top_p < ONE) {
        int64_t cum = 0;
        while (cum < top_p) {
            int best = -1;
            for (int i = 0; i < V; i++) {
                if (w[i] <= 0) continue;
                if (best < 0 || w[i] > w[best]) best = i;
            }
            if (best < 0) break;
            cum += w[best];
            w[best] = -w[best];
        }
        for (int i = 0; i < V; i++) w[i] = w[i] < 0 ? -w[i] : 0;
        int64_t sum = 0;
        for (int i = 0; i < V; i++) sum += w[i];
        if (sum > 0) for (int i = 0; i < V; i++) if (w[i] > 0) w[i] = o_div(w[i], sum);
    }
    orng r = {rng[0], rng[1]};
    const int64_t thr = (int64_t)(r_next(&r) >> 16);
    rng[0] = r.s0;
    rng[1] = r.s1;
    int64_t cum = 0;
    int sel = -1;
    for (int i = 0; i < V; i++) {
        cum += w[i];
        if (cum > thr) { sel = i; break; }
    }
    if (sel < 0) sel = o_argmax(w, V);
    free(w);
    return sel;
}

/* rng_seed (llama_int.c:2909-2919) into {s0, s1}. */
void iqo_rng_seed(uint64_t seed, uint64_t rng[2]) {
    orng r;
    r_seed(&r, seed);
    rng[0] = r.s0;
    rng[1] = r.s1;
}

/* generate() with sampling parameters (llama_int.c:3067-3135 with sp != NULL):
 * the generator is seeded once (rng_seed), every prefill-end and decode sample
 * goes through sample_token, EOS stops. */
int iqo_model_generate_sampled(void *h, const int *prompt, int plen, int max_new, int64_t temp, int top_k,
                               int64_t top_p, uint64_t seed, int *out, uint64_t *logit_hash_out) {
    omodel *m = (omodel *)h;
    iqo_model_reset(m);
    uint64_t rng[2];
    iqo_rng_seed(seed, rng);
    int64_t *lg = (int64_t *)malloc((size_t)m->vocab * 8);
    uint64_t lh = 1469598103934665603ULL;
    memcpy(out, prompt, (size_t)plen * sizeof(int));
    int total = plen;
    for (int p = 0; p < plen; p++) {
        if (iqo_model_forward(m, out[p], p, lg) < 0) { free(lg); return -1; }
        for (int i = 0; i < m->vocab; i++) lh = iqo_fnv_mix_i64(lh, lg[i]);
        if (p == plen - 1) out[total++] = iqo_sample_token(lg, m->vocab, temp, top_k, top_p, rng);
    }
    for (int i = 1; i < max_new; i++) {
        int p = plen + i - 1;
        if (iqo_model_forward(m, out[p], p, lg) < 0) break;
        for (int j = 0; j < m->vocab; j++) lh = iqo_fnv_mix_i64(lh, lg[j]);
        int a = iqo_sample_token(lg, m->vocab, temp, top_k, top_p, rng);
        if (a == 2) break;
        out[total++] = a;
    }
    free(lg);
    if (logit_hash_out) *logit_hash_out = lh;
    return total;
}
