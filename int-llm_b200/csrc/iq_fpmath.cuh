// iq_fpmath.cuh -- bit-exact device ports of the fp_math.h primitives on the
// llama_int path. Each function restates the reference algorithm (fp_math.h
// line ranges cited) with device integer arithmetic; results must equal the
// reference bit for bit, which tests pin with the determinism-gate grid
// (fp_determinism.c:162-200, golden c0d933ea340452ec).
//
// The one piece of arithmetic the reference gets from the compiler is the
// signed 128-bit truncating division (fp_math.h:258-265). It is written here
// as u128 / u64 long division in base 2^32 (Knuth, TAOCP vol. 2, 4.3.1,
// Algorithm D, in the two-digit form of Warren, Hacker's Delight, 9-4
// "divlu"); digit estimates use the plain 64-bit `/` and `%` operators.
#pragma once
#include "iq_common.cuh"

namespace iq {

// ---- 128-bit helpers ----------------------------------------------------

__device__ __forceinline__ int d_clz64(uint64_t v) { return __clzll((long long)v); }

// floor((a*b) / 2^48), low 64 bits: fp_mul (fp_math.h:491-506).
__device__ __forceinline__ int64_t d_mul(int64_t a, int64_t b) {
    uint64_t lo = (uint64_t)a * (uint64_t)b;
    int64_t hi = __mul64hi(a, b);
    return (int64_t)(((uint64_t)hi << 16) | (lo >> 48));
}

// 128 / 64 -> 64 for a normalised case: requires u1 < v (quotient fits 64 bits).
// Two base-2^32 digit steps with the Algorithm D qhat correction.
__device__ __forceinline__ uint64_t d_divlu(uint64_t u1, uint64_t u0, uint64_t v, uint64_t *rem) {
    const uint64_t b = 1ull << 32;
    int s = d_clz64(v);
    v <<= s;
    uint64_t vn1 = v >> 32, vn0 = v & 0xffffffffull;
    uint64_t un32 = s ? ((u1 << s) | (u0 >> (64 - s))) : u1;
    uint64_t un10 = u0 << s;
    uint64_t un1 = un10 >> 32, un0 = un10 & 0xffffffffull;
    uint64_t q1 = un32 / vn1, rhat = un32 - q1 * vn1;
    while (q1 >= b || q1 * vn0 > ((rhat << 32) | un1)) {
        q1--; rhat += vn1;
        if (rhat >= b) break;
    }
    uint64_t un21 = (un32 << 32) + un1 - q1 * v;
    uint64_t q0 = un21 / vn1;
    rhat = un21 - q0 * vn1;
    while (q0 >= b || q0 * vn0 > ((rhat << 32) | un0)) {
        q0--; rhat += vn1;
        if (rhat >= b) break;
    }
    if (rem) *rem = ((un21 << 32) + un0 - q0 * v) >> s;
    return (q1 << 32) | q0;
}

// unsigned 128 / 64 -> 128 (v != 0).
__device__ __forceinline__ u128 d_udiv128_64(u128 n, uint64_t v) {
    uint64_t hi = (uint64_t)(n >> 64), lo = (uint64_t)n;
    uint64_t qh = 0;
    if (hi >= v) { qh = hi / v; hi = hi % v; }
    uint64_t ql = d_divlu(hi, lo, v, nullptr);
    return ((u128)qh << 64) | ql;
}

// signed truncating 128 / int64 (fp_w_divs, fp_math.h:258-265, divisor in int64 range).
__device__ __forceinline__ i128 d_sdiv128_64(i128 a, int64_t b) {
    bool na = a < 0, nb = b < 0;
    u128 ua = na ? (u128)0 - (u128)a : (u128)a;
    uint64_t ub = nb ? (uint64_t)0 - (uint64_t)b : (uint64_t)b;
    u128 q = d_udiv128_64(ua, ub);
    return (na != nb) ? (i128)((u128)0 - q) : (i128)q;
}

// fp_div (fp_math.h:508-524): sign-magnitude |a| << 48, truncating divide,
// q = floor(|a| 2^48 / |b|) with the sign of a b.
// Fast path: a double estimate of the quotient (three roundings of relative
// size 2^-53 each: |a|, |b| and the quotient) is within 3/8 of the exact value
// while it is below 2^50, so its truncation is q - 1, q or q + 1; one exact
// remainder r = |a| 2^48 - q' |b| (|r| < 2 |b| < 2^62, so its low 64 bits are
// exact) picks q. Larger quotients or divisors take the 128 / 64 long division.
// b == 0 never occurs on the reference path (its callers guard it); 0 is returned.
__device__ __forceinline__ int64_t d_div(int64_t a, int64_t b) {
    if (b == 0) return 0;
    uint64_t ma = a < 0 ? (uint64_t)0 - (uint64_t)a : (uint64_t)a;
    uint64_t mb = b < 0 ? (uint64_t)0 - (uint64_t)b : (uint64_t)b;
    uint64_t ql;
    const double qd = (double)ma * 281474976710656.0 / (double)mb;   // 2^48 |a| / |b|
    if (qd < 1125899906842624.0 && mb < (1ull << 61)) {              // 2^50
        ql = (uint64_t)qd;
        const int64_t r = (int64_t)((ma << 48) - ql * mb);
        if (r < 0) ql--;
        else if ((uint64_t)r >= mb) ql++;
    } else {
        // |a| << 48 as (hi, lo): hi < 2^47 so the 128/64 division has hi < mb or not.
        ql = (uint64_t)d_udiv128_64((u128)ma << 48, mb);
    }
    return ((a < 0) != (b < 0)) ? (int64_t)((uint64_t)0 - ql) : (int64_t)ql;
}

__device__ __forceinline__ int64_t d_from_int(int x) {
    return (int64_t)((uint64_t)(int64_t)x << 48);
}

// ---- roots ------------------------------------------------------------

// fp_sqrt_fast (fp_math.h:605-620)
__device__ __forceinline__ int64_t d_sqrt_fast(int64_t x) {
    if (x <= 0) return 0;
    uint64_t ux = (uint64_t)x;
    int bw = 64 - d_clz64(ux);
    uint64_t r = 1ull << ((bw + 1) / 2);
    for (int i = 0; i < 5; i++) {
        uint64_t nr = (r + ux / r) >> 1;
        if (nr >= r) break;
        r = nr;
    }
    return (int64_t)(r << 24);
}

// fp_sqrt (fp_math.h:624-650): Newton on isqrt(x << 48), 7 rounds, r^2 <= n fix-up.
__device__ __forceinline__ int64_t d_sqrt(int64_t x) {
    if (x <= 0) return 0;
    u128 n = (u128)(uint64_t)x << 48;
    uint64_t nh = (uint64_t)(n >> 64);
    int bw = nh ? 128 - d_clz64(nh) : 64 - d_clz64((uint64_t)n);
    uint64_t r = 1ull << ((bw + 1) / 2);
    for (int i = 0; i < 7; i++) {
        if (r == 0) return 0;
        uint64_t q = (uint64_t)d_udiv128_64(n, r);
        uint64_t nr = (r + q) >> 1;
        if (nr >= r) break;
        r = nr;
    }
    while ((i128)(int64_t)r * (int64_t)r > (i128)n) r--;
    return (int64_t)r;
}

// fp_inv_sqrt (fp_math.h:658-707)
__device__ __forceinline__ int64_t d_inv_sqrt(int64_t x) {
    if (x <= 0) return 0;
    int msb = 63 - d_clz64((uint64_t)x);
    int k = (msb - 48) >> 1;
    int64_t xn = k >= 0 ? (x >> (2 * k)) : (int64_t)((uint64_t)x << (-2 * k));
    int msbn = 63 - d_clz64((uint64_t)xn);
    int64_t y = msbn == 48 ? IQ_ONE : (IQ_ONE >> 1);
    const int64_t three = 3 * IQ_ONE;
    for (int i = 0; i < 8; i++) {
        int64_t y2 = d_mul(y, y);
        int64_t xy2 = d_mul(xn, y2);
        int64_t f = three - xy2;
        // asr by 49 of the signed product
        uint64_t lo = (uint64_t)y * (uint64_t)f;
        int64_t hi = __mul64hi(y, f);
        y = (int64_t)(((uint64_t)hi << 15) | (lo >> 49));
        if (y <= 0) { y = 1; break; }
    }
    if (k >= 0) {
        int64_t r = y >> k;
        return r < 0 ? 0 : r;
    }
    int sh = -k;  // 1..24: y << sh as a 128-bit value, saturate to INT64_MAX
    i128 r = (i128)((u128)(i128)y << sh);
    if (r > (i128)INT64_MAX) return INT64_MAX;
    if (r < 0) return 0;
    return (int64_t)r;
}

// ---- exp / log --------------------------------------------------------

// fp_mul(r, r) (fp_math.h:491-506) from the unsigned square of |r|: r r = |r|^2,
// so the low 64 bits of |r|^2 >> 48 are the same value.
__device__ __forceinline__ int64_t d_sqr(int64_t r) {
    const uint64_t m = r < 0 ? (uint64_t)0 - (uint64_t)r : (uint64_t)r;
    return (int64_t)(((m * m) >> 48) | (__umul64hi(m, m) << 16));
}

// fp_exp_dyadic (fp_math.h:714-720)
__device__ __forceinline__ int64_t d_exp_dyadic(int64_t x, int k) {
    int64_t r = IQ_ONE + (x >> k);
    for (int i = 0; i < k; i++) r = d_sqr(r);
    return r;
}

// fp_exp (fp_math.h:724-732)
__device__ __forceinline__ int64_t d_exp(int64_t x) {
    if (x >= 0) return d_exp_dyadic(x, 14);
    int64_t p = d_exp_dyadic(-x, 14);
    if (p == 0) return 0;
    return d_div(IQ_ONE, p);
}

// fp_safe_exp (fp_math.h:739-744)
__device__ __forceinline__ int64_t d_safe_exp(int64_t x) {
    const int64_t ten = 10 * IQ_ONE;
    if (x > ten) x = ten;
    if (x < -ten) return 0;
    return d_exp(x);
}

// fp_log (fp_math.h:752-771)
__device__ __forceinline__ int64_t d_log(int64_t x) {
    if (x <= 0) return -50 * IQ_ONE;
    const int64_t ln2 = 195103586505167LL;
    int lz = d_clz64((uint64_t)x);
    int64_t y = (int64_t)(63 - lz - 48) * ln2;
    for (int i = 0; i < 10; i++) {
        int64_t ey = d_exp(y);
        if (ey == 0) break;
        int64_t yn = y - IQ_ONE + d_div(x, ey);
        int64_t d = yn - y;
        if (d < 0) d = -d;
        if (d < 2) break;
        y = yn;
    }
    return y;
}

// ---- CORDIC -----------------------------------------------------------

struct CordicTables {
    int64_t angles[48];
    int64_t gain;
    int64_t pi;
};

// fp_atan_taylor (fp_math.h:785-795)
__device__ __forceinline__ int64_t d_atan_taylor(int64_t x, int terms) {
    int64_t x2 = d_mul(x, x), t = x, s = x;
    for (int n = 1; n <= terms; n++) {
        t = -d_mul(t, x2);
        int64_t c = t / (2 * n + 1);
        if (c == 0) break;
        s += c;
    }
    return s;
}

// fp_math_init (fp_math.h:833-858): pi by Machin, atan(2^-i), CORDIC gain.
__device__ inline void d_cordic_init(CordicTables *t) {
    int64_t a5 = d_atan_taylor(IQ_ONE / 5, 40), a239 = d_atan_taylor(IQ_ONE / 239, 15);
    t->pi = (int64_t)(((uint64_t)a5 << 4) - ((uint64_t)a239 << 2));
    t->angles[0] = t->pi >> 2;
    for (int i = 1; i < 48; i++) t->angles[i] = i >= 25 ? (IQ_ONE >> i) : d_atan_taylor(IQ_ONE >> i, 40);
    int64_t ksq = IQ_ONE;
    for (int i = 0; i < 48; i++) ksq = d_mul(ksq, IQ_ONE + (2 * i < 63 ? (IQ_ONE >> (2 * i)) : 0));
    t->gain = d_div(IQ_ONE, d_sqrt(ksq));
}

// fp_sincos (fp_math.h:861-902)
__device__ __forceinline__ void d_sincos(const CordicTables &t, int64_t a, int64_t *c, int64_t *s) {
    const int64_t pi = t.pi, two_pi = pi << 1, half_pi = pi >> 1;
    while (a > pi) a -= two_pi;
    while (a < -pi) a += two_pi;
    bool neg = false;
    if (a > half_pi) { a = pi - a; neg = true; }
    else if (a < -half_pi) { a = -pi - a; neg = true; }
    int64_t x = t.gain, y = 0, z = a;
#pragma unroll 4
    for (int i = 0; i < 48; i++) {
        int64_t xs = x >> i, ys = y >> i;
        if (z >= 0) { x -= ys; y += xs; z -= t.angles[i]; }
        else        { x += ys; y -= xs; z += t.angles[i]; }
    }
    *c = neg ? -x : x;
    *s = y;
}

// ---- activations ------------------------------------------------------

// fp_sigmoid / fp_silu (fp_math.h:911-921)
__device__ __forceinline__ int64_t d_sigmoid(int64_t x) {
    const int64_t ten = 10 * IQ_ONE;
    if (x > ten) return IQ_ONE;
    if (x < -ten) return 0;
    return d_div(IQ_ONE, IQ_ONE + d_safe_exp(-x));
}
__device__ __forceinline__ int64_t d_silu(int64_t x) { return d_mul(x, d_sigmoid(x)); }

}  // namespace iq
