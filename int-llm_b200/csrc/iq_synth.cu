// iq_synth.cu -- seeded synthetic inputs for the benchmark configurations
// (host code). Weights follow the reference's own value path: a CLT-12
// Gaussian (shape of fp_gaussian, fp_math.h:944-952) from xoroshiro128+
// seeded by SplitMix64 (llama_int.c:2909-2929), scaled by sigma = 0.02 with
// fp_mul, rounded to nearest-even bf16 and converted exactly to Q16.48 with
// the bfloat16_to_q1648 rule (safetensors.h:115-152). No device work.
#include <stdint.h>
#include <string.h>
#include "../../include/iq.h"

namespace {
struct Xoro { uint64_t s0, s1; };
void xseed(Xoro *r, uint64_t seed) {
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
inline uint64_t xnext(Xoro *r) {
    uint64_t a = r->s0, b = r->s1, out = a + b;
    b ^= a;
    r->s0 = ((a << 55) | (a >> 9)) ^ b ^ (b << 14);
    r->s1 = (b << 36) | (b >> 28);
    return out;
}
inline int64_t mul_q48(int64_t a, int64_t b) { return (int64_t)(((__int128)a * b) >> 48); }
}  // namespace

extern "C" {

IQ_API int iq_rng_seed(uint64_t seed, uint64_t state[2]) {
    if (!state) return IQ_ERR_ARG;
    Xoro r;
    xseed(&r, seed);
    state[0] = r.s0;
    state[1] = r.s1;
    return IQ_OK;
}

IQ_API uint16_t iq_q1648_to_bf16(int64_t w) {
    if (w == 0) return 0;
    uint16_t sgn = w < 0 ? 0x8000 : 0;
    uint64_t mag = w < 0 ? (uint64_t)0 - (uint64_t)w : (uint64_t)w;
    int p = 63 - __builtin_clzll(mag);
    uint64_t sig;
    if (p <= 7) {
        sig = mag << (7 - p);
    } else {
        int drop = p - 7;
        sig = mag >> drop;
        uint64_t rem = mag & ((1ull << drop) - 1), half = 1ull << (drop - 1);
        if (rem > half || (rem == half && (sig & 1))) sig++;
        if (sig == 256) { sig = 128; p++; }
    }
    return (uint16_t)(sgn | (uint16_t)((p + 79) << 7) | (uint16_t)(sig - 128));
}

IQ_API int64_t iq_bf16_to_q1648(uint16_t b) {
    int s = (b >> 15) & 1, e = (b >> 7) & 0xFF, m = b & 0x7F;
    if (e == 0 && m == 0) return 0;
    if (e == 0xFF) return s ? -((int64_t)32000 << 48) : ((int64_t)32000 << 48);
    int64_t r = 0;
    if (e != 0) {
        int sh = e - 86;
        int64_t sig = 128 + m;
        if (sh >= 0 && sh < 64) r = (int64_t)((uint64_t)sig << sh);
        else if (sh < 0 && sh > -64) r = sig >> -sh;
    }
    return s ? -r : r;
}

IQ_API uint64_t iq_tensor_seed(int config_index, const char *name) {
    uint64_t h = 1469598103934665603ULL;
    for (const char *p = name; p && *p; p++) { h ^= (uint8_t)*p; h *= 1099511628211ULL; }
    return 0x494E544C4C4D0000ULL ^ ((uint64_t)(uint32_t)config_index << 32) ^ h;
}

IQ_API int iq_synth_weights(uint64_t seed, int64_t *out, int64_t n) {
    if (!out || n < 0) return IQ_ERR_ARG;
    Xoro r;
    xseed(&r, seed);
    const int64_t one = (int64_t)1 << 48;
    for (int64_t i = 0; i < n; i++) {
        int64_t g = 0;
        for (int k = 0; k < 12; k++) g += (int64_t)(xnext(&r) >> 16);
        g -= 6 * one;
        out[i] = iq_bf16_to_q1648(iq_q1648_to_bf16(mul_q48(5629499534213LL, g)));
    }
    return IQ_OK;
}

IQ_API int iq_synth_acts(uint64_t seed, int64_t *out, int64_t n) {
    if (!out || n < 0) return IQ_ERR_ARG;
    Xoro r;
    xseed(&r, seed);
    for (int64_t i = 0; i < n; i++) out[i] = (int64_t)(xnext(&r) >> 12) - ((int64_t)1 << 51);
    return IQ_OK;
}

IQ_API int iq_synth_tokens(uint64_t seed, int *out, int n, int vocab) {
    if (!out || n < 0 || vocab <= 0) return IQ_ERR_ARG;
    Xoro r;
    xseed(&r, seed);
    for (int i = 0; i < n; i++) out[i] = (int)(xnext(&r) % (uint64_t)vocab);
    return IQ_OK;
}

}  // extern "C"
