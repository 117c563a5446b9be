/*
 * kq_oracle.c -- CPU restatement of the Q4_K / Q6_K decode, the f64 reference matvec and the
 * counter-based synthetic generator. TEST INFRASTRUCTURE ONLY (see kq_oracle.h).
 *
 * Compiled with -ffp-contract=off: every float operation below is one IEEE binary32 (or
 * binary64) operation, rounded to nearest even, in the order written.
 */
#include "kq_oracle.h"

#include <math.h>
#include <string.h>

/* ---------------------------------------------------------------- fp16 <-> f32 (bit level) */

static float bits_f32(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint32_t f32_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

/* Exact widening, as kernite's f16::to_f32 (crates/cuda/src/half.rs:62-78): a normal number
 * re-biases its exponent (15 -> 127) and shifts its 10 fraction bits up by 13; a subnormal
 * (exponent 0) is normalised so that its leading one becomes the implicit bit. */
float kqo_fp16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t frac = h & 0x3ffu;
    if (exp == 0) {
        if (frac == 0) return bits_f32(sign);
        /* value = frac * 2^-24; highest set bit `top` gives exponent top - 24. */
        int top = 31 - __builtin_clz(frac);
        uint32_t e = (uint32_t)(top - 24 + 127);
        uint32_t m = (frac << (23 - top)) & 0x7fffffu;
        return bits_f32(sign | (e << 23) | m);
    }
    if (exp == 0x1f) return bits_f32(sign | 0x7f800000u | (frac << 13));
    return bits_f32(sign | ((exp + 112u) << 23) | (frac << 13));
}

/* Round-to-nearest-even narrowing. The generator uses it on values in [2^-12, 2^-6], all normal
 * in binary16; the general cases are kept so that the unit tests can sweep it. */
uint16_t kqo_f32_to_fp16(float x) {
    uint32_t u = f32_bits(x);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    int32_t exp = (int32_t)((u >> 23) & 0xffu);
    uint32_t frac = u & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (frac ? (0x200u | (frac >> 13)) : 0u));
    int32_t e = exp - 127 + 15; /* biased binary16 exponent */
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    uint32_t mant; /* significand with its implicit bit, 24 bits */
    int shift;     /* bits dropped from `mant` */
    if (e >= 1) {
        mant = frac | 0x800000u;
        shift = 13;
    } else {
        if (e < -10) return sign; /* below half the smallest subnormal: rounds to zero */
        mant = frac | 0x800000u;
        shift = 14 - e; /* 14..24 */
    }
    uint32_t kept = mant >> shift;
    uint32_t rest = mant & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rest > half || (rest == half && (kept & 1u))) kept += 1u;
    if (e >= 1) {
        /* kept includes the implicit bit at position 10; a carry past 11 bits bumps the
         * exponent, which the addition below does by itself. */
        uint32_t bits = ((uint32_t)e << 10) + (kept - 0x400u);
        if (bits >= 0x7c00u) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | bits);
    }
    return (uint16_t)(sign | kept); /* subnormal, or the smallest normal after a carry */
}

/* ---------------------------------------------------------------- Q4_K */

/* GGML Q4_K scale packing: bytes 0-3 hold scale j (low 6 bits) for j < 4 and the top 2 bits of
 * scale j+4; bytes 4-7 hold min j (low 6 bits) for j < 4 and the top 2 bits of min j+4; bytes
 * 8-11 hold the low 4 bits of scale j+4 (low nibble) and min j+4 (high nibble). */
void kqo_q4k_scale_min(const uint8_t s[12], int j, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = s[j] & 63u;
        *m = s[j + 4] & 63u;
    } else {
        *sc = (uint8_t)((s[j + 4] & 0x0fu) | ((s[j - 4] >> 6) << 4));
        *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* 256 weights of chunk c (0..3) of 64: qs[32c + l] low nibble is element 64c + l (sub-block 2c),
 * its high nibble element 64c + 32 + l (sub-block 2c + 1). */
void kqo_dequant_q4k(const uint8_t* blocks, size_t n, float* out) {
    for (size_t b = 0; b < n; ++b) {
        const uint8_t* blk = blocks + b * KQ_Q4K_BYTES;
        float d = kqo_fp16_to_f32(rd16(blk));
        float dmin = kqo_fp16_to_f32(rd16(blk + 2));
        const uint8_t* scales = blk + 4;
        const uint8_t* qs = blk + 16;
        float* o = out + b * KQ_QK;
        for (int j = 0; j < 8; ++j) {
            uint8_t sc, m;
            kqo_q4k_scale_min(scales, j, &sc, &m);
            float ds = d * (float)sc;
            float dm = dmin * (float)m;
            int c = j >> 1, hi = j & 1;
            for (int l = 0; l < 32; ++l) {
                uint8_t q = hi ? (uint8_t)(qs[32 * c + l] >> 4) : (uint8_t)(qs[32 * c + l] & 15u);
                float t = ds * (float)q;
                o[32 * j + l] = t - dm;
            }
        }
    }
}

/* ---------------------------------------------------------------- Q6_K */

/* Half h (0..1) of 128 weights uses ql[64h..], qh[32h..], scales[8h..]. For l in 0..31:
 * element l     = ql[l] low nibble    | (qh[l] bits 0-1) << 4
 * element l+32  = ql[l+32] low nibble | (qh[l] bits 2-3) << 4
 * element l+64  = ql[l] high nibble   | (qh[l] bits 4-5) << 4
 * element l+96  = ql[l+32] high nibble| (qh[l] bits 6-7) << 4
 * and element e of the block has scale scales[e / 16]. w = (d * scale) * (q - 32). */
void kqo_dequant_q6k(const uint8_t* blocks, size_t n, float* out) {
    for (size_t b = 0; b < n; ++b) {
        const uint8_t* blk = blocks + b * KQ_Q6K_BYTES;
        const uint8_t* ql = blk;
        const uint8_t* qh = blk + 128;
        const int8_t* sc = (const int8_t*)(blk + 192);
        float d = kqo_fp16_to_f32(rd16(blk + 208));
        float* o = out + b * KQ_QK;
        for (int h = 0; h < 2; ++h) {
            for (int l = 0; l < 32; ++l) {
                uint8_t L0 = ql[64 * h + l], L1 = ql[64 * h + l + 32], H = qh[32 * h + l];
                int q[4];
                q[0] = (L0 & 15) | ((H & 3) << 4);
                q[1] = (L1 & 15) | (((H >> 2) & 3) << 4);
                q[2] = (L0 >> 4) | (((H >> 4) & 3) << 4);
                q[3] = (L1 >> 4) | (((H >> 6) & 3) << 4);
                for (int g = 0; g < 4; ++g) {
                    int e = 128 * h + 32 * g + l;
                    float ds = d * (float)sc[e / 16];
                    o[e] = ds * (float)(q[g] - 32);
                }
            }
        }
    }
}

/* ---------------------------------------------------------------- Q5_K */

/* As Q4_K (qs at byte 48 instead of 16), with the fifth bit of element 32g + l in bit g of
 * qh[l]: chunk c's low nibbles are group 2c, its high nibbles group 2c + 1. */
void kqo_dequant_q5k(const uint8_t* blocks, size_t n, float* out) {
    for (size_t b = 0; b < n; ++b) {
        const uint8_t* blk = blocks + b * KQ_Q5K_BYTES;
        float d = kqo_fp16_to_f32(rd16(blk));
        float dmin = kqo_fp16_to_f32(rd16(blk + 2));
        const uint8_t* scales = blk + 4;
        const uint8_t* qh = blk + 16;
        const uint8_t* qs = blk + 48;
        float* o = out + b * KQ_QK;
        for (int j = 0; j < 8; ++j) {
            uint8_t sc, m;
            kqo_q4k_scale_min(scales, j, &sc, &m);
            float ds = d * (float)sc;
            float dm = dmin * (float)m;
            int c = j >> 1, hi = j & 1;
            for (int l = 0; l < 32; ++l) {
                uint8_t nib = hi ? (uint8_t)(qs[32 * c + l] >> 4) : (uint8_t)(qs[32 * c + l] & 15u);
                uint8_t q = (uint8_t)(nib | (((qh[l] >> j) & 1u) << 4));
                float t = ds * (float)q;
                o[32 * j + l] = t - dm;
            }
        }
    }
}

/* ---------------------------------------------------------------- reference matvec */

void kqo_matvec_ref(int type, const uint8_t* W, const float* x, uint32_t K, uint32_t r0,
                    uint32_t r1, uint32_t batch, uint64_t ldx, uint64_t ldy, double* y,
                    double* bound) {
    const uint32_t nb = K / KQ_QK;
    const size_t blk_bytes =
        type == 4 ? KQ_Q4K_BYTES : type == 5 ? KQ_Q5K_BYTES : KQ_Q6K_BYTES;
    float w[KQ_QK];
    for (uint32_t r = r0; r < r1; ++r) {
        for (uint32_t b = 0; b < batch; ++b) {
            y[b * ldy + r] = 0.0;
            bound[b * ldy + r] = 0.0;
        }
        for (uint32_t kb = 0; kb < nb; ++kb) {
            const uint8_t* blk = W + ((size_t)r * nb + kb) * blk_bytes;
            if (type == 4)
                kqo_dequant_q4k(blk, 1, w);
            else if (type == 5)
                kqo_dequant_q5k(blk, 1, w);
            else
                kqo_dequant_q6k(blk, 1, w);
            for (uint32_t b = 0; b < batch; ++b) {
                const float* xb = x + b * ldx + (size_t)kb * KQ_QK;
                double acc = 0.0, mag = 0.0;
                for (int i = 0; i < KQ_QK; ++i) {
                    double p = (double)w[i] * (double)xb[i];
                    acc += p;
                    mag += fabs(p);
                }
                y[b * ldy + r] += acc;
                bound[b * ldy + r] += mag;
            }
        }
    }
}

/* ---------------------------------------------------------------- generator */

static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

uint64_t kqo_splitmix_at(uint64_t key, uint64_t i) {
    return mix64(key + (i + 1) * 0x9e3779b97f4a7c15ull);
}

uint64_t kqo_stream_key(uint64_t seed, uint64_t tensor) {
    return mix64(mix64(seed * 0xd1342543de82ef95ull + tensor) ^ 0x632be59bd9b4e019ull);
}

/* lo + u * span with u = top 24 bits of `word` times 2^-24: one binary32 multiply, then one
 * add, then binary16 rounding to nearest even. */
static uint16_t uniform_fp16(uint64_t word, float lo, float span) {
    float u = (float)(uint32_t)(word >> 40) * 0x1p-24f;
    float t = u * span;
    float v = lo + t;
    return kqo_f32_to_fp16(v);
}

static void put_bytes(uint8_t* dst, uint64_t key, uint64_t base, int nbytes) {
    for (int i = 0; i < nbytes; i += 8) {
        uint64_t w = kqo_splitmix_at(key, base + (uint64_t)(i / 8));
        for (int j = 0; j < 8 && i + j < nbytes; ++j) dst[i + j] = (uint8_t)(w >> (8 * j));
    }
}

/* Block b draws counters [20b, 20b+20): words 0-17 are its 144 bytes (bytes 0-3 then
 * overwritten), word 18 gives d and word 19 gives dmin. */
void kqo_fill_q4k(uint8_t* out, uint64_t key, uint64_t b0, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t b = b0 + i;
        uint8_t* blk = out + i * KQ_Q4K_BYTES;
        put_bytes(blk, key, 20 * b, KQ_Q4K_BYTES);
        uint16_t d = uniform_fp16(kqo_splitmix_at(key, 20 * b + 18), 0x1p-10f, 15.0f * 0x1p-10f);
        uint16_t m = uniform_fp16(kqo_splitmix_at(key, 20 * b + 19), 0x1p-10f, 15.0f * 0x1p-10f);
        blk[0] = (uint8_t)d;
        blk[1] = (uint8_t)(d >> 8);
        blk[2] = (uint8_t)m;
        blk[3] = (uint8_t)(m >> 8);
    }
}

/* Block b draws counters [28b, 28b+28): words 0-26 give bytes 0-207 (ql, qh, and the raw
 * scale bytes, each mapped to (raw & 127) - 64), word 27 gives d. */
void kqo_fill_q6k(uint8_t* out, uint64_t key, uint64_t b0, uint64_t n) {
    uint8_t tmp[216];
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t b = b0 + i;
        uint8_t* blk = out + i * KQ_Q6K_BYTES;
        put_bytes(tmp, key, 28 * b, 216);
        memcpy(blk, tmp, 192);
        for (int s = 0; s < 16; ++s) blk[192 + s] = (uint8_t)(int8_t)((tmp[192 + s] & 127) - 64);
        uint16_t d = uniform_fp16(kqo_splitmix_at(key, 28 * b + 27), 0x1p-12f, 15.0f * 0x1p-12f);
        blk[208] = (uint8_t)d;
        blk[209] = (uint8_t)(d >> 8);
    }
}

/* Block b draws counters [24b, 24b+24): words 0-21 are its 176 bytes (bytes 0-3 then
 * overwritten), word 22 gives d and word 23 gives dmin. */
void kqo_fill_q5k(uint8_t* out, uint64_t key, uint64_t b0, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t b = b0 + i;
        uint8_t* blk = out + i * KQ_Q5K_BYTES;
        put_bytes(blk, key, 24 * b, KQ_Q5K_BYTES);
        uint16_t d = uniform_fp16(kqo_splitmix_at(key, 24 * b + 22), 0x1p-11f, 15.0f * 0x1p-11f);
        uint16_t m = uniform_fp16(kqo_splitmix_at(key, 24 * b + 23), 0x1p-11f, 15.0f * 0x1p-11f);
        blk[0] = (uint8_t)d;
        blk[1] = (uint8_t)(d >> 8);
        blk[2] = (uint8_t)m;
        blk[3] = (uint8_t)(m >> 8);
    }
}
