/*
 * kq_oracle.c -- CPU restatement of the GGML Q2_K / Q3_K / Q4_K / Q5_K / Q6_K / Q8_0 decode, the
 * f64 reference matvec and the counter-based synthetic generator. TEST INFRASTRUCTURE ONLY (see
 * kq_oracle.h).
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

/* ---------------------------------------------------------------- Q2_K */

/* scales[16] at 0 (low nibble: scale, high nibble: min of 16-element sub-block i), qs[64] at 16,
 * d at 80, dmin at 82. Element 128h + 32s + l (h 0..1, s 0..3, l 0..31) is bits 2s..2s+1 of
 * qs[32h + l]; its sub-block is element / 16. w = (d*f32(sc))*f32(q) - dmin*f32(m), the product
 * of d and the scale rounded first (gguf-py/gguf/quants.py Q2_K.dequantize_blocks). */
void kqo_dequant_q2k(const uint8_t* blocks, size_t n, float* out) {
    for (size_t b = 0; b < n; ++b) {
        const uint8_t* blk = blocks + b * KQ_Q2K_BYTES;
        const uint8_t* sc = blk;
        const uint8_t* qs = blk + 16;
        float d = kqo_fp16_to_f32(rd16(blk + 80));
        float dmin = kqo_fp16_to_f32(rd16(blk + 82));
        float* o = out + b * KQ_QK;
        for (int e = 0; e < KQ_QK; ++e) {
            int h = e >> 7, s4 = (e >> 5) & 3, l = e & 31;
            uint8_t q = (uint8_t)((qs[32 * h + l] >> (2 * s4)) & 3u);
            uint8_t si = sc[e >> 4];
            float dl = d * (float)(si & 15u);
            float ml = dmin * (float)(si >> 4);
            float t = dl * (float)q;
            o[e] = t - ml;
        }
    }
}

/* ---------------------------------------------------------------- Q3_K */

/* The 6-bit scale i (0..15) of a Q3_K block, as the signed value scale - 32: low 4 bits from
 * nibble i / 8 of byte i % 8, high 2 bits from bits 2 (i / 4).. of byte 8 + i % 4. */
int kqo_q3k_scale(const uint8_t s[12], int i) {
    int lo = (s[i % 8] >> (4 * (i / 8))) & 15;
    int hi = (s[8 + i % 4] >> (2 * (i / 4))) & 3;
    return (lo | (hi << 4)) - 32;
}

/* hmask[32] at 0, qs[64] at 32, scales[12] at 96, d at 108. Element 128h + 32s + l has low bits
 * 2s..2s+1 of qs[32h + l] and high bit k = 4h + s of hmask[l]; q = low - 4 when that bit is
 * clear, low when it is set. Sub-block element / 16. w = (d*f32(scale - 32))*f32(q)
 * (gguf-py/gguf/quants.py Q3_K.dequantize_blocks). */
void kqo_dequant_q3k(const uint8_t* blocks, size_t n, float* out) {
    for (size_t b = 0; b < n; ++b) {
        const uint8_t* blk = blocks + b * KQ_Q3K_BYTES;
        const uint8_t* hm = blk;
        const uint8_t* qs = blk + 32;
        const uint8_t* sc = blk + 96;
        float d = kqo_fp16_to_f32(rd16(blk + 108));
        float* o = out + b * KQ_QK;
        for (int e = 0; e < KQ_QK; ++e) {
            int h = e >> 7, s4 = (e >> 5) & 3, l = e & 31;
            int low = (qs[32 * h + l] >> (2 * s4)) & 3;
            int high = (hm[l] >> (4 * h + s4)) & 1;
            int q = low - (high ? 0 : 4);
            float dl = d * (float)kqo_q3k_scale(sc, e >> 4);
            o[e] = dl * (float)q;
        }
    }
}

/* ---------------------------------------------------------------- Q8_0 */

/* Eight consecutive 32-element Q8_0 blocks (34 bytes each: f16 d, then int8 qs[32]) make one
 * 256-element unit of 272 bytes, so that rows of K (a multiple of 256) elements are whole units.
 * w = f32(q) * d (gguf-py/gguf/quants.py Q8_0.dequantize_blocks). */
void kqo_dequant_q8_0(const uint8_t* units, size_t n, float* out) {
    for (size_t u = 0; u < n * 8; ++u) {
        const uint8_t* blk = units + u * KQ_Q8_0_BLOCK_BYTES;
        float d = kqo_fp16_to_f32(rd16(blk));
        const int8_t* q = (const int8_t*)(blk + 2);
        for (int l = 0; l < 32; ++l) out[u * 32 + l] = (float)q[l] * d;
    }
}

/* Bytes per 256 weights of `type` (2, 3, 4, 5, 6, 8), 0 for an unknown type. */
size_t kqo_unit_bytes(int type) {
    switch (type) {
        case 2: return KQ_Q2K_BYTES;
        case 3: return KQ_Q3K_BYTES;
        case 4: return KQ_Q4K_BYTES;
        case 5: return KQ_Q5K_BYTES;
        case 6: return KQ_Q6K_BYTES;
        case 8: return KQ_Q8_0_UNIT_BYTES;
        default: return 0;
    }
}

/* Decode n 256-weight units of `type`; returns -1 for an unknown type. */
int kqo_dequant(int type, const uint8_t* units, size_t n, float* out) {
    switch (type) {
        case 2: kqo_dequant_q2k(units, n, out); return 0;
        case 3: kqo_dequant_q3k(units, n, out); return 0;
        case 4: kqo_dequant_q4k(units, n, out); return 0;
        case 5: kqo_dequant_q5k(units, n, out); return 0;
        case 6: kqo_dequant_q6k(units, n, out); return 0;
        case 8: kqo_dequant_q8_0(units, n, out); return 0;
        default: return -1;
    }
}

/* ---------------------------------------------------------------- reference matvec */

void kqo_matvec_ref(int type, const uint8_t* W, const float* x, uint32_t K, uint32_t r0,
                    uint32_t r1, uint32_t batch, uint64_t ldx, uint64_t ldy, double* y,
                    double* bound) {
    const uint32_t nb = K / KQ_QK;
    const size_t blk_bytes = kqo_unit_bytes(type);
    float w[KQ_QK];
    if (blk_bytes == 0) return;
    for (uint32_t r = r0; r < r1; ++r) {
        for (uint32_t b = 0; b < batch; ++b) {
            y[b * ldy + r] = 0.0;
            bound[b * ldy + r] = 0.0;
        }
        for (uint32_t kb = 0; kb < nb; ++kb) {
            const uint8_t* blk = W + ((size_t)r * nb + kb) * blk_bytes;
            kqo_dequant(type, blk, 1, w);
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

/* Block b draws counters [13b, 13b+13): words 0-10 give its 84 bytes (bytes 80-83 then
 * overwritten), word 11 gives d and word 12 gives dmin, both fp16(uniform [2^-9, 2^-5]). */
void kqo_fill_q2k(uint8_t* out, uint64_t key, uint64_t b0, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t b = b0 + i;
        uint8_t* blk = out + i * KQ_Q2K_BYTES;
        put_bytes(blk, key, 13 * b, KQ_Q2K_BYTES);
        uint16_t d = uniform_fp16(kqo_splitmix_at(key, 13 * b + 11), 0x1p-9f, 15.0f * 0x1p-9f);
        uint16_t m = uniform_fp16(kqo_splitmix_at(key, 13 * b + 12), 0x1p-9f, 15.0f * 0x1p-9f);
        blk[80] = (uint8_t)d;
        blk[81] = (uint8_t)(d >> 8);
        blk[82] = (uint8_t)m;
        blk[83] = (uint8_t)(m >> 8);
    }
}

/* Block b draws counters [15b, 15b+15): words 0-13 give its 110 bytes (bytes 108-109 then
 * overwritten), word 14 gives d = fp16(uniform [2^-11, 2^-7]). */
void kqo_fill_q3k(uint8_t* out, uint64_t key, uint64_t b0, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t b = b0 + i;
        uint8_t* blk = out + i * KQ_Q3K_BYTES;
        put_bytes(blk, key, 15 * b, KQ_Q3K_BYTES);
        uint16_t d = uniform_fp16(kqo_splitmix_at(key, 15 * b + 14), 0x1p-11f, 15.0f * 0x1p-11f);
        blk[108] = (uint8_t)d;
        blk[109] = (uint8_t)(d >> 8);
    }
}

/* Units [b0, b0+n) of 8 blocks; Q8_0 block j = 8u + v draws counters [6j, 6j+6): words 0-4
 * give its 34 bytes (bytes 0-1 then overwritten), word 5 gives d = fp16(uniform [2^-12, 2^-8]). */
void kqo_fill_q8_0(uint8_t* out, uint64_t key, uint64_t b0, uint64_t n) {
    for (uint64_t i = 0; i < n * 8; ++i) {
        uint64_t j = b0 * 8 + i;
        uint8_t* blk = out + i * KQ_Q8_0_BLOCK_BYTES;
        put_bytes(blk, key, 6 * j, KQ_Q8_0_BLOCK_BYTES);
        uint16_t d = uniform_fp16(kqo_splitmix_at(key, 6 * j + 5), 0x1p-12f, 15.0f * 0x1p-12f);
        blk[0] = (uint8_t)d;
        blk[1] = (uint8_t)(d >> 8);
    }
}
