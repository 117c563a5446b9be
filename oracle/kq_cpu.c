/*
 * kq_cpu.c -- the CPU baseline: a multithreaded AVX2 + FMA (x86-64-v3) Q2_K / Q3_K / Q4_K / Q5_K /
 * Q6_K / Q8_0 matvec.
 * TEST / BASELINE INFRASTRUCTURE ONLY (see kq_oracle.h): bench.py times it beside the GPU
 * numbers; the product never calls it.
 *
 * fxeqxmulfx/kernite has no x86 k-quant kernel, so this stands in for one. Its inner loop is the
 * shape of kernite's x86 `dot::<4>` (examples/my-app/src/main.rs:39-70): independent 8-lane FMA
 * accumulators over the row. Rows are split in contiguous ranges, one per thread, each thread
 * pinned to one core, as kernite_cpu's Grid::on places threads (GUIDE.md:512-523).
 *
 * Algebra per sub-block j of 32 (Q4_K) or 16 (Q6_K) weights:
 *   sum_k w_k x_k = d*sc_j * sum_k q_k x_k - dmin*m_j * sum_k x_k        (Q4_K, Q5_K)
 *   sum_k w_k x_k = d*sc_j * (sum_k q_k x_k - 32 * sum_k x_k)             (Q6_K)
 *   sum_k w_k x_k = d*sc_j * sum_k q_k x_k - dmin*m_j * sum_k x_k        (Q2_K, 16 weights)
 *   sum_k w_k x_k = d*sc_j * (sum_k (q_k + 4) x_k - 4 * sum_k x_k)       (Q3_K, 16 weights)
 *   sum_k w_k x_k = d_j * sum_k q_k x_k                                  (Q8_0, 32 weights)
 * with the per-sub-block sums of x computed once per vector.
 */
#define _GNU_SOURCE
#include <immintrin.h>
#include <pthread.h>
#include <sched.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "kq_oracle.h"

typedef struct {
    int type;
    const uint8_t* W;
    const float* x;
    const float* xsum; /* per-vector sums of x over each sub-block (32 for Q4_K, 16 for Q6_K) */
    uint32_t r0, r1, K, batch, rows;
    float* y;
    int cpu;
} job_t;

/* weights per sub-block whose sums of x the rows use */
static uint32_t sub_block(int type) { return (type == 4 || type == 5 || type == 8) ? 32 : 16; }

static inline float hsum8(__m256 v) {
    __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
    lo = _mm_add_ps(lo, hi);
    lo = _mm_add_ps(lo, _mm_movehl_ps(lo, lo));
    lo = _mm_add_ss(lo, _mm_movehdup_ps(lo));
    return _mm_cvtss_f32(lo);
}

/* 8 bytes of 4-bit-or-6-bit quants (already masked) as 8 floats */
static inline __m256 u8x8_to_f32(__m128i bytes8) {
    return _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(bytes8));
}

/* Q4_K, or (q5) Q5_K: the same block with qh[32] before qs, bit j of qh[l] the fifth bit of
 * element 32 j + l */
static float row_q45k(const uint8_t* row, const float* x, const float* xsum, uint32_t nb, int q5) {
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(),
                     _mm256_setzero_ps()};
    float tail = 0.0f;
    const __m128i low = _mm_set1_epi8(0x0f), one = _mm_set1_epi8(1);
    const size_t bb = q5 ? KQ_Q5K_BYTES : KQ_Q4K_BYTES;
    for (uint32_t kb = 0; kb < nb; ++kb) {
        const uint8_t* blk = row + (size_t)kb * bb;
        uint16_t dh, mh;
        memcpy(&dh, blk, 2);
        memcpy(&mh, blk + 2, 2);
        float d = _cvtsh_ss(dh), dmin = _cvtsh_ss(mh);
        const uint8_t* qs = blk + (q5 ? 48 : 16);
        const float* xb = x + (size_t)kb * KQ_QK;
        __m128i qh0 = _mm_setzero_si128(), qh1 = _mm_setzero_si128();
        if (q5) {
            qh0 = _mm_loadu_si128((const __m128i*)(blk + 16));
            qh1 = _mm_loadu_si128((const __m128i*)(blk + 32));
        }
        for (int c = 0; c < 4; ++c) {
            uint8_t sc0, m0, sc1, m1;
            kqo_q4k_scale_min(blk + 4, 2 * c, &sc0, &m0);
            kqo_q4k_scale_min(blk + 4, 2 * c + 1, &sc1, &m1);
            __m128i q0 = _mm_loadu_si128((const __m128i*)(qs + 32 * c));
            __m128i q1 = _mm_loadu_si128((const __m128i*)(qs + 32 * c + 16));
            __m128i lo0 = _mm_and_si128(q0, low), lo1 = _mm_and_si128(q1, low);
            __m128i hi0 = _mm_and_si128(_mm_srli_epi16(q0, 4), low);
            __m128i hi1 = _mm_and_si128(_mm_srli_epi16(q1, 4), low);
            if (q5) { /* bits 2c (sub-block 2c) and 2c + 1 (sub-block 2c + 1) of qh, to bit 4 */
                const __m128i s0 = _mm_cvtsi32_si128(2 * c), s1 = _mm_cvtsi32_si128(2 * c + 1);
                lo0 = _mm_or_si128(lo0, _mm_slli_epi16(_mm_and_si128(_mm_srl_epi16(qh0, s0), one), 4));
                lo1 = _mm_or_si128(lo1, _mm_slli_epi16(_mm_and_si128(_mm_srl_epi16(qh1, s0), one), 4));
                hi0 = _mm_or_si128(hi0, _mm_slli_epi16(_mm_and_si128(_mm_srl_epi16(qh0, s1), one), 4));
                hi1 = _mm_or_si128(hi1, _mm_slli_epi16(_mm_and_si128(_mm_srl_epi16(qh1, s1), one), 4));
            }
            __m256 s0 = _mm256_set1_ps(d * (float)sc0), s1 = _mm256_set1_ps(d * (float)sc1);
            const float* xa = xb + 64 * c;
            /* sub-block 2c: low nibbles, 32 elements, 4 accumulators */
            acc[0] = _mm256_fmadd_ps(_mm256_mul_ps(s0, u8x8_to_f32(lo0)), _mm256_loadu_ps(xa), acc[0]);
            acc[1] = _mm256_fmadd_ps(_mm256_mul_ps(s0, u8x8_to_f32(_mm_srli_si128(lo0, 8))),
                                     _mm256_loadu_ps(xa + 8), acc[1]);
            acc[2] = _mm256_fmadd_ps(_mm256_mul_ps(s0, u8x8_to_f32(lo1)), _mm256_loadu_ps(xa + 16), acc[2]);
            acc[3] = _mm256_fmadd_ps(_mm256_mul_ps(s0, u8x8_to_f32(_mm_srli_si128(lo1, 8))),
                                     _mm256_loadu_ps(xa + 24), acc[3]);
            /* sub-block 2c+1: high nibbles */
            acc[0] = _mm256_fmadd_ps(_mm256_mul_ps(s1, u8x8_to_f32(hi0)), _mm256_loadu_ps(xa + 32), acc[0]);
            acc[1] = _mm256_fmadd_ps(_mm256_mul_ps(s1, u8x8_to_f32(_mm_srli_si128(hi0, 8))),
                                     _mm256_loadu_ps(xa + 40), acc[1]);
            acc[2] = _mm256_fmadd_ps(_mm256_mul_ps(s1, u8x8_to_f32(hi1)), _mm256_loadu_ps(xa + 48), acc[2]);
            acc[3] = _mm256_fmadd_ps(_mm256_mul_ps(s1, u8x8_to_f32(_mm_srli_si128(hi1, 8))),
                                     _mm256_loadu_ps(xa + 56), acc[3]);
            const float* xs = xsum + (size_t)kb * 8 + 2 * c;
            tail -= dmin * (float)m0 * xs[0] + dmin * (float)m1 * xs[1];
        }
    }
    acc[0] = _mm256_add_ps(_mm256_add_ps(acc[0], acc[1]), _mm256_add_ps(acc[2], acc[3]));
    return hsum8(acc[0]) + tail;
}

static float row_q6k(const uint8_t* row, const float* x, const float* xsum, uint32_t nb) {
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(),
                     _mm256_setzero_ps()};
    float tail = 0.0f;
    const __m128i low = _mm_set1_epi8(0x0f), three = _mm_set1_epi8(3);
    for (uint32_t kb = 0; kb < nb; ++kb) {
        const uint8_t* blk = row + (size_t)kb * KQ_Q6K_BYTES;
        const int8_t* sc = (const int8_t*)(blk + 192);
        uint16_t dh;
        memcpy(&dh, blk + 208, 2);
        float d = _cvtsh_ss(dh);
        const float* xb = x + (size_t)kb * KQ_QK;
        for (int h = 0; h < 2; ++h) {
            for (int half = 0; half < 2; ++half) { /* l in [16*half, 16*half + 16) */
                int l0 = 16 * half;
                __m128i L0 = _mm_loadu_si128((const __m128i*)(blk + 64 * h + l0));
                __m128i L1 = _mm_loadu_si128((const __m128i*)(blk + 64 * h + 32 + l0));
                __m128i H = _mm_loadu_si128((const __m128i*)(blk + 128 + 32 * h + l0));
                __m128i q[4];
                q[0] = _mm_or_si128(_mm_and_si128(L0, low), _mm_slli_epi16(_mm_and_si128(H, three), 4));
                q[1] = _mm_or_si128(_mm_and_si128(L1, low),
                                    _mm_slli_epi16(_mm_and_si128(_mm_srli_epi16(H, 2), three), 4));
                q[2] = _mm_or_si128(_mm_and_si128(_mm_srli_epi16(L0, 4), low),
                                    _mm_slli_epi16(_mm_and_si128(_mm_srli_epi16(H, 4), three), 4));
                q[3] = _mm_or_si128(_mm_and_si128(_mm_srli_epi16(L1, 4), low),
                                    _mm_slli_epi16(_mm_and_si128(_mm_srli_epi16(H, 6), three), 4));
                for (int g = 0; g < 4; ++g) {
                    int e = 128 * h + 32 * g + l0; /* first element; one scale covers all 16 */
                    __m256 s = _mm256_set1_ps(d * (float)sc[e / 16]);
                    acc[g] = _mm256_fmadd_ps(_mm256_mul_ps(s, u8x8_to_f32(q[g])), _mm256_loadu_ps(xb + e), acc[g]);
                    acc[g] = _mm256_fmadd_ps(_mm256_mul_ps(s, u8x8_to_f32(_mm_srli_si128(q[g], 8))),
                                             _mm256_loadu_ps(xb + e + 8), acc[g]);
                    tail -= 32.0f * d * (float)sc[e / 16] * xsum[(size_t)kb * 16 + e / 16];
                }
            }
        }
    }
    acc[0] = _mm256_add_ps(_mm256_add_ps(acc[0], acc[1]), _mm256_add_ps(acc[2], acc[3]));
    return hsum8(acc[0]) + tail;
}

/* 16 bytes of small unsigned quants as two 8-lane float vectors */
static inline void u8x16_to_f32(__m128i q, __m256* lo, __m256* hi) {
    *lo = u8x8_to_f32(q);
    *hi = u8x8_to_f32(_mm_srli_si128(q, 8));
}

/* Q2_K (q2 = 1) or Q3_K (q2 = 0): element 128h + 32s + l is bits 2s..2s+1 of qs[32h + l]
 * (Q3_K: plus 4 * bit 4h + s of hmask[l], the stored quant being q + 4); sub-block = element / 16 */
static float row_q23k(const uint8_t* row, const float* x, const float* xsum, uint32_t nb, int q2) {
    __m256 acc[2] = {_mm256_setzero_ps(), _mm256_setzero_ps()};
    float tail = 0.0f;
    const __m128i three = _mm_set1_epi8(3), one = _mm_set1_epi8(1);
    const size_t bb = q2 ? KQ_Q2K_BYTES : KQ_Q3K_BYTES;
    for (uint32_t kb = 0; kb < nb; ++kb) {
        const uint8_t* blk = row + (size_t)kb * bb;
        const uint8_t* qs = blk + (q2 ? 16 : 32);
        uint16_t dh, mh = 0;
        memcpy(&dh, blk + (q2 ? 80 : 108), 2);
        if (q2) memcpy(&mh, blk + 82, 2);
        float d = _cvtsh_ss(dh), dmin = _cvtsh_ss(mh);
        const float* xb = x + (size_t)kb * KQ_QK;
        const float* sb = xsum + (size_t)kb * 16;
        for (int h = 0; h < 2; ++h) {
            __m128i Q0 = _mm_loadu_si128((const __m128i*)(qs + 32 * h));
            __m128i Q1 = _mm_loadu_si128((const __m128i*)(qs + 32 * h + 16));
            __m128i H0 = _mm_setzero_si128(), H1 = _mm_setzero_si128();
            if (!q2) {
                H0 = _mm_loadu_si128((const __m128i*)blk);
                H1 = _mm_loadu_si128((const __m128i*)(blk + 16));
            }
            for (int s4 = 0; s4 < 4; ++s4) {
                const __m128i sh = _mm_cvtsi32_si128(2 * s4);
                __m128i c0 = _mm_and_si128(_mm_srl_epi16(Q0, sh), three);
                __m128i c1 = _mm_and_si128(_mm_srl_epi16(Q1, sh), three);
                if (!q2) {
                    const __m128i hk = _mm_cvtsi32_si128(4 * h + s4);
                    c0 = _mm_or_si128(c0, _mm_slli_epi16(_mm_and_si128(_mm_srl_epi16(H0, hk), one), 2));
                    c1 = _mm_or_si128(c1, _mm_slli_epi16(_mm_and_si128(_mm_srl_epi16(H1, hk), one), 2));
                }
                const int e = 128 * h + 32 * s4, i0 = e / 16;
                float s0, s1;
                if (q2) {
                    s0 = d * (float)(blk[i0] & 15);
                    s1 = d * (float)(blk[i0 + 1] & 15);
                    tail -= dmin * (float)(blk[i0] >> 4) * sb[i0] + dmin * (float)(blk[i0 + 1] >> 4) * sb[i0 + 1];
                } else {
                    s0 = d * (float)kqo_q3k_scale(blk + 96, i0);
                    s1 = d * (float)kqo_q3k_scale(blk + 96, i0 + 1);
                    tail -= 4.0f * (s0 * sb[i0] + s1 * sb[i0 + 1]);
                }
                __m256 a, b;
                u8x16_to_f32(c0, &a, &b);
                acc[0] = _mm256_fmadd_ps(_mm256_mul_ps(_mm256_set1_ps(s0), a), _mm256_loadu_ps(xb + e), acc[0]);
                acc[1] = _mm256_fmadd_ps(_mm256_mul_ps(_mm256_set1_ps(s0), b), _mm256_loadu_ps(xb + e + 8), acc[1]);
                u8x16_to_f32(c1, &a, &b);
                acc[0] = _mm256_fmadd_ps(_mm256_mul_ps(_mm256_set1_ps(s1), a), _mm256_loadu_ps(xb + e + 16), acc[0]);
                acc[1] = _mm256_fmadd_ps(_mm256_mul_ps(_mm256_set1_ps(s1), b), _mm256_loadu_ps(xb + e + 24), acc[1]);
            }
        }
    }
    return hsum8(_mm256_add_ps(acc[0], acc[1])) + tail;
}

/* Q8_0: 32-weight blocks of 34 bytes, eight per 256 weights */
static float row_q8_0(const uint8_t* row, const float* x, uint32_t nb) {
    __m256 acc = _mm256_setzero_ps();
    for (uint32_t j = 0; j < nb * 8; ++j) {
        const uint8_t* blk = row + (size_t)j * KQ_Q8_0_BLOCK_BYTES;
        uint16_t dh;
        memcpy(&dh, blk, 2);
        const float* xb = x + (size_t)j * 32;
        __m256 s = _mm256_setzero_ps();
        for (int c = 0; c < 4; ++c) {
            __m128i q8 = _mm_loadl_epi64((const __m128i*)(blk + 2 + 8 * c));
            __m256 qf = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(q8));
            s = _mm256_fmadd_ps(qf, _mm256_loadu_ps(xb + 8 * c), s);
        }
        acc = _mm256_fmadd_ps(s, _mm256_set1_ps(_cvtsh_ss(dh)), acc);
    }
    return hsum8(acc);
}

static void* worker(void* arg) {
    job_t* j = (job_t*)arg;
    if (j->cpu >= 0) {
        cpu_set_t set;
        CPU_ZERO(&set);
        CPU_SET(j->cpu, &set);
        pthread_setaffinity_np(pthread_self(), sizeof(set), &set);
    }
    const uint32_t nb = j->K / KQ_QK;
    const size_t rb = (size_t)nb * kqo_unit_bytes(j->type);
    const uint32_t per = sub_block(j->type);
    /* rows outer, vectors inner: each weight row is read from memory once for all vectors */
    for (uint32_t r = j->r0; r < j->r1; ++r) {
        const uint8_t* row = j->W + (size_t)r * rb;
        for (uint32_t b = 0; b < j->batch; ++b) {
            const float* xb = j->x + (size_t)b * j->K;
            const float* sb = j->xsum + (size_t)b * (j->K / per);
            float v;
            switch (j->type) {
                case 2: v = row_q23k(row, xb, sb, nb, 1); break;
                case 3: v = row_q23k(row, xb, sb, nb, 0); break;
                case 6: v = row_q6k(row, xb, sb, nb); break;
                case 8: v = row_q8_0(row, xb, nb); break;
                default: v = row_q45k(row, xb, sb, nb, j->type == 5); break;
            }
            j->y[(size_t)b * j->rows + r] = v;
        }
    }
    return NULL;
}

int kqo_matvec_cpu(int type, const uint8_t* W, const float* x, uint32_t rows, uint32_t K,
                   uint32_t batch, float* y, int threads) {
    if (kqo_unit_bytes(type) == 0 || K % KQ_QK != 0 || threads < 1) return -1;
    const uint32_t per = sub_block(type);
    const size_t nsub = (size_t)K / per;
    float* xsum = (float*)malloc(sizeof(float) * nsub * (batch ? batch : 1));
    if (!xsum) return -2;
    for (uint32_t b = 0; b < batch; ++b)
        for (size_t s = 0; s < nsub; ++s) {
            float t = 0.0f;
            for (uint32_t i = 0; i < per; ++i) t += x[(size_t)b * K + s * per + i];
            xsum[(size_t)b * nsub + s] = t;
        }
    if ((uint32_t)threads > rows && rows > 0) threads = (int)rows;
    job_t* jobs = (job_t*)calloc((size_t)threads, sizeof(job_t));
    pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    int ncpu = (int)sysconf(_SC_NPROCESSORS_ONLN);
    for (int t = 0; t < threads; ++t) {
        job_t* j = &jobs[t];
        j->type = type;
        j->W = W;
        j->x = x;
        j->xsum = xsum;
        j->r0 = (uint32_t)((uint64_t)rows * (uint64_t)t / (uint64_t)threads);
        j->r1 = (uint32_t)((uint64_t)rows * (uint64_t)(t + 1) / (uint64_t)threads);
        j->K = K;
        j->batch = batch;
        j->rows = rows;
        j->y = y;
        j->cpu = threads > 1 && ncpu > 0 ? t % ncpu : -1;
    }
    for (int t = 1; t < threads; ++t) pthread_create(&tids[t], NULL, worker, &jobs[t]);
    worker(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tids[t], NULL);
    free(tids);
    free(jobs);
    free(xsum);
    return 0;
}
