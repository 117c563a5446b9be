// kq_matvec.cu -- the Q4_K / Q6_K streaming matvec on the CUDA cores, batch 1..8.
//
// y[b, r] = sum_k W[r, k] * x[b, k], W in GGML k-quant blocks (144-byte Q4_K, 210-byte Q6_K).
//
// Shape of the kernel (one persistent CTA per SM):
//  * Each CTA owns a contiguous range of rows, i.e. a contiguous byte range of W. A producer
//    warp streams it, a tile of P rows at a time, into a ring of shared-memory slots with
//    cp.async.bulk (TMA, 1-D) copies of the 16-byte-aligned superset of each tile; an mbarrier
//    per slot counts the bytes in. Q6_K rows whose blocks start at any even offset need nothing
//    special: the consumer reads bytes at the tile's offset from the aligned base.
//  * The consumer warps form P "teams", one row of the tile each. Within a team every lane owns
//    a fixed 64/B-weight part of each row (part `pi` of block `kb`), so its slice of x stays in
//    registers for the whole kernel and shared memory only carries weights.
//  * A lane turns each 4- or 6-bit quant q into the float 2 + q/64 with one PRMT (q placed in
//    mantissa bits 16..23 under exponent 2^1; Q4_K's high nibbles sit in bits 8..15, giving
//    2 + q/1024) and accumulates x * that with packed f32x2 FMAs. The offsets are removed per
//    sub-block with the lane's own sums of x:  sum q*x = 64*S - 128*X  (or 1024*S - 2048*X).
//    Q4_K: y += d*(sc_A*sum q*x_A + sc_B*sum q*x_B) - dmin*(m_A*X_A + m_B*X_B).
//    Q6_K: y += d*sc_g*(sum q*x_g - 32*X_g) per group of 16.
//  * Lanes reduce by warp shuffles, warps of a team through shared memory, once per tile.
//
// The GGML block layouts and the decode follow the public format (see the CPU restatement in
// oracle/kq_oracle.c); the pattern "one output row per team, FMA chain over k" is the matvec of
// fxeqxmulfx/kernite's examples/microgpt/src/gpu.rs:100-131, re-shaped for HBM streaming.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>

#include "kq_device.cuh"
#include "kq_internal.h"

// 1: accumulate with packed f32x2 FMAs (two weights an instruction); 0: scalar FMAs.
#ifndef KQ_PACKED_FMA
#define KQ_PACKED_FMA 0
#endif

namespace kq {
namespace {

struct MatvecArgs {
  const uint8_t* W;
  const float* x;
  float* y;
  unsigned* err;
  uint64_t ldx, ldy;      // floats between vectors
  uint64_t total_bytes;   // rows * row bytes
  uint32_t rows, nb, batch;
  uint32_t team_warps, teams, per_team, ring, slot_bytes;  // tile = teams * per_team rows
  uint32_t row_unit, prologue, epilogue, flags;
  float eps, pair_scale;
  // push exchange (kq_matvec_push); npush == 0 otherwise
  uint32_t npush, push_rows;
  float* push_y[8];
  unsigned long long* push_cnt[8];
  const unsigned long long* wait_cnt;
  const unsigned long long* epoch;
  uint64_t wait_mul, wait_add;
};

// x loads: L1-cached, so the teams of a CTA share one L2 read of each line. Not the
// non-coherent path: with the push exchange x is written by other GPUs while this kernel runs
// (before thread 0's acquire, which the CTA barrier orders before these loads).
__device__ __forceinline__ float4 ld_x4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

// Named barrier among the consumer warps for the push exchange (teams use 1..14).
constexpr uint32_t kPushBarrier = 15;

template <int QT>
struct Fmt;
template <>
struct Fmt<4> {
  static constexpr int kBlk = kQ4KBytes;
  static constexpr int kSpan = 128;  // parts per block = kSpan / L
  static constexpr int kGroups = 2;  // sub-block groups per part (low / high nibbles)
};
template <>
struct Fmt<6> {
  static constexpr int kBlk = kQ6KBytes;
  static constexpr int kSpan = 64;
  static constexpr int kGroups = 4;  // elements l, l+32, l+64, l+96 of a half
};

// Batch template -> l-values per lane part, and the block size the registers allow.
template <int B>
struct Geo {
  static constexpr int kL4 = B == 1 ? 32 : (B == 2 ? 16 : 8);  // Q4_K
  static constexpr int kL6 = B == 1 ? 16 : (B == 2 ? 8 : 4);   // Q6_K
  // 512 threads leave 128 registers a thread; 384 leave 168; 288 (rounded to 384) the same.
  static constexpr int kMaxThreads = B <= 2 ? 512 : (B == 4 ? 384 : 288);
};

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// quant byte i of `v` (< 128) as the float 2 + q/64
template <int I>
__device__ __forceinline__ float prmt_lo(uint32_t v) {
  return as_f32(__byte_perm(v, 0x40u, 0x4055u | (I << 8)));
}
// high-nibble byte i of `v` (16*q) as the float 2 + q/1024
template <int I>
__device__ __forceinline__ float prmt_hi(uint32_t v) {
  return as_f32(__byte_perm(v, 0x40u, 0x4505u | (I << 4)));
}

template <int QT, int B>
__global__ void __launch_bounds__(Geo<B>::kMaxThreads, 1) matvec_kernel(const MatvecArgs a) {
  constexpr int kBlk = Fmt<QT>::kBlk;
  constexpr int L = QT == 4 ? Geo<B>::kL4 : Geo<B>::kL6;
  constexpr int PPB = Fmt<QT>::kSpan / L;  // lane parts per block
  constexpr int G = Fmt<QT>::kGroups;
  constexpr int W = L / 4;                  // quant words per group per row

  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int s_failed;
  __shared__ double s_norm[16][8];  // [consumer warp][batch]; static shared memory stays < 2 KB

  const uint32_t RB = a.nb * kBlk;
  const uint32_t consumers = a.teams * a.team_warps;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // The ring starts at the first 128-byte boundary of dynamic shared memory (the host adds
  // 128 bytes of slack for this).
  uint8_t* ring = smem + ((128u - (smem_u32(smem) & 127u)) & 127u);
  float* red = reinterpret_cast<float*>(ring + a.ring * a.slot_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + 2 * consumers * a.per_team * B);
  const uint32_t ring_s = smem_u32(ring);
  auto full_bar = [&](uint32_t s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](uint32_t s) { return smem_u32(&bars[a.ring + s]); };

  // This CTA's rows, in units of row_unit (pairs for the pair-product epilogue).
  const uint64_t units = a.rows / a.row_unit;
  const uint32_t r_begin = static_cast<uint32_t>(units * blockIdx.x / gridDim.x) * a.row_unit;
  const uint32_t r_end = static_cast<uint32_t>(units * (blockIdx.x + 1) / gridDim.x) * a.row_unit;
  const uint32_t SR = a.teams * a.per_team;  // rows per tile; row rs0 + u*teams + team
  const uint32_t ntiles = (r_end - r_begin + SR - 1) / SR;

  if (threadIdx.x == 0) {
    s_failed = 0;
    for (uint32_t s = 0; s < a.ring; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), consumers);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // ------------------------------------------------------------------ producer warp
  if (warp == consumers) {
    if (lane == 0) {
      if (!(a.flags & KQ_FLAG_WEIGHTS_STATIC)) pdl_wait();
      const uint64_t pol = policy_evict_first();
      const uint64_t end_floor = a.total_bytes & ~uint64_t(15);
      uint32_t s = 0, phase = 0;  // slot and the parity of its current use
      for (uint32_t t = 0; t < ntiles; ++t, s = (s + 1 == a.ring) ? 0 : s + 1, phase ^= (s == 0)) {
        if (t >= a.ring) {
          if (s_failed) break;
          if (!mbar_wait(empty_bar(s), phase ^ 1)) {
            s_failed = 1;
            report_error(a.err, kErrWaitEmpty);
            break;
          }
        }
        const uint32_t rs0 = r_begin + t * SR;
        const uint32_t rs1 = min(rs0 + SR, r_end);
        const uint64_t b0 = uint64_t(rs0) * RB, b1 = uint64_t(rs1) * RB;
        const uint64_t a0 = b0 & ~uint64_t(15);
        uint64_t a1 = (b1 + 15) & ~uint64_t(15);
        const uint32_t slot = ring_s + s * a.slot_bytes;
        if (a1 > end_floor) {
          // The last tile of W ends off a 16-byte boundary: its last bytes (fewer than 16, an
          // even count) are read with plain loads, the rest by the bulk copy.
          for (uint64_t i = end_floor; i < a.total_bytes; i += 2) {
            const uint16_t v = __ldg(reinterpret_cast<const unsigned short*>(a.W + i));
            sts_u16(slot + static_cast<uint32_t>(i - a0), v);
          }
          a1 = end_floor;
        }
        const uint32_t bytes = static_cast<uint32_t>(a1 - a0);
        mbar_arrive_expect_tx(full_bar(s), bytes);
        if (bytes) bulk_g2s(slot, a.W + a0, bytes, full_bar(s), pol);
      }
    }
    return;
  }

  // ------------------------------------------------------------------ consumers
  const uint32_t team = warp / a.team_warps;
  const uint32_t tw = warp % a.team_warps;
  const uint32_t tl = tw * 32 + lane;
  const bool active = tl < PPB * a.nb;
  const uint32_t kb = active ? tl / PPB : 0;
  const uint32_t pi = tl % PPB;
  // The part's place in its block: Q4_K chunk c (64 weights) or Q6_K half h (128 weights),
  // and its first l-value.
  constexpr uint32_t kPartsPerUnit = 32 / L;
  const uint32_t unit = pi / kPartsPerUnit;           // c (Q4_K) or h (Q6_K)
  const uint32_t l0 = (pi % kPartsPerUnit) * L;
  const uint32_t base_off = QT == 4 ? 64 * unit : 128 * unit;  // element offset in the block

  pdl_wait();  // x may be the previous kernel's output
  if (a.wait_cnt) {
    // x is a full vector other GPUs push into: wait until every rank's rows of this step are in
    if (threadIdx.x == 0 && !wait_count(a.err, a.wait_cnt, a.epoch, a.wait_mul, a.wait_add))
      s_failed = 1;
    named_barrier(kPushBarrier, consumers * 32);
  }

  // x slice in registers, in pairs: xr[b][g][m] = x[b, e], x[b, e+1] with
  // e = kb*256 + base_off + 32g + l0 + 2m
  float2 xr[B][G][L / 2];
  float xs[B][G];
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int m = 0; m < L / 2; ++m) xr[b][g][m] = f2(0.f, 0.f);
  if (active) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (b < static_cast<int>(a.batch)) {
        const float* xb = a.x + b * a.ldx + uint64_t(kb) * kQK + base_off + l0;
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int m = 0; m < L / 4; ++m) {
            const float4 v = ld_x4(xb + 32 * g + 4 * m);
            xr[b][g][2 * m] = f2(v.x, v.y);
            xr[b][g][2 * m + 1] = f2(v.z, v.w);
          }
        }
      }
    }
  }

  if (a.prologue == KQ_PROLOGUE_RMSNORM) {
    // Every team's lanes hold all of x, so team 0's registers give the sum of squares. It is
    // taken in f64, where the square of any finite f32 neither overflows nor underflows.
#pragma unroll
    for (int b = 0; b < B; ++b) {
      double t = 0.0;
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int m = 0; m < L / 2; ++m) {
          const double u = xr[b][g][m].x, v = xr[b][g][m].y;
          t = fma(u, u, t);
          t = fma(v, v, t);
        }
#pragma unroll
      for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (lane == 0) s_norm[warp][b] = t;
    }
    named_barrier(1, consumers * 32);
    const double K = static_cast<double>(a.nb) * kQK;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      double t = 0.0;
      for (uint32_t w = 0; w < a.team_warps; ++w) t += s_norm[w][b];
      const float scale = static_cast<float>(1.0 / sqrt(t / K + static_cast<double>(a.eps)));
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int m = 0; m < L / 2; ++m) {
          xr[b][g][m].x *= scale;
          xr[b][g][m].y *= scale;
        }
    }
  }

  // The lane's sums of x per group, for the offset removal.
#pragma unroll
  for (int b = 0; b < B; ++b)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float t = 0.f;
#pragma unroll
      for (int m = 0; m < L / 2; ++m) t += xr[b][g][m].x + xr[b][g][m].y;
      xs[b][g] = t;
    }

  // Q4_K scale/min unpack constants for the lane's two sub-blocks j0 = 2c, j1 = 2c+1.
  const bool upper = unit >= 2;
  const uint32_t sh0 = 8 * ((2 * unit) & 3), sh1 = 8 * ((2 * unit + 1) & 3);

  // Rows: a tile holds teams * per_team rows; this team takes row_unit consecutive rows per
  // round, so the two rows of a pair-product stay in one team.
  const uint32_t R = a.row_unit;
  float* tbuf = red + team * (2u * a.team_warps * a.per_team * B);
  float held[B];
#pragma unroll
  for (int b = 0; b < B; ++b) held[b] = 0.f;

  const uint32_t rounds = a.per_team / R;     // rounds of R rows per tile for this team
  const uint32_t round_stride = a.teams * R;  // rows between a team's rounds
  uint32_t s = 0, phase = 0;                  // ring slot and the parity of its current use
  for (uint32_t t = 0; t < ntiles; ++t) {
    if (!s_failed && !mbar_wait(full_bar(s), phase)) {
      s_failed = 1;
      report_error(a.err, kErrWaitFull);
    }
    const bool failed = s_failed != 0;
    const uint32_t rs0 = r_begin + t * SR;
    const uint32_t rs1 = min(rs0 + SR, r_end);
    const uint32_t delta = static_cast<uint32_t>((uint64_t(rs0) * RB) & 15);
    const uint32_t slot_base = ring_s + s * a.slot_bytes + delta + kb * kBlk;
    float* tb = tbuf + (t & 1) * a.team_warps * a.per_team * B;
    for (uint32_t rr = 0, u = 0; rr < rounds; ++rr)
    for (uint32_t sub = 0; sub < R; ++sub, ++u) {
      const uint32_t rho = rr * round_stride + team * R + sub;  // row within the tile
      const uint32_t row = rs0 + rho;
      float acc[B];
#pragma unroll
      for (int b = 0; b < B; ++b) acc[b] = 0.f;

      if (active && row < rs1 && !failed) {
        const uint32_t blk = slot_base + rho * RB;
        if constexpr (QT == 4) {
          const uint4 hdr = lds_v4(blk);
          uint32_t q[W];
          if constexpr (W == 8) {
            const uint4 q0 = lds_v4(blk + 16 + 32 * unit + l0);
            const uint4 q1 = lds_v4(blk + 32 + 32 * unit + l0);
            q[0] = q0.x; q[1] = q0.y; q[2] = q0.z; q[3] = q0.w;
            q[4] = q1.x; q[5] = q1.y; q[6] = q1.z; q[7] = q1.w;
          } else if constexpr (W == 4) {
            const uint4 q0 = lds_v4(blk + 16 + 32 * unit + l0);
            q[0] = q0.x; q[1] = q0.y; q[2] = q0.z; q[3] = q0.w;
          } else {
            const uint2 q0 = lds_v2(blk + 16 + 32 * unit + l0);
            q[0] = q0.x; q[1] = q0.y;
          }
          // Accumulate S_A = sum x (2 + q/64) over the low nibbles (sub-block 2c) and
          // S_B = sum x (2 + q/1024) over the high nibbles (sub-block 2c+1).
#if KQ_PACKED_FMA
          float2 sa[B], sb[B];
#pragma unroll
          for (int b = 0; b < B; ++b) { sa[b] = f2(0.f, 0.f); sb[b] = f2(0.f, 0.f); }
#pragma unroll
          for (int w = 0; w < W; ++w) {
            const uint32_t lo = q[w] & 0x0F0F0F0Fu, hi = q[w] & 0xF0F0F0F0u;
            const float2 fa = f2(prmt_lo<0>(lo), prmt_lo<1>(lo));
            const float2 fb = f2(prmt_lo<2>(lo), prmt_lo<3>(lo));
            const float2 ga = f2(prmt_hi<0>(hi), prmt_hi<1>(hi));
            const float2 gb = f2(prmt_hi<2>(hi), prmt_hi<3>(hi));
#pragma unroll
            for (int b = 0; b < B; ++b) {
              sa[b] = __ffma2_rn(xr[b][0][2 * w], fa, sa[b]);
              sb[b] = __ffma2_rn(xr[b][1][2 * w], ga, sb[b]);
              sa[b] = __ffma2_rn(xr[b][0][2 * w + 1], fb, sa[b]);
              sb[b] = __ffma2_rn(xr[b][1][2 * w + 1], gb, sb[b]);
            }
          }
#define KQ_SA(b) (sa[b].x + sa[b].y)
#define KQ_SB(b) (sb[b].x + sb[b].y)
#else
          float sa[B][2], sb[B][2];
#pragma unroll
          for (int b = 0; b < B; ++b) { sa[b][0] = sa[b][1] = sb[b][0] = sb[b][1] = 0.f; }
#pragma unroll
          for (int w = 0; w < W; ++w) {
            const uint32_t lo = q[w] & 0x0F0F0F0Fu, hi = q[w] & 0xF0F0F0F0u;
            const float f0 = prmt_lo<0>(lo), f1 = prmt_lo<1>(lo), f2v = prmt_lo<2>(lo), f3 = prmt_lo<3>(lo);
            const float g0 = prmt_hi<0>(hi), g1 = prmt_hi<1>(hi), g2 = prmt_hi<2>(hi), g3 = prmt_hi<3>(hi);
#pragma unroll
            for (int b = 0; b < B; ++b) {
              float& A = sa[b][w & 1];
              float& Bv = sb[b][w & 1];
              A = fmaf(xr[b][0][2 * w].x, f0, A);
              Bv = fmaf(xr[b][1][2 * w].x, g0, Bv);
              A = fmaf(xr[b][0][2 * w].y, f1, A);
              Bv = fmaf(xr[b][1][2 * w].y, g1, Bv);
              A = fmaf(xr[b][0][2 * w + 1].x, f2v, A);
              Bv = fmaf(xr[b][1][2 * w + 1].x, g2, Bv);
              A = fmaf(xr[b][0][2 * w + 1].y, f3, A);
              Bv = fmaf(xr[b][1][2 * w + 1].y, g3, Bv);
            }
          }
#define KQ_SA(b) (sa[b][0] + sa[b][1])
#define KQ_SB(b) (sb[b][0] + sb[b][1])
#endif
          // scales and mins of sub-blocks 2c and 2c+1
          uint32_t sc0, m0, sc1, m1;
          if (!upper) {
            sc0 = (hdr.y >> sh0) & 63u; m0 = (hdr.z >> sh0) & 63u;
            sc1 = (hdr.y >> sh1) & 63u; m1 = (hdr.z >> sh1) & 63u;
          } else {
            sc0 = ((hdr.w >> sh0) & 15u) | (((hdr.y >> (sh0 + 6)) & 3u) << 4);
            m0 = ((hdr.w >> (sh0 + 4)) & 15u) | (((hdr.z >> (sh0 + 6)) & 3u) << 4);
            sc1 = ((hdr.w >> sh1) & 15u) | (((hdr.y >> (sh1 + 6)) & 3u) << 4);
            m1 = ((hdr.w >> (sh1 + 4)) & 15u) | (((hdr.z >> (sh1 + 6)) & 3u) << 4);
          }
          const float d = h2f(hdr.x & 0xffffu), dmin = h2f(hdr.x >> 16);
          const float fsc0 = static_cast<float>(sc0), fsc1 = static_cast<float>(sc1);
          const float fm0 = static_cast<float>(m0), fm1 = static_cast<float>(m1);
#pragma unroll
          for (int b = 0; b < B; ++b) {
            const float qa = fmaf(64.f, KQ_SA(b), -128.f * xs[b][0]);
            const float qb = fmaf(1024.f, KQ_SB(b), -2048.f * xs[b][1]);
            const float pos = fmaf(fsc0, qa, fsc1 * qb);
            const float neg = fmaf(fm0, xs[b][0], fm1 * xs[b][1]);
            acc[b] = fmaf(d, pos, -dmin * neg);
          }
#undef KQ_SA
#undef KQ_SB
        } else {
          uint32_t qa[W], qb[W], qh[W];
          lds_words_unaligned<W>(blk + 64 * unit + l0, qa);
          lds_words_unaligned<W>(blk + 64 * unit + 32 + l0, qb);
          lds_words_unaligned<W>(blk + 128 + 32 * unit + l0, qh);
          const uint32_t sbase = blk + 192 + 8 * unit + (l0 >> 4);
          float fsc[4];
#pragma unroll
          for (int g = 0; g < 4; ++g) fsc[g] = static_cast<float>(lds_s8(sbase + 2 * g));
          const float d = h2f(lds_u16(blk + 208));
#if KQ_PACKED_FMA
          float2 sg[B][4];
#pragma unroll
          for (int b = 0; b < B; ++b)
#pragma unroll
            for (int g = 0; g < 4; ++g) sg[b][g] = f2(0.f, 0.f);
#else
          float sg[B][4];
#pragma unroll
          for (int b = 0; b < B; ++b)
#pragma unroll
            for (int g = 0; g < 4; ++g) sg[b][g] = 0.f;
#endif
#pragma unroll
          for (int w = 0; w < W; ++w) {
            uint32_t qg[4];
            qg[0] = (qa[w] & 0x0F0F0F0Fu) | ((qh[w] << 4) & 0x30303030u);
            qg[1] = (qb[w] & 0x0F0F0F0Fu) | ((qh[w] << 2) & 0x30303030u);
            qg[2] = ((qa[w] >> 4) & 0x0F0F0F0Fu) | (qh[w] & 0x30303030u);
            qg[3] = ((qb[w] >> 4) & 0x0F0F0F0Fu) | ((qh[w] >> 2) & 0x30303030u);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
#if KQ_PACKED_FMA
              const float2 f01 = f2(prmt_lo<0>(qg[g]), prmt_lo<1>(qg[g]));
              const float2 f23 = f2(prmt_lo<2>(qg[g]), prmt_lo<3>(qg[g]));
#pragma unroll
              for (int b = 0; b < B; ++b) {
                sg[b][g] = __ffma2_rn(xr[b][g][2 * w], f01, sg[b][g]);
                sg[b][g] = __ffma2_rn(xr[b][g][2 * w + 1], f23, sg[b][g]);
              }
#else
              const float f0 = prmt_lo<0>(qg[g]), f1 = prmt_lo<1>(qg[g]);
              const float f2v = prmt_lo<2>(qg[g]), f3 = prmt_lo<3>(qg[g]);
#pragma unroll
              for (int b = 0; b < B; ++b) {
                sg[b][g] = fmaf(xr[b][g][2 * w].x, f0, sg[b][g]);
                sg[b][g] = fmaf(xr[b][g][2 * w].y, f1, sg[b][g]);
                sg[b][g] = fmaf(xr[b][g][2 * w + 1].x, f2v, sg[b][g]);
                sg[b][g] = fmaf(xr[b][g][2 * w + 1].y, f3, sg[b][g]);
              }
#endif
            }
          }
#pragma unroll
          for (int b = 0; b < B; ++b) {
            float tt = 0.f;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              // sum (q - 32) x = 64 S - 128 X - 32 X
#if KQ_PACKED_FMA
              const float qx = fmaf(64.f, sg[b][g].x + sg[b][g].y, -160.f * xs[b][g]);
#else
              const float qx = fmaf(64.f, sg[b][g], -160.f * xs[b][g]);
#endif
              tt = fmaf(fsc[g], qx, tt);
            }
            acc[b] = d * tt;
          }
        }
      }

      // lanes -> warp
#pragma unroll
      for (int b = 0; b < B; ++b) {
#pragma unroll
        for (int o = 16; o; o >>= 1) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
      }
      if (a.team_warps == 1) {
        // one warp is the whole team: lane 0 has the row
        if (lane == 0 && row < rs1) {
#pragma unroll
          for (int b = 0; b < B; ++b) {
            if (b < static_cast<int>(a.batch)) {
              if (R == 1) {
                a.y[b * a.ldy + row] = acc[b];
              } else if ((u & 1) == 0) {
                held[b] = acc[b];
              } else {
                a.y[b * a.ldy + row / 2] = pair_value(held[b], acc[b], a.epilogue, a.pair_scale);
              }
            }
          }
        }
      } else if (lane == 0) {
#pragma unroll
        for (int b = 0; b < B; ++b) tb[(u * a.team_warps + tw) * B + b] = acc[b];
      }
    }  // rows of this team in the tile
    __syncwarp();
    if (lane == 0) mbar_arrive(empty_bar(s));  // this warp is done reading slot s
    if (++s == a.ring) {
      s = 0;
      phase ^= 1;
    }

    if (a.team_warps > 1) {
      // warps of a team -> its rows, by the team's first warp
      named_barrier(1 + team, a.team_warps * 32);
      if (tw == 0) {
        const uint32_t nout = (a.per_team / R) * B;
        for (uint32_t o = lane; o < nout; o += 32) {
          const uint32_t i = o / B, b = o % B;  // B is a compile-time power of two
          const uint32_t u0 = i * R;
          const uint32_t rho = i * round_stride + team * R;
          const uint32_t row = rs0 + rho;
          if (row < rs1 && b < a.batch) {
            float v0 = 0.f;
            for (uint32_t w = 0; w < a.team_warps; ++w) v0 += tb[(u0 * a.team_warps + w) * B + b];
            if (R == 1) {
              a.y[b * a.ldy + row] = v0;
            } else {
              float v1 = 0.f;
              for (uint32_t w = 0; w < a.team_warps; ++w)
                v1 += tb[((u0 + 1) * a.team_warps + w) * B + b];
              a.y[b * a.ldy + row / 2] = pair_value(v0, v1, a.epilogue, a.pair_scale);
            }
          }
        }
      }
    }
  }

  if (a.npush) {
    // Batch-1 push: once the CTA's outputs are in y, copy those below push_rows into every
    // rank's full vector, and only then (system fence) add their count on each rank.
    named_barrier(kPushBarrier, consumers * 32);
    const uint32_t o0 = r_begin / a.row_unit, o1 = min(r_end / a.row_unit, a.push_rows);
    for (uint32_t o = o0 + threadIdx.x; o < o1; o += consumers * 32) {
      const float v = __ldcg(a.y + o);
      for (uint32_t p = 0; p < a.npush; ++p) a.push_y[p][o] = v;
    }
    __threadfence_system();
    named_barrier(kPushBarrier, consumers * 32);
    if (threadIdx.x == 0 && o1 > o0)
      for (uint32_t p = 0; p < a.npush; ++p) atomicAdd_system(a.push_cnt[p], (unsigned long long)(o1 - o0));
  }
}

struct Instance {
  const void* fn;
  int max_threads;
  int l4, l6;
};

template <int QT, int B>
Instance instance() {
  return Instance{reinterpret_cast<const void*>(&matvec_kernel<QT, B>), Geo<B>::kMaxThreads,
                  Geo<B>::kL4, Geo<B>::kL6};
}

Instance pick(int qt, int bt) {
  if (qt == 4) {
    switch (bt) {
      case 1: return instance<4, 1>();
      case 2: return instance<4, 2>();
      case 4: return instance<4, 4>();
      default: return instance<4, 8>();
    }
  }
  switch (bt) {
    case 1: return instance<6, 1>();
    case 2: return instance<6, 2>();
    case 4: return instance<6, 4>();
    default: return instance<6, 8>();
  }
}

// Tiles of ~96 KB in a ring of ~210 KB: fewer, larger tiles amortise the per-tile hand-offs
// (mbarrier waits, the team barrier and reduction), which measured faster than 24-64 KB tiles.
#ifndef KQ_TILE_KB
#define KQ_TILE_KB 96
#endif
#ifndef KQ_RING_KB
#define KQ_RING_KB 210
#endif
constexpr uint32_t kRingBudget = KQ_RING_KB * 1024;  // bytes of ring per CTA we aim for
constexpr uint64_t kTileTarget = KQ_TILE_KB * 1024;  // bytes per tile we aim for

}  // namespace

int matvec_prepare(kq_ctx* ctx) {
  for (int qt : {4, 6})
    for (int bt : {1, 2, 4, 8}) {
      const Instance in = pick(qt, bt);
      cudaError_t e = cudaFuncSetAttribute(in.fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           ctx->max_smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute", "matvec kernel");
    }
  return KQ_OK;
}

int check_desc(const kq_matvec_desc& d, const char* call) {
  int qt;
  if (d.type == KQ_TYPE_Q4_K)
    qt = 4;
  else if (d.type == KQ_TYPE_Q5_K)
    qt = 5;
  else if (d.type == KQ_TYPE_Q6_K)
    qt = 6;
  else
    return fail(KQ_E_INVALID, call,
                "type must be KQ_TYPE_Q4_K (12), KQ_TYPE_Q5_K (13) or KQ_TYPE_Q6_K (14)");
  if (d.rows == 0 || d.k == 0 || d.k % kQK != 0)
    return fail(KQ_E_INVALID, call,
                "rows must be > 0 and k a positive multiple of 256 (rows " +
                    std::to_string(d.rows) + ", k " + std::to_string(d.k) + ")");
  const uint32_t max_batch = qt == 6 ? 8 : 64;
  if (d.batch < 1 || d.batch > max_batch)
    return fail(KQ_E_INVALID, call,
                "batch must be 1.." + std::to_string(max_batch) + " (got " + std::to_string(d.batch) + ")");
  {
    const uint32_t paths = d.flags & (KQ_FLAG_TENSOR_CORES | KQ_FLAG_CUDA_CORES | KQ_FLAG_WARP_MMA);
    if (paths & (paths - 1))
      return fail(KQ_E_INVALID, call,
                  "KQ_FLAG_TENSOR_CORES, KQ_FLAG_CUDA_CORES and KQ_FLAG_WARP_MMA exclude each other");
  }
  if (!d.w || !d.x || !d.y) return fail(KQ_E_INVALID, call, "null pointer");
  if (d.w % 16 || d.x % 16 || d.y % 4)
    return fail(KQ_E_INVALID, call, "w and x must be 16-byte aligned, y 4-byte aligned");
  if (d.prologue > KQ_PROLOGUE_RMSNORM || d.epilogue > KQ_EPILOGUE_SILU_PRODUCT)
    return fail(KQ_E_INVALID, call, "unknown prologue or epilogue");
  const bool pair = d.epilogue != KQ_EPILOGUE_NONE;  // the products take rows in pairs
  if (pair && d.rows % 2) return fail(KQ_E_INVALID, call, "pair product needs an even row count");
  const uint64_t ldx = d.ldx ? d.ldx : d.k;
  const uint64_t out_rows = pair ? d.rows / 2 : d.rows;
  const uint64_t ldy = d.ldy ? d.ldy : out_rows;
  if (ldx < d.k || ldx % 4) return fail(KQ_E_INVALID, call, "ldx must be >= k and a multiple of 4");
  if (ldy < out_rows) return fail(KQ_E_INVALID, call, "ldy must be >= the output rows");
  return KQ_OK;
}

int matvec(kq_ctx* ctx, const kq_matvec_desc& d, cudaStream_t stream, const kq_push_desc* push) {
  const char* call = push ? "kq_matvec_push" : "kq_matvec";
  if (d.type == KQ_TYPE_Q2_K || d.type == KQ_TYPE_Q3_K || d.type == KQ_TYPE_Q8_0) {
    if (push) return fail(KQ_E_UNSUPPORTED, call, "the push exchange serves Q4_K, Q5_K and Q6_K");
    return types_matvec(ctx, d, stream);
  }
  const int rc = check_desc(d, call);
  if (rc) return rc;
  const int qt = d.type == KQ_TYPE_Q4_K ? 4 : d.type == KQ_TYPE_Q5_K ? 5 : 6;
  const bool pair = d.epilogue != KQ_EPILOGUE_NONE;
  const uint64_t ldx = d.ldx ? d.ldx : d.k;
  const uint64_t ldy = d.ldy ? d.ldy : (pair ? d.rows / 2 : d.rows);

  // Path: the tensor cores above batch 8 (and when asked), the CUDA cores otherwise.
  if (push) {
    if (d.batch != 1 || (d.flags & KQ_FLAG_TENSOR_CORES))
      return fail(KQ_E_INVALID, call,
                  "the push exchange serves batch 1 on the warp-MMA or CUDA-core kernel");
    if (push->npush > 8) return fail(KQ_E_INVALID, call, "npush must be 0..8");
    const bool tagged = (push->flags & KQ_PUSH_TAGGED) != 0;
    if (push->flags & ~uint32_t(KQ_PUSH_TAGGED | KQ_PUSH_TAGGED_X))
      return fail(KQ_E_INVALID, call, "unknown push flags");
    if ((push->flags & KQ_PUSH_TAGGED_X) && !tagged)
      return fail(KQ_E_INVALID, call, "KQ_PUSH_TAGGED_X goes with KQ_PUSH_TAGGED");
    if (tagged && (d.flags & KQ_FLAG_CUDA_CORES))
      return fail(KQ_E_UNSUPPORTED, call, "tagged pushes run on the warp-MMA kernel");
    for (uint32_t p = 0; p < push->npush; ++p)
      if (!push->y[p] || (tagged ? push->y[p] % 8 : (!push->counter[p] || push->y[p] % 4 || push->counter[p] % 8)))
        return fail(KQ_E_INVALID, call, "push target " + std::to_string(p) + " is null or misaligned");
    if (push->wait_counter && (!push->epoch || push->wait_counter % 8 || push->epoch % 8))
      return fail(KQ_E_INVALID, call, "wait_counter needs an 8-byte aligned epoch and counter");
  }
  // The push exchange: the warp-MMA kernel's integer path unless the CUDA cores are asked for.
  if (push && !(d.flags & KQ_FLAG_CUDA_CORES)) return warpmma_push(ctx, d, *push, ldx, ldy, stream);
  if (qt == 5) {  // Q5_K: batch 1 on the warp-MMA kernel, batch 2..64 (or when asked) on the tensor cores
    if (d.flags & KQ_FLAG_CUDA_CORES)
      return fail(KQ_E_UNSUPPORTED, call, "Q5_K has no CUDA-core kernel");
    if (d.batch == 1 && !(d.flags & KQ_FLAG_TENSOR_CORES)) return warpmma_matvec(ctx, d, ldx, ldy, stream);
    if ((d.flags & KQ_FLAG_WARP_MMA) || !mma_supports(d))
      return fail(KQ_E_UNSUPPORTED, call,
                  "Q5_K above batch 1 is served by the tensor-core kernel, batch 2..64 without "
                  "prologue or epilogue");
    return mma_matvec(ctx, d, ldx, ldy, stream);
  }
  if (d.flags & KQ_FLAG_WARP_MMA) {
    if (push || !warpmma_supports(d))
      return fail(KQ_E_UNSUPPORTED, call,
                  "the warp-MMA kernel serves Q4_K batch 1..8 and Q6_K batch 1, without push");
    return warpmma_matvec(ctx, d, ldx, ldy, stream);
  }
  if (!push && !(d.flags & (KQ_FLAG_TENSOR_CORES | KQ_FLAG_CUDA_CORES)) && warpmma_supports(d)) {
    const int rc = warpmma_matvec(ctx, d, ldx, ldy, stream);
    if (rc != KQ_E_UNSUPPORTED) return rc;  // a shape it cannot hold goes to the CUDA cores
  }
  const bool want_tc = !push && ((d.flags & KQ_FLAG_TENSOR_CORES) || (d.batch > 8 && !(d.flags & KQ_FLAG_CUDA_CORES)));
  if (want_tc) {
    if (!mma_supports(d))
      return fail(KQ_E_UNSUPPORTED, call,
                  "the tensor-core kernel serves Q4_K and Q5_K without prologue/epilogue, batch 1..64");
    return mma_matvec(ctx, d, ldx, ldy, stream);
  }
  if (d.batch > 8)
    return fail(KQ_E_UNSUPPORTED, call, "the CUDA-core kernel serves batch 1..8");
  const int bt = d.batch == 1 ? 1 : d.batch == 2 ? 2 : d.batch <= 4 ? 4 : 8;
  const Instance in = pick(qt, bt);
  const int L = qt == 4 ? in.l4 : in.l6;
  const uint32_t blk = qt == 4 ? kQ4KBytes : kQ6KBytes;
  const uint32_t ppb = (qt == 4 ? 128 : 64) / L;
  const uint32_t nb = d.k / kQK;
  const uint32_t team_lanes = ppb * nb;
  const uint32_t team_warps = (team_lanes + 31) / 32;
  const uint32_t max_consumers = in.max_threads / 32 - 1;
  if (team_warps > max_consumers)
    return fail(KQ_E_UNSUPPORTED, call,
                "k " + std::to_string(d.k) + " is past this build's limit for batch " +
                    std::to_string(d.batch) + " (" + std::to_string(max_consumers * 32 / ppb * kQK) +
                    ")");
  const uint32_t pmax = std::min<uint32_t>(14, max_consumers / team_warps);  // named barriers 1..14

  const uint32_t row_unit = pair ? 2 : 1;
  const uint64_t units = d.rows / row_unit;
  const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>(ctx->sm_count, units));
  const uint64_t rows_per_cta = ((units + grid - 1) / grid) * row_unit;
  // Teams: as many as fit, trimmed so that the CTA's rows split evenly over its tiles.
  const uint64_t rounds = (rows_per_cta + pmax - 1) / pmax;
  const uint32_t P = static_cast<uint32_t>((rows_per_cta + rounds - 1) / rounds);
  const uint64_t rb = uint64_t(nb) * blk;
  // Rows per team per tile: tiles of about kTileTarget bytes, no more rows than the CTA has.
  uint32_t U = static_cast<uint32_t>(std::max<uint64_t>(1, kTileTarget / (uint64_t(P) * rb)));
  U = static_cast<uint32_t>(std::min<uint64_t>(U, (rows_per_cta + P - 1) / P));
  if (pair) U += U & 1;  // a team takes both rows of a pair
  const uint32_t slot = static_cast<uint32_t>(((uint64_t(P) * U * rb + 32 + 127) / 128) * 128);
  const uint32_t consumers = P * team_warps;
  const uint32_t red_bytes = 2 * consumers * U * bt * 4;
  const uint32_t fixed = red_bytes + 2 * 8 * 8 + 128;
  uint32_t ring = std::min<uint32_t>(8, std::max<uint32_t>(2, kRingBudget / slot));
  while (ring > 2 && ring * slot + fixed > static_cast<uint32_t>(ctx->max_smem)) --ring;
  const uint32_t smem = ring * slot + fixed;
  if (smem > static_cast<uint32_t>(ctx->max_smem))
    return fail(KQ_E_UNSUPPORTED, call, "row tile does not fit in shared memory (k too large)");

  MatvecArgs args;
  args.W = reinterpret_cast<const uint8_t*>(d.w);
  args.x = reinterpret_cast<const float*>(d.x);
  args.y = reinterpret_cast<float*>(d.y);
  args.err = ctx->err;
  args.ldx = ldx;
  args.ldy = ldy;
  args.total_bytes = uint64_t(d.rows) * rb;
  args.rows = d.rows;
  args.nb = nb;
  args.batch = d.batch;
  args.team_warps = team_warps;
  args.teams = P;
  args.per_team = U;
  args.ring = ring;
  args.slot_bytes = slot;
  args.row_unit = row_unit;
  args.prologue = d.prologue;
  args.epilogue = d.epilogue;
  args.flags = d.flags;
  args.eps = d.eps;
  args.pair_scale = d.pair_scale;
  args.npush = push ? push->npush : 0;
  args.push_rows = push ? push->push_rows : 0;
  for (int p = 0; p < 8; ++p) {
    args.push_y[p] = push && p < static_cast<int>(push->npush) ? reinterpret_cast<float*>(push->y[p]) : nullptr;
    args.push_cnt[p] = push && p < static_cast<int>(push->npush)
                           ? reinterpret_cast<unsigned long long*>(push->counter[p]) : nullptr;
  }
  args.wait_cnt = push && push->wait_counter ? reinterpret_cast<const unsigned long long*>(push->wait_counter) : nullptr;
  args.epoch = push && push->wait_counter ? reinterpret_cast<const unsigned long long*>(push->epoch) : nullptr;
  args.wait_mul = push ? push->wait_mul : 0;
  args.wait_add = push ? push->wait_add : 0;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((consumers + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (d.flags & KQ_FLAG_NO_PDL) ? 0 : 1;
  void* params[] = {&args};
  cudaError_t e = cudaLaunchKernelExC(&cfg, in.fn, params);
  if (e != cudaSuccess)
    return cuda_fail(e, "cudaLaunchKernelExC",
                     "matvec grid " + std::to_string(grid) + " x " +
                         std::to_string((consumers + 1) * 32) + " threads, " +
                         std::to_string(smem) + " B shared");
  return KQ_OK;
}

}  // namespace kq
