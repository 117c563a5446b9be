// kq_mma.cu -- the Q4_K / Q5_K small-batch matmul (batch 2..64) on the 5th-generation tensor cores.
//
// Y[b, r] = sum_k W[r, k] X[b, k] as D = A * B^T per tile of TM <= 128 weight rows:
//   raw W: one 2-D TMA copy per super-block column of the tile (TM rows x 144 bytes: a box of a
//     tensor map over W viewed as rows x row-bytes), into a ring of kRaw shared-memory stages.
//     The rows land 144 bytes apart, so eight consecutive rows read at one offset hit eight
//     different bank groups (144 / 16 = 9 is odd): the dequantisers' loads do not conflict;
//   A (128 lanes x 256 K per super-block, f16) is written by the dequantising threads straight
//     into tensor memory (tcgen05.st): no shared-memory A tile, whose write and read by the tensor
//     core (512 bytes per row and super-block, 3.5x the raw bytes) would bound the kernel at these
//     batch sizes;
//   B (N = batch padded to 16/32/64, K-major f16) is X, converted once per call by a small
//     pre-pass into the exact shared-memory layout of the B operand (kept in the context's
//     scratch buffer), and fetched per super-block with one bulk copy;
//   D (128 lanes x N f32 columns) accumulates in tensor memory over the whole row; four epilogue
//     warps read it back with tcgen05.ld and write Y.
// A warp may only reach the tensor-memory lanes of its quadrant (warp % 4), which is also its
// scheduler, so a tile's rows are spread evenly over the four quadrants: row q * nq + t of the
// tile (nq = TM / 4 rounded up) is lane 32 q + t. Every scheduler then dequantises the same
// number of rows whatever TM is. The rows are cut into tiles of equal height TM (the last one
// shorter), tile t going to CTA t % grid. Warp roles:
//   0       tensor-memory owner and MMA issuer: 16 tcgen05.mma (K = 16) per super-block, then
//           tcgen05.commit to free the A and B slots, and at the end of a tile to publish D;
//   1       loader: the raw W copies, up to kRaw super-blocks ahead, and the B copies;
//   2..9    dequantisers: lane quadrant w % 4, half (w - 2) / 4 of each super-block; thread t
//           holds row q * nq + t (threads past the quadrant's rows store don't-care lanes);
//   10..13  epilogue.
// The dequantiser keeps the canonical weight w = d*sc*q - dmin*m to one f16 rounding: q comes
// out of the 1024 + q magic exactly (one LOP3 per two weights and one HSUB2), then one HFMA2
// computes q * (d*sc) - dmin*m. The K order inside each 8-weight group follows the byte lanes
// (l, l+2, l+1, l+3 of the low nibbles, then the same of the high nibbles); the pre-pass
// permutes X alike, so the contraction is unchanged.
//
// Every wait is bounded (kq_device.cuh): a wait that gives up records an error word, and all
// roles then run to the end without waiting; the loader then waits (bounded) for its copies in
// flight, and the CTA frees its tensor memory and exits.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "kq_device.cuh"
#include "kq_internal.h"
#include "kq_tc.cuh"

namespace kq {
namespace {

constexpr int kTileM = 128;           // MMA M = tensor-memory lanes; a tile holds TM <= 128 rows
// raw W stages (super-blocks in flight per CTA): fewer for Q5_K's 176-byte blocks
template <int QT>
constexpr int kRawStages = QT == 4 ? 8 : 6;
template <int QT>
constexpr uint32_t kBlockBytes = QT == 4 ? kQ4KBytes : kQ5KBytes;
constexpr int kASlots = 3;            // A slots in tensor memory, one super-block (128 columns) each
constexpr int kThreads = 14 * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kDCol = kASlots * 128;  // first D column

struct MmaArgs {
  const uint8_t* xp;  // X in B-operand layout: per block 32 k-groups x NPAD rows x 16 B
  float* y;
  unsigned* err;
  uint64_t ldy;
  uint32_t rows, nb, batch, flags;
  uint32_t tm;          // rows per tile
  uint32_t nq;          // rows per lane quadrant: ceil(tm / 4)
  uint32_t ntiles;      // tiles of the matrix
  uint32_t raw_stride;  // bytes per raw stage (tm * 144 rounded up to 1024)
};

// B slots: one super-block of X each (NPAD x 512 bytes), as many as leave room for the raw ring.
__host__ __device__ constexpr uint32_t b_slots(uint32_t npad) { return npad <= 16 ? 4 : npad <= 32 ? 3 : 2; }
__host__ __device__ constexpr uint32_t b_slot_bytes(uint32_t npad) { return npad * 512; }

template <int QT>
__host__ __device__ constexpr uint32_t smem_bytes(uint32_t npad, uint32_t raw_stride) {
  return 1024 + kRawStages<QT> * raw_stride + b_slots(npad) * b_slot_bytes(npad) + 512;  // + barriers
}

// Waits on `bar` for `parity` as one warp: lane 0 polls, every lane gets the outcome.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int* failed,
                                          unsigned* err, unsigned code) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    if (*reinterpret_cast<volatile int*>(failed)) {
      ok = 0;
    } else if (!mbar_wait(bar, parity)) {
      *reinterpret_cast<volatile int*>(failed) = 1;
      report_error(err, code);
      ok = 0;
    }
  }
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// 2-D tiled TMA load of box (x, y) of `tmap` into shared `dst`, completing on `bar`; no multicast.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tmap, uint32_t x,
                                            uint32_t y, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// X (f32, batch vectors of stride ldx) -> B-operand layout in f16: for block kb, k-group
// j = 8c + ww and row n, 16 bytes at ((kb*32 + j) * NPAD + n) * 16 holding x[e+0], x[e+2],
// x[e+1], x[e+3], x[e+32], x[e+34], x[e+33], x[e+35] with e = kb*256 + 64c + 4ww; zeros for
// n >= batch. One thread per 16 bytes.
__global__ void xperm_kernel(uint4* xp, const float* x, uint64_t ldx, uint32_t nb, uint32_t batch,
                             uint32_t npad) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t total = nb * 32 * npad;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t n = i % npad, kj = i / npad;
    const uint32_t kb = kj >> 5, j = kj & 31, c = j >> 3, ww = j & 7;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < batch) {
      const float* e = x + n * ldx + uint64_t(kb) * kQK + 64 * c + 4 * ww;
      const float4 lo = *reinterpret_cast<const float4*>(e);
      const float4 hi = *reinterpret_cast<const float4*>(e + 32);
      v.x = h2_bits(__floats2half2_rn(lo.x, lo.z));
      v.y = h2_bits(__floats2half2_rn(lo.y, lo.w));
      v.z = h2_bits(__floats2half2_rn(hi.x, hi.z));
      v.w = h2_bits(__floats2half2_rn(hi.y, hi.w));
    }
    xp[i] = v;
  }
}

template <int QT, int NPAD>
__global__ void __launch_bounds__(kThreads, 1)
    mma_kernel(const __grid_constant__ CUtensorMap wmap, const MmaArgs a) {
  constexpr uint32_t BS = b_slots(NPAD), kB = b_slot_bytes(NPAD);
  constexpr int kRaw = kRawStages<QT>;
  constexpr uint32_t kBlk = kBlockBytes<QT>;
  constexpr uint32_t kQs = QT == 4 ? 16 : 48;  // offset of qs in a block (Q5_K: qh[32] before it)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t raw_s = base;                        // [kRaw][raw_stride]
  const uint32_t b_s = raw_s + kRaw * a.raw_stride;   // [BS][kB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + (b_s + BS * kB - smem_u32(smem_raw)));
  uint64_t* raw_full = bars;                 // [kRaw]    loader (tx bytes) -> dequantisers
  uint64_t* raw_empty = raw_full + kRaw;     // [kRaw]    dequantisers -> loader
  uint64_t* a_full = raw_empty + kRaw;       // [kASlots] dequantisers -> MMA
  uint64_t* a_empty = a_full + kASlots;      // [kASlots] MMA commit -> dequantisers
  uint64_t* b_full = a_empty + kASlots;      // [BS]      loader (tx bytes) -> MMA
  uint64_t* b_empty = b_full + BS;           // [BS]      MMA commit -> loader
  uint64_t* d_full = b_empty + BS;           // [2]       MMA commit -> epilogue
  uint64_t* d_empty = d_full + 2;            // [2]       epilogue -> MMA
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(d_empty + 2);
  int* failed = reinterpret_cast<int*>(tmem_holder + 1);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tiles blockIdx.x, blockIdx.x + gridDim.x, ...
  const uint32_t ntiles = (a.ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x;
  const uint32_t total = ntiles * a.nb;  // super-blocks this CTA streams

  if (threadIdx.x == 0) {
    *failed = 0;
    for (int i = 0; i < kRaw; ++i) {
      mbar_init(smem_u32(&raw_full[i]), 1);
      mbar_init(smem_u32(&raw_empty[i]), 8);
    }
    for (int i = 0; i < kASlots; ++i) {
      mbar_init(smem_u32(&a_full[i]), 8);
      mbar_init(smem_u32(&a_empty[i]), 1);
    }
    for (uint32_t i = 0; i < BS; ++i) {
      mbar_init(smem_u32(&b_full[i]), 1);
      mbar_init(smem_u32(&b_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&d_full[i]), 1);
      mbar_init(smem_u32(&d_empty[i]), 4);
    }
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = idesc_f16_f32(kTileM, NPAD);
    uint32_t g = 0;
    for (uint32_t T = 0; T < ntiles; ++T) {
      const uint32_t dbuf = T & 1;
      if (T >= 2) warp_wait(smem_u32(&d_empty[dbuf]), ((T / 2) - 1) & 1, failed, a.err, kErrWaitEmpty);
      tc_fence_after();
      const uint32_t dcol = tmem + kDCol + dbuf * NPAD;
      for (uint32_t kb = 0; kb < a.nb; ++kb, ++g) {
        const uint32_t as = g % kASlots, bs = g % BS;
        const bool ok = warp_wait(smem_u32(&a_full[as]), (g / kASlots) & 1, failed, a.err, kErrWaitFull) &&
                        warp_wait(smem_u32(&b_full[bs]), (g / BS) & 1, failed, a.err, kErrWaitFull);
        tc_fence_after();
        if (lane == 0) {
          if (ok) {
            const uint32_t bslot = b_s + bs * kB;
#pragma unroll
            for (uint32_t s = 0; s < 16; ++s) {
              const uint64_t bdesc = smem_desc(bslot + s * 2 * NPAD * 16, NPAD * 16, 128);
              mma_f16_ts(dcol, tmem + as * 128 + s * 8, bdesc, idesc, (kb | s) != 0);
            }
          }
          mma_commit(smem_u32(&a_empty[as]));
          mma_commit(smem_u32(&b_empty[bs]));
        }
        __syncwarp();
      }
      if (lane == 0) mma_commit(smem_u32(&d_full[dbuf]));
      __syncwarp();
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- loader
    const uint64_t pol = policy_evict_first();
    const uint32_t raw_bytes = a.tm * kBlk;
    constexpr uint32_t kLag = kRaw / 2;  // the B copies trail the raw copies by this many blocks
    if (!(a.flags & KQ_FLAG_WEIGHTS_STATIC)) pdl_wait();  // W may be the previous kernel's output
    for (uint32_t step = 0; step < total + kLag; ++step) {
      if (step < total) {
        const uint32_t g = step, rs = g % kRaw;
        if (g >= kRaw) warp_wait(smem_u32(&raw_empty[rs]), ((g / kRaw) - 1) & 1, failed, a.err, kErrWaitEmpty);
        if (lane == 0) {
          const uint32_t T = g / a.nb, kb = g - T * a.nb;
          const uint32_t row0 = (blockIdx.x + T * gridDim.x) * a.tm;
          const uint32_t full = smem_u32(&raw_full[rs]);
          mbar_arrive_expect_tx(full, raw_bytes);
          tma_load_2d(raw_s + rs * a.raw_stride, &wmap, kb * kBlk, row0, full, pol);
        }
        __syncwarp();
      }
      if (step >= kLag) {
        if (step == kLag) pdl_wait();  // the B tiles come from the pre-pass just before this kernel
        const uint32_t gb = step - kLag, kb = gb % a.nb, bs = gb % BS;
        if (gb >= BS) warp_wait(smem_u32(&b_empty[bs]), ((gb / BS) - 1) & 1, failed, a.err, kErrWaitEmpty);
        if (lane == 0) {
          const uint32_t full = smem_u32(&b_full[bs]);
          mbar_arrive_expect_tx(full, kB);
          bulk_g2s(b_s + bs * kB, a.xp + uint64_t(kb) * kB, kB, full);
        }
        __syncwarp();
      }
    }
    // every copy must have landed before the CTA exits, also when a wait gave up
    if (lane == 0 && *reinterpret_cast<volatile int*>(failed)) {
      for (uint32_t g = total > kRaw ? total - kRaw : 0; g < total; ++g)
        mbar_wait(smem_u32(&raw_full[g % kRaw]), (g / kRaw) & 1);
      for (uint32_t g = total > BS ? total - BS : 0; g < total; ++g)
        mbar_wait(smem_u32(&b_full[g % BS]), (g / BS) & 1);
    }
    __syncwarp();
  } else if (warp < 10) {
    // ---------------------------------------------------------------- dequantisers
    const uint32_t quad = warp & 3;         // tensor-memory lanes 32 quad .. +31
    const uint32_t part = (warp - 2) >> 2;  // chunks 2 part, 2 part + 1 of each block
    const uint32_t trow = quad * a.nq + lane;  // this thread's row of the tile
    const bool valid = lane < a.nq && trow < a.tm;
    const uint32_t src_row = (valid ? trow : 0) * kBlk;
    const uint32_t lane_base = tmem + ((quad * 32) << 16) + part * 64;
    const __half2 magic = __half2half2(__ushort_as_half(0x6400));  // 1024
    for (uint32_t g = 0; g < total; ++g) {
      const uint32_t rs = g % kRaw, as = g % kASlots;
      const bool ok = warp_wait(smem_u32(&raw_full[rs]), (g / kRaw) & 1, failed, a.err, kErrWaitFull);
      if (g >= kASlots) warp_wait(smem_u32(&a_empty[as]), ((g / kASlots) - 1) & 1, failed, a.err, kErrWaitEmpty);
      tc_fence_after();
      const uint32_t src = raw_s + rs * a.raw_stride + src_row;
      const uint4 hdr = ok ? lds_v4(src) : make_uint4(0, 0, 0, 0);
      const float d = h2f(hdr.x & 0xffffu), dmin = h2f(hdr.x >> 16);
      // Q5_K: the fifth bits of chunk c's byte l are bits 2c (low nibble) and 2c+1 (high nibble)
      // of qh[l]; the 16 qh bytes of half hh serve both of this thread's chunks
      uint4 qh[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      if (QT == 5 && ok) {
        qh[0] = lds_v4(src + 16);
        qh[1] = lds_v4(src + 32);
      }
      const uint32_t taddr = lane_base + as * 128;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t sc0, m0, sc1, m1;  // sub-blocks 2c (low nibbles) and 2c+1 (high nibbles)
        if (part == 0) {
          sc0 = (hdr.y >> (16 * cc)) & 63u;
          m0 = (hdr.z >> (16 * cc)) & 63u;
          sc1 = (hdr.y >> (16 * cc + 8)) & 63u;
          m1 = (hdr.z >> (16 * cc + 8)) & 63u;
        } else {
          const uint32_t s0 = 16 * cc, s1 = 16 * cc + 8;
          sc0 = ((hdr.w >> s0) & 15u) | (((hdr.y >> (s0 + 6)) & 3u) << 4);
          m0 = ((hdr.w >> (s0 + 4)) & 15u) | (((hdr.z >> (s0 + 6)) & 3u) << 4);
          sc1 = ((hdr.w >> s1) & 15u) | (((hdr.y >> (s1 + 6)) & 3u) << 4);
          m1 = ((hdr.w >> (s1 + 4)) & 15u) | (((hdr.z >> (s1 + 6)) & 3u) << 4);
        }
        // low nibbles: q * s0 - m0; high nibbles hold 16 q: 16q * (s1 / 16) - m1
        const __half2 s_lo = __half2half2(__float2half_rn(d * static_cast<float>(sc0)));
        const __half2 mn_lo = __half2half2(__float2half_rn(-dmin * static_cast<float>(m0)));
        const __half2 s_hi = __half2half2(__float2half_rn(d * static_cast<float>(sc1) * 0.0625f));
        const __half2 mn_hi = __half2half2(__float2half_rn(-dmin * static_cast<float>(m1)));
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {  // 16 bytes of qs -> 16 tensor-memory columns
          const uint4 q = ok ? lds_v4(src + kQs + 64 * part + 32 * cc + 16 * hh) : make_uint4(0, 0, 0, 0);
          const uint32_t words[4] = {q.x, q.y, q.z, q.w};
          const uint32_t hwords[4] = {qh[hh].x, qh[hh].y, qh[hh].z, qh[hh].w};
          uint32_t v[16];
#pragma unroll
          for (int ww = 0; ww < 4; ++ww) {
            const uint32_t w = words[ww], w8 = w >> 8;
            uint32_t la0 = (w & 0x000F000Fu) | 0x64006400u, la1 = (w8 & 0x000F000Fu) | 0x64006400u;
            uint32_t lb0 = (w & 0x00F000F0u) | 0x64006400u, lb1 = (w8 & 0x00F000F0u) | 0x64006400u;
            if (QT == 5) {  // 1024 + q + 16 h and 1024 + 16 (q + 16 h)
              const uint32_t h = hwords[ww] >> (2 * (2 * part + cc));
              la0 |= (h << 4) & 0x00100010u;  // bytes 0, 2, bit 2c
              la1 |= (h >> 4) & 0x00100010u;  // bytes 1, 3, bit 2c
              lb0 |= (h << 7) & 0x01000100u;  // bytes 0, 2, bit 2c+1
              lb1 |= (h >> 1) & 0x01000100u;  // bytes 1, 3, bit 2c+1
            }
            const __half2 a0 = __hsub2(bits_h2(la0), magic);
            const __half2 a1 = __hsub2(bits_h2(la1), magic);
            const __half2 b0 = __hsub2(bits_h2(lb0), magic);
            const __half2 b1 = __hsub2(bits_h2(lb1), magic);
            v[4 * ww + 0] = h2_bits(__hfma2(a0, s_lo, mn_lo));
            v[4 * ww + 1] = h2_bits(__hfma2(a1, s_lo, mn_lo));
            v[4 * ww + 2] = h2_bits(__hfma2(b0, s_hi, mn_hi));
            v[4 * ww + 3] = h2_bits(__hfma2(b1, s_hi, mn_hi));
          }
          tmem_st16(taddr + 32 * cc + 16 * hh, v);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&a_full[as]));
        mbar_arrive(smem_u32(&raw_empty[rs]));
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    pdl_wait();
    const uint32_t quad = warp & 3;
    const uint32_t trow = quad * a.nq + lane;
    for (uint32_t T = 0; T < ntiles; ++T) {
      const uint32_t dbuf = T & 1;
      const bool ok = warp_wait(smem_u32(&d_full[dbuf]), (T / 2) & 1, failed, a.err, kErrWaitFull);
      tc_fence_after();
      uint32_t v[NPAD];
#pragma unroll
      for (int c = 0; c < NPAD / 16; ++c) {
        uint32_t t16[16];
        tmem_ld16(tmem + ((quad * 32) << 16) + kDCol + dbuf * NPAD + 16 * c, t16);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[16 * c + j] = t16[j];
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&d_empty[dbuf]));
      const uint32_t row = (blockIdx.x + T * gridDim.x) * a.tm + trow;
      if (ok && lane < a.nq && trow < a.tm && row < a.rows) {
#pragma unroll
        for (int n = 0; n < NPAD; ++n)
          if (n < static_cast<int>(a.batch)) a.y[n * a.ldy + row] = __uint_as_float(v[n]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int QT>
const void* mma_fn(uint32_t npad) {
  return npad == 16   ? reinterpret_cast<const void*>(&mma_kernel<QT, 16>)
         : npad == 32 ? reinterpret_cast<const void*>(&mma_kernel<QT, 32>)
                      : reinterpret_cast<const void*>(&mma_kernel<QT, 64>);
}

const void* mma_fn_for(int qt, uint32_t npad) { return qt == 4 ? mma_fn<4>(npad) : mma_fn<5>(npad); }

uint32_t npad_for(uint32_t batch) { return batch <= 16 ? 16 : batch <= 32 ? 32 : 64; }

uint32_t raw_stride_for(int qt, uint32_t tm) {
  return (tm * (qt == 4 ? kBlockBytes<4> : kBlockBytes<5>) + 1023u) & ~1023u;
}

uint32_t smem_for(int qt, uint32_t npad, uint32_t raw_stride) {
  return qt == 4 ? smem_bytes<4>(npad, raw_stride) : smem_bytes<5>(npad, raw_stride);
}

// The opt-in shared memory the kernel for (qt, npad) is given: enough for 128-row tiles.
int smem_limit(int qt, uint32_t npad) { return static_cast<int>(smem_for(qt, npad, raw_stride_for(qt, kTileM))); }

// Sets every instance's shared-memory limit (with the device the kernels run on current).
cudaError_t set_smem_limits() {
  for (int qt : {4, 5})
    for (uint32_t n : {16u, 32u, 64u}) {
      const cudaError_t e =
          cudaFuncSetAttribute(mma_fn_for(qt, n), cudaFuncAttributeMaxDynamicSharedMemorySize, smem_limit(qt, n));
      if (e != cudaSuccess) return e;
    }
  return cudaSuccess;
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library links only the
// runtime); null when the driver has none.
EncodeTiled encode_tiled() {
  static const EncodeTiled fn = []() -> EncodeTiled {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// One call of the pre-pass and the kernel on `stream`: tiles of equal height (rows / SMs rounded
// up, at most 128, at least 16 or all rows), the tensor map over W with one tile's super-block
// column as its box.
int mma_launch(const char* call, int sm_count, int qt, uint64_t w, uint64_t x, uint64_t ldx, uint64_t y,
               uint64_t ldy, uint32_t rows, uint32_t k, uint32_t batch, uint32_t flags, void* scratch,
               unsigned* err, cudaStream_t stream) {
  const uint32_t npad = npad_for(batch);
  const uint32_t blk = qt == 4 ? kBlockBytes<4> : kBlockBytes<5>;
  const uint32_t nb = k / kQK;
  const uint32_t sms = static_cast<uint32_t>(std::max(sm_count, 1));
  const uint32_t per_cta = (rows + sms * kTileM - 1) / (sms * kTileM);  // tiles per CTA
  uint32_t tm = (rows + sms * per_cta - 1) / (sms * per_cta);
  tm = std::min<uint32_t>(kTileM, std::max<uint32_t>(tm, std::min<uint32_t>(rows, 16)));
  const uint32_t ntiles = (rows + tm - 1) / tm;

  CUtensorMap map;
  const uint64_t dims[2] = {uint64_t(nb) * blk, rows};
  const uint64_t strides[1] = {uint64_t(nb) * blk};
  const uint32_t box[2] = {blk, tm};
  const int erc = encode_tensor_map(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, reinterpret_cast<const void*>(w),
                                    dims, strides, box, call);
  if (erc) return erc;

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const unsigned nattr = (flags & KQ_FLAG_NO_PDL) ? 0 : 1;
  {  // pre-pass: X -> B-operand layout
    const uint32_t total = nb * 32 * npad;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min<uint32_t>((total + 255) / 256, sms * 4));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = nattr;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, xperm_kernel, reinterpret_cast<uint4*>(scratch),
                                             reinterpret_cast<const float*>(x), ldx, nb, batch, npad);
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx", "X pre-pass");
  }
  MmaArgs args;
  args.xp = static_cast<const uint8_t*>(scratch);
  args.y = reinterpret_cast<float*>(y);
  args.err = err;
  args.ldy = ldy;
  args.rows = rows;
  args.nb = nb;
  args.batch = batch;
  args.flags = flags;
  args.tm = tm;
  args.ntiles = ntiles;
  args.nq = (tm + 3) / 4;
  args.raw_stride = raw_stride_for(qt, tm);
  const uint32_t grid = std::min<uint32_t>(sms, ntiles);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_for(qt, npad, args.raw_stride);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  void* params[] = {&map, &args};
  const cudaError_t e = cudaLaunchKernelExC(&cfg, mma_fn_for(qt, npad), params);
  if (e != cudaSuccess)
    return cuda_fail(e, "cudaLaunchKernelExC", "tensor-core matvec grid " + std::to_string(grid));
  return KQ_OK;
}

}  // namespace

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                      const char* call) {
  const EncodeTiled encode = encode_tiled();
  if (!encode) return fail(KQ_E_UNSUPPORTED, call, "the driver has no cuTensorMapEncodeTiled");
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  const CUresult r = encode(map, type, rank, const_cast<void*>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(KQ_E_INVALID, call, "cuTensorMapEncodeTiled refused W (error " + std::to_string(int(r)) + ")");
  return KQ_OK;
}

int mma_prepare(kq_ctx* ctx) {
  const cudaError_t e = set_smem_limits();
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute", "tensor-core matvec kernel");
  return KQ_OK;
}

uint64_t mma_scratch_bytes(uint32_t k, uint32_t batch) {
  return uint64_t(k / kQK) * 32 * npad_for(batch) * 16;
}

bool mma_supports(const kq_matvec_desc& d) {
  return (d.type == KQ_TYPE_Q4_K || d.type == KQ_TYPE_Q5_K) && d.batch >= 1 && d.batch <= 64 &&
         d.prologue == KQ_PROLOGUE_NONE && d.epilogue == KQ_EPILOGUE_NONE;
}

int mma_matvec(kq_ctx* ctx, const kq_matvec_desc& d, uint64_t ldx, uint64_t ldy,
               cudaStream_t stream) {
  const uint64_t need = mma_scratch_bytes(d.k, d.batch);
  if (need > ctx->scratch_bytes)
    return fail(KQ_E_UNSUPPORTED, "kq_matvec",
                "the tensor-core path needs " + std::to_string(need) + " bytes of scratch for k " +
                    std::to_string(d.k) + ", batch " + std::to_string(d.batch) + "; the context has " +
                    std::to_string(ctx->scratch_bytes));
  return mma_launch("kq_matvec", ctx->sm_count, d.type == KQ_TYPE_Q4_K ? 4 : 5, d.w, d.x, ldx, d.y, ldy,
                    d.rows, d.k, d.batch, d.flags, ctx->scratch, ctx->err, stream);
}

}  // namespace kq

// ------------------------------------------------------------------------------------------------
// kq_matvec_q4k_noalloc: the tensor-core Q4_K matvec for callers that cannot allocate device
// memory -- code that runs while a CUDA graph is being captured, inside a server whose memory
// pool has already reserved the GPU, or anywhere a cudaMalloc would stall a latency budget. It
// needs no kq_ctx (whose creation allocates scratch): the X scratch lives in the file-scope
// array below, which every GPU that loads this library holds until the process exits.

namespace {

// 1 MiB: the f16 B operand of one call, k * (batch rounded up to 16, 32 or 64) * 2 bytes.
constexpr uint64_t kNoAllocScratchBytes = 1ull << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
struct NoAllocDevice {
  bool ready = false;
  int sm_count = 0;
  void* scratch = nullptr;  // device address of g_noalloc_scratch on this GPU
  unsigned* err = nullptr;  // device address of the library's error word on this GPU
};
NoAllocDevice g_noalloc_devices[kMaxDevices];
std::mutex g_noalloc_mutex;

// Set-up, once per device, with that device current: attributes, the kernels' shared-memory
// limit, and the device addresses of the static scratch and of the error word. The names of
// those arrays are host-side stand-ins in host code, so only cudaGetSymbolAddress gives an
// address a kernel may use.
int noalloc_setup(int dev, NoAllocDevice** out) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  NoAllocDevice& d = g_noalloc_devices[dev];
  if (!d.ready) {
    int major = 0, minor = 0;
    cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess) return kq::cuda_fail(e, "cudaDeviceGetAttribute", "compute capability");
    if (major != 10 || minor != 0)
      return kq::fail(KQ_E_UNSUPPORTED, "kq_matvec_q4k_noalloc", "this library is built for sm_100a (B200)");
    e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return kq::cuda_fail(e, "cudaDeviceGetAttribute");
    e = kq::set_smem_limits();
    if (e != cudaSuccess) return kq::cuda_fail(e, "cudaFuncSetAttribute", "tensor-core matvec kernel");
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return kq::cuda_fail(e, "cudaGetSymbolAddress", "static scratch");
    d.scratch = p;
    const int rc = kq::error_word_address(&d.err);
    if (rc) return rc;
    d.ready = true;
  }
  *out = &d;
  return KQ_OK;
}

}  // namespace

extern "C" int kq_matvec_q4k_noalloc(uint64_t y, uint64_t w, uint64_t x, uint32_t rows, uint32_t k,
                                     uint32_t batch, kq_stream stream) {
  const char* call = "kq_matvec_q4k_noalloc";
  if (rows == 0 || k == 0 || k % kq::kQK != 0)
    return kq::fail(KQ_E_INVALID, call, "rows must be > 0 and k a positive multiple of 256");
  if (batch < 1 || batch > 64) return kq::fail(KQ_E_INVALID, call, "batch must be 1..64");
  if (!w || !x || !y) return kq::fail(KQ_E_INVALID, call, "null pointer");
  if (w % 16 || x % 16 || y % 4)
    return kq::fail(KQ_E_INVALID, call, "w and x must be 16-byte aligned, y 4-byte aligned");
  const uint64_t need = kq::mma_scratch_bytes(k, batch);
  if (need > kNoAllocScratchBytes)
    return kq::fail(KQ_E_INVALID, call,
                    "k " + std::to_string(k) + " at batch " + std::to_string(batch) + " needs " +
                        std::to_string(need) + " bytes of scratch, past the static " +
                        std::to_string(kNoAllocScratchBytes) +
                        " (k <= 32768 up to batch 16, 16384 up to 32, 8192 up to 64)");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return kq::cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return kq::fail(KQ_E_UNSUPPORTED, call, "device ordinal past 63");
  NoAllocDevice* d = nullptr;
  const int rc = noalloc_setup(dev, &d);
  if (rc) return rc;
  return kq::mma_launch(call, d->sm_count, 4, w, x, k, y, rows, rows, k, batch, 0, d->scratch, d->err,
                        static_cast<cudaStream_t>(stream));
}
