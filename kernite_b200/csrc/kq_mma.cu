// kq_mma.cu -- the Q4_K matvec / small-batch matmul on the 5th-generation tensor cores.
//
// Y[b, r] = sum_k W[r, k] X[b, k] as D = A * B^T per tile of 128 weight rows:
//   A (128 rows x 256 K per super-block, f16) is written by the dequantising threads straight
//     into tensor memory: thread = weight row = TMEM lane, so there is no shared-memory A tile;
//   B (N = batch padded to 16/32/64, K-major f16) is X, converted once per call by a small
//     pre-pass into the exact shared-memory layout of the B operand (kept in the context's
//     scratch buffer), and fetched per super-block with one bulk copy;
//   D (128 lanes x N f32 columns) accumulates in tensor memory over the whole row; four epilogue
//     warps read it back with tcgen05.ld and write Y.
// One persistent CTA per SM owns a contiguous range of rows. Warp roles:
//   0       tensor-memory owner and MMA issuer: 16 tcgen05.mma (K = 16) per super-block, then
//           tcgen05.commit to free the A and B slots, and at the end of a tile to publish D;
//   1       B loader: one cp.async.bulk of the super-block's B tile into a ring of slots;
//   2..9    dequantisers: TMEM lane quadrant w % 4, half (w - 2) / 4 of each super-block. Each
//           thread streams its own row with 16-byte cp.async copies into a private ring of
//           shared memory several super-blocks deep (weights never pass through the TMA unit,
//           whose per-request cost would bound a copy per row);
//   10..13  epilogue.
// The dequantiser keeps the canonical weight w = d*sc*q - dmin*m to one f16 rounding: q comes
// out of the 1024 + q magic exactly (one LOP3 per two weights and one HSUB2), then one HFMA2
// computes q * (d*sc) - dmin*m. The K order inside each 8-weight group follows the byte lanes
// (l, l+2, l+1, l+3 of the low nibbles, then the same of the high nibbles); the pre-pass
// permutes X alike, so the contraction is unchanged.
//
// Every wait is bounded (kq_device.cuh): a wait that gives up records an error word, and all
// roles then run to the end without waiting, so the CTA frees its tensor memory and exits.
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

constexpr int kTileM = 128;
constexpr int kASlots = 3;            // A slots in TMEM, one super-block (128 columns) each
constexpr int kDQ = 4;                // depth of each dequantiser's private copy ring (blocks)
constexpr int kDqThreads = 256;
constexpr int kDqBytes = 80;          // bytes a dequantiser copies per block: header + 64 B of qs
constexpr uint32_t kDqRing = kDQ * kDqThreads * kDqBytes;
constexpr int kThreads = 14 * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kDCol = kASlots * 128;  // first D column

struct MmaArgs {
  const uint8_t* W;
  const uint8_t* xp;  // X in B-operand layout: per block 32 k-groups x NPAD rows x 16 B
  float* y;
  unsigned* err;
  uint64_t ldy;
  uint32_t rows, nb, batch, flags;
};

template <int NPAD>
struct MmaGeo {
  static constexpr int kBSlots = NPAD <= 32 ? 8 : 4;
  static constexpr uint32_t kBSlotBytes = 32 * NPAD * 16;
  static constexpr uint32_t kSmem = kDqRing + kBSlots * kBSlotBytes + 1024 + 1024;
};

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

template <int NPAD>
__global__ void __launch_bounds__(kThreads, 1) mma_q4k_kernel(const MmaArgs a) {
  using G = MmaGeo<NPAD>;
  constexpr int BS = G::kBSlots;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* dq = smem;                  // [kDQ][256 threads][80 B]
  uint8_t* bring = smem + kDqRing;     // [BS][B tile]
  uint64_t* bars = reinterpret_cast<uint64_t*>(bring + BS * G::kBSlotBytes);
  uint64_t* a_full = bars;                 // [3]  dequantisers -> MMA
  uint64_t* a_empty = a_full + kASlots;    // [3]  MMA commit -> dequantisers
  uint64_t* b_full = a_empty + kASlots;    // [BS] B loader (tx bytes) -> MMA
  uint64_t* b_empty = b_full + BS;         // [BS] MMA commit -> B loader
  uint64_t* d_full = b_empty + BS;         // [2]  MMA commit -> epilogue
  uint64_t* d_empty = d_full + 2;          // [2]  epilogue -> MMA
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(d_empty + 2);
  int* failed = reinterpret_cast<int*>(tmem_holder + 1);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t RB = a.nb * kQ4KBytes;
  const uint32_t r_begin = static_cast<uint32_t>(uint64_t(a.rows) * blockIdx.x / gridDim.x);
  const uint32_t r_end = static_cast<uint32_t>(uint64_t(a.rows) * (blockIdx.x + 1) / gridDim.x);
  const uint32_t ntiles = (r_end - r_begin + kTileM - 1) / kTileM;

  if (threadIdx.x == 0) {
    *failed = 0;
    for (int i = 0; i < kASlots; ++i) {
      mbar_init(smem_u32(&a_full[i]), 8);
      mbar_init(smem_u32(&a_empty[i]), 1);
    }
    for (int i = 0; i < BS; ++i) {
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
    const uint32_t idesc = idesc_f16_f32(kTileM, NPAD);
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
            const uint32_t bslot = smem_u32(bring) + bs * G::kBSlotBytes;
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
    // ---------------------------------------------------------------- B loader
    pdl_wait();  // the B tiles come from the pre-pass just before this kernel
    const uint32_t tile_bytes = G::kBSlotBytes;
    uint32_t g = 0;
    for (uint32_t T = 0; T < ntiles; ++T) {
      for (uint32_t kb = 0; kb < a.nb; ++kb, ++g) {
        const uint32_t bs = g % BS;
        if (g >= BS) warp_wait(smem_u32(&b_empty[bs]), ((g / BS) - 1) & 1, failed, a.err, kErrWaitEmpty);
        if (lane == 0) {
          const uint32_t full = smem_u32(&b_full[bs]);
          mbar_arrive_expect_tx(full, tile_bytes);
          bulk_g2s(smem_u32(bring) + bs * tile_bytes, a.xp + uint64_t(kb) * tile_bytes, tile_bytes,
                   full);
        }
        __syncwarp();
      }
    }
  } else if (warp < 10) {
    // ---------------------------------------------------------------- dequantisers
    const uint32_t quad = warp & 3;              // TMEM lanes 32*quad .. +31
    const uint32_t part = (warp - 2) >> 2;       // chunks 2*part, 2*part+1 of each block
    const uint32_t t = (warp - 2) * 32 + lane;   // private ring column
    const uint32_t lrow = quad * 32 + lane;      // row within the tile
    const uint32_t my_ring = smem_u32(dq) + t * kDqBytes;
    const uint32_t lane_base = tmem + ((quad * 32) << 16) + part * 64;
    const uint32_t total = ntiles * a.nb;
    if (!(a.flags & KQ_FLAG_WEIGHTS_STATIC)) pdl_wait();  // W may be the previous kernel's output
    // issue position (tile, block) of the next copy
    uint32_t iT = 0, ikb = 0, issued = 0;
    auto issue = [&]() {
      if (issued < total) {
        const uint32_t row = r_begin + iT * kTileM + lrow;
        if (row < r_end) {
          const uint8_t* src = a.W + uint64_t(row) * RB + uint64_t(ikb) * kQ4KBytes;
          const uint32_t dst = my_ring + (issued % kDQ) * (kDqThreads * kDqBytes);
          cp_async16(dst, src);                    // d, dmin, scales
          const uint8_t* qs = src + 16 + 64 * part;
#pragma unroll
          for (int i = 0; i < 4; ++i) cp_async16(dst + 16 + 16 * i, qs + 16 * i);
        }
        if (++ikb == a.nb) {
          ikb = 0;
          ++iT;
        }
      }
      cp_async_commit();  // possibly empty: keeps one group per block
      ++issued;
    };
#pragma unroll 1
    for (int i = 0; i < kDQ - 1; ++i) issue();
    const __half2 magic = __half2half2(__ushort_as_half(0x6400));  // 1024
    uint32_t g = 0;
    for (uint32_t T = 0; T < ntiles; ++T) {
      const bool valid = lrow < r_end - (r_begin + T * kTileM);
      for (uint32_t kb = 0; kb < a.nb; ++kb, ++g) {
        issue();
        cp_async_wait<kDQ - 1>();  // this thread's copy of block g has landed
        const uint32_t as = g % kASlots;
        if (g >= kASlots)
          warp_wait(smem_u32(&a_empty[as]), ((g / kASlots) - 1) & 1, failed, a.err, kErrWaitEmpty);
        tc_fence_after();
        const uint32_t src = my_ring + (g % kDQ) * (kDqThreads * kDqBytes);
        const uint4 hdr = valid ? lds_v4(src) : make_uint4(0, 0, 0, 0);
        const float d = h2f(hdr.x & 0xffffu), dmin = h2f(hdr.x >> 16);
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
          for (int hh = 0; hh < 2; ++hh) {  // 16 bytes of qs -> 16 TMEM columns
            const uint4 q = valid ? lds_v4(src + 16 + 32 * cc + 16 * hh) : make_uint4(0, 0, 0, 0);
            const uint32_t words[4] = {q.x, q.y, q.z, q.w};
            uint32_t v[16];
#pragma unroll
            for (int ww = 0; ww < 4; ++ww) {
              const uint32_t w = words[ww], w8 = w >> 8;
              const __half2 a0 = __hsub2(bits_h2((w & 0x000F000Fu) | 0x64006400u), magic);
              const __half2 a1 = __hsub2(bits_h2((w8 & 0x000F000Fu) | 0x64006400u), magic);
              const __half2 b0 = __hsub2(bits_h2((w & 0x00F000F0u) | 0x64006400u), magic);
              const __half2 b1 = __hsub2(bits_h2((w8 & 0x00F000F0u) | 0x64006400u), magic);
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
        if (lane == 0) mbar_arrive(smem_u32(&a_full[as]));
      }
    }
    cp_async_wait<0>();
  } else {
    // ---------------------------------------------------------------- epilogue
    pdl_wait();
    const uint32_t quad = warp & 3;
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
      const uint32_t row = r_begin + T * kTileM + quad * 32 + lane;
      if (ok && row < r_end) {
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

template <int NPAD>
const void* mma_fn() {
  return reinterpret_cast<const void*>(&mma_q4k_kernel<NPAD>);
}

uint32_t npad_for(uint32_t batch) { return batch <= 16 ? 16 : batch <= 32 ? 32 : 64; }

int smem_for(uint32_t npad) {
  return npad == 16 ? MmaGeo<16>::kSmem : npad == 32 ? MmaGeo<32>::kSmem : MmaGeo<64>::kSmem;
}

}  // namespace

int mma_prepare(kq_ctx* ctx) {
  for (uint32_t n : {16u, 32u, 64u}) {
    const void* fn = n == 16 ? mma_fn<16>() : n == 32 ? mma_fn<32>() : mma_fn<64>();
    const cudaError_t e =
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_for(n));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute", "tensor-core matvec kernel");
  }
  return KQ_OK;
}

uint64_t mma_scratch_bytes(uint32_t k, uint32_t batch) {
  return uint64_t(k / kQK) * 32 * npad_for(batch) * 16;
}

bool mma_supports(const kq_matvec_desc& d) {
  return d.type == KQ_TYPE_Q4_K && d.batch >= 1 && d.batch <= 64 &&
         d.prologue == KQ_PROLOGUE_NONE && d.epilogue == KQ_EPILOGUE_NONE;
}

int mma_matvec(kq_ctx* ctx, const kq_matvec_desc& d, uint64_t ldx, uint64_t ldy,
               cudaStream_t stream) {
  const uint32_t npad = npad_for(d.batch);
  const uint32_t nb = d.k / kQK;
  const uint64_t need = mma_scratch_bytes(d.k, d.batch);
  if (need > ctx->scratch_bytes)
    return fail(KQ_E_UNSUPPORTED, "kq_matvec",
                "the tensor-core path needs " + std::to_string(need) + " bytes of scratch for k " +
                    std::to_string(d.k) + ", batch " + std::to_string(d.batch) + "; the context has " +
                    std::to_string(ctx->scratch_bytes));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const unsigned nattr = (d.flags & KQ_FLAG_NO_PDL) ? 0 : 1;

  // pre-pass: X -> B-operand layout
  {
    const uint32_t total = nb * 32 * npad;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min<uint32_t>((total + 255) / 256, ctx->sm_count * 4));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = nattr;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, xperm_kernel, reinterpret_cast<uint4*>(ctx->scratch),
                                             reinterpret_cast<const float*>(d.x), ldx, nb, d.batch, npad);
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx", "X pre-pass");
  }
  MmaArgs args;
  args.W = reinterpret_cast<const uint8_t*>(d.w);
  args.xp = static_cast<const uint8_t*>(ctx->scratch);
  args.y = reinterpret_cast<float*>(d.y);
  args.err = ctx->err;
  args.ldy = ldy;
  args.rows = d.rows;
  args.nb = nb;
  args.batch = d.batch;
  args.flags = d.flags;
  const void* fn = npad == 16 ? mma_fn<16>() : npad == 32 ? mma_fn<32>() : mma_fn<64>();
  const uint32_t grid = std::min<uint32_t>(ctx->sm_count, d.rows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_for(npad);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  void* params[] = {&args};
  const cudaError_t e = cudaLaunchKernelExC(&cfg, fn, params);
  if (e != cudaSuccess)
    return cuda_fail(e, "cudaLaunchKernelExC", "tensor-core matvec grid " + std::to_string(grid));
  return KQ_OK;
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
    for (uint32_t n : {16u, 32u, 64u}) {
      const void* fn = n == 16 ? kq::mma_fn<16>() : n == 32 ? kq::mma_fn<32>() : kq::mma_fn<64>();
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kq::smem_for(n));
      if (e != cudaSuccess) return kq::cuda_fail(e, "cudaFuncSetAttribute", "tensor-core matvec kernel");
    }
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
  int rc = noalloc_setup(dev, &d);
  if (rc) return rc;

  const uint32_t npad = kq::npad_for(batch);
  const uint32_t nb = k / kq::kQK;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    const uint32_t total = nb * 32 * npad;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min<uint32_t>((total + 255) / 256, d->sm_count * 4));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kq::xperm_kernel, reinterpret_cast<uint4*>(d->scratch),
                           reinterpret_cast<const float*>(x), uint64_t(k), nb, batch, npad);
    if (e != cudaSuccess) return kq::cuda_fail(e, "cudaLaunchKernelEx", "X pre-pass");
  }
  kq::MmaArgs args;
  args.W = reinterpret_cast<const uint8_t*>(w);
  args.xp = static_cast<const uint8_t*>(d->scratch);
  args.y = reinterpret_cast<float*>(y);
  args.err = d->err;
  args.ldy = rows;
  args.rows = rows;
  args.nb = nb;
  args.batch = batch;
  args.flags = 0;
  const void* fn = npad == 16 ? kq::mma_fn<16>() : npad == 32 ? kq::mma_fn<32>() : kq::mma_fn<64>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min<uint32_t>(d->sm_count, rows));
  cfg.blockDim = dim3(kq::kThreads);
  cfg.dynamicSmemBytes = kq::smem_for(npad);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* params[] = {&args};
  e = cudaLaunchKernelExC(&cfg, fn, params);
  if (e != cudaSuccess) return kq::cuda_fail(e, "cudaLaunchKernelExC", "tensor-core matvec");
  return KQ_OK;
}
