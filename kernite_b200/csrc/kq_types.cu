// kq_types.cu -- the batch-1 matvec y = W.x for the k-quant types beyond Q4_K/Q5_K/Q6_K: Q2_K
// (84-byte blocks), Q3_K (110-byte blocks) and Q8_0 (34-byte blocks of 32, counted in units of
// eight: 272 bytes per 256 weights). A CUDA-core kernel: every CTA keeps x in shared memory; a
// warp takes a row at a time and walks its 256-weight units, each lane the 8 consecutive weights
// 8l..8l+7 of a unit (so the lanes read x conflict-free and a unit's bytes in one pass), with the
// products of a lane's weights of one sub-block summed before the sub-block's scale is applied:
//   Q2_K  sum_i (d sc q_i - dmin m) x_i = d sc sum_i q_i x_i - dmin m sum_i x_i
//   Q3_K  sum_i d (scale - 32) q_i x_i = d (scale - 32) sum_i q_i x_i
//   Q8_0  sum_i d q_i x_i              = d sum_i q_i x_i
// then the row's lanes are summed by shuffles. The block layouts and field packings are GGML's
// (the CPU restatement in oracle/kq_oracle.c; the device decoder in kq_decode.cuh); the pattern --
// one output row per group of lanes, an FMA chain over k -- is the matvec of fxeqxmulfx/kernite's
// examples/microgpt/src/gpu.rs:100-131.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "kq_decode.cuh"
#include "kq_device.cuh"
#include "kq_internal.h"

namespace kq {
namespace {

constexpr uint32_t kTypeThreads = 256;  // 8 warps
// units of a row in flight per warp: eight for Q2_K and Q3_K (measured on B200, 14336 x 4096:
// 32.6 -> 23.6 us and 44.6 -> 32.5 us against two), two for Q8_0 (eight: 29.7 -> 31.6 us)
template <int T>
constexpr int kUnroll = T == 8 ? 2 : 8;

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
  return *reinterpret_cast<const unsigned short*>(p);
}

// 8 bytes from a 2-byte aligned address as two words (little endian)
__device__ __forceinline__ uint2 ld8_a2(const uint8_t* p) {
  const uint32_t a = ld_u16(p), b = ld_u16(p + 2), c = ld_u16(p + 4), d = ld_u16(p + 6);
  return make_uint2(a | (b << 16), c | (d << 16));
}

__device__ __forceinline__ float f16_bits(uint32_t h) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// Lane l's part of one 256-weight unit at b: its weights 8l..8l+7 against xs[0..7].
template <int T>
__device__ __forceinline__ float unit_part(const uint8_t* __restrict__ b, const float* xs, uint32_t l) {
  const float4 x0 = *reinterpret_cast<const float4*>(xs);
  const float4 x1 = *reinterpret_cast<const float4*>(xs + 4);
  const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  if constexpr (T == 8) {
    // block l / 4 of the unit, its quants 8 (l % 4) .. + 7
    const uint8_t* blk = b + (l >> 2) * dec::kQ8Block;
    const uint2 q = ld8_a2(blk + 2 + 8 * (l & 3));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = static_cast<int8_t>(((i < 4 ? q.x : q.y) >> (8 * (i & 3))) & 0xffu);
      s = fmaf(static_cast<float>(v), xv[i], s);
    }
    return f16_bits(ld_u16(blk)) * s;
  } else if constexpr (T == 2) {
    // element 8l + i = 128 h + 32 s + (8 (l % 4) + i): crumb s of qs[32 h + 8 (l % 4) + i]
    const uint32_t h = l >> 4, s2 = 2 * ((l >> 2) & 3);
    // (units are 84 bytes: 4-byte aligned, so two word loads)
    const uint32_t* qw = reinterpret_cast<const uint32_t*>(b + 16 + 32 * h + 8 * (l & 3));
    const uint2 q = make_uint2(qw[0], qw[1]);
    float sq = 0.f, sx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t v = ((i < 4 ? q.x : q.y) >> (8 * (i & 3) + s2)) & 3u;
      sq = fmaf(static_cast<float>(v), xv[i], sq);
      sx += xv[i];
    }
    const uint32_t sm = b[l >> 1];  // sub-block (8l) / 16: scale low nibble, min high nibble
    const uint32_t dd = *reinterpret_cast<const uint32_t*>(b + 80);
    return f16_bits(dd & 0xffffu) * static_cast<float>(sm & 15u) * sq -
           f16_bits(dd >> 16) * static_cast<float>(sm >> 4) * sx;
  } else {
    // Q3_K: low bits from qs[32 + 32 h + ...], the high bit from hmask[8 (l % 4) + i] bit 4h + s
    const uint32_t h = l >> 4, s = (l >> 2) & 3;
    const uint2 q = ld8_a2(b + 32 + 32 * h + 8 * (l & 3));
    const uint2 m = ld8_a2(b + 8 * (l & 3));
    const uint32_t hb = 4 * h + s;
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t sh = 8 * (i & 3);
      const int low = static_cast<int>(((i < 4 ? q.x : q.y) >> (sh + 2 * s)) & 3u);
      const int hi = static_cast<int>(((i < 4 ? m.x : m.y) >> (sh + hb)) & 1u);
      sq = fmaf(static_cast<float>(low - (hi ? 0 : 4)), xv[i], sq);
    }
    const int sc = dec::q3k_scale(b + 96, l >> 1);
    return f16_bits(ld_u16(b + 108)) * static_cast<float>(sc) * sq;
  }
}

// y[r] = sum_k W[r,k] x[k] for the rows of W (rows x nu units), batch 1. x goes to shared memory
// once per CTA; then warps take rows, kUnroll units per step.
template <int T>
__global__ void __launch_bounds__(kTypeThreads) unit_matvec_kernel(const uint8_t* __restrict__ W,
                                                                    const float* __restrict__ x,
                                                                    float* __restrict__ y,
                                                                    uint32_t rows, uint32_t nu) {
  constexpr uint32_t kUnit = T == 2 ? dec::kQ2KBytes : T == 3 ? dec::kQ3KBytes : dec::kQ8Unit;
  extern __shared__ __align__(16) float xs[];
  const uint32_t K = nu * kQK;
  for (uint32_t i = threadIdx.x; i < K / 4; i += blockDim.x)
    reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(x)[i];
  __syncthreads();
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t nwarps = gridDim.x * (blockDim.x / 32);
  for (uint32_t r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); r < rows; r += nwarps) {
    const uint8_t* row = W + uint64_t(r) * nu * kUnit;
    // kUnroll units a step, their partial sums apart, so that every load of the step is in
    // flight at once (one memory latency per kUnroll units instead of per two)
    constexpr int U = kUnroll<T>;
    float acc[U];
#pragma unroll
    for (int i = 0; i < U; ++i) acc[i] = 0.f;
    uint32_t u = 0;
    for (; u + U <= nu; u += U) {
#pragma unroll
      for (int i = 0; i < U; ++i)
        acc[i] += unit_part<T>(row + uint64_t(u + i) * kUnit, xs + (u + i) * kQK + 8 * lane, lane);
    }
    for (; u < nu; ++u) acc[0] += unit_part<T>(row + uint64_t(u) * kUnit, xs + u * kQK + 8 * lane, lane);
    float v = 0.f;
#pragma unroll
    for (int i = 0; i < U; ++i) v += acc[i];
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) y[r] = v;
  }
}

const void* unit_fn(int t) {
  return t == 2   ? reinterpret_cast<const void*>(&unit_matvec_kernel<2>)
         : t == 3 ? reinterpret_cast<const void*>(&unit_matvec_kernel<3>)
                  : reinterpret_cast<const void*>(&unit_matvec_kernel<8>);
}

}  // namespace

int types_prepare(kq_ctx* ctx) {
  for (int t : {2, 3, 8}) {
    const cudaError_t e =
        cudaFuncSetAttribute(unit_fn(t), cudaFuncAttributeMaxDynamicSharedMemorySize, ctx->max_smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute", "Q2_K/Q3_K/Q8_0 matvec kernel");
  }
  return KQ_OK;
}

int types_matvec(kq_ctx* ctx, const kq_matvec_desc& d, cudaStream_t stream) {
  const char* call = "kq_matvec";
  const int t = d.type == KQ_TYPE_Q2_K ? 2 : d.type == KQ_TYPE_Q3_K ? 3 : 8;
  if (d.rows == 0 || d.k == 0 || d.k % kQK)
    return fail(KQ_E_INVALID, call, "rows must be > 0 and k a positive multiple of 256");
  if (d.batch != 1 || d.prologue != KQ_PROLOGUE_NONE || d.epilogue != KQ_EPILOGUE_NONE ||
      (d.flags & (KQ_FLAG_TENSOR_CORES | KQ_FLAG_WARP_MMA)))
    return fail(KQ_E_UNSUPPORTED, call,
                "Q2_K, Q3_K and Q8_0 are served at batch 1 without prologue or epilogue, on the "
                "CUDA cores");
  if (d.ldx > d.k || d.ldy > d.rows) return fail(KQ_E_INVALID, call, "batch 1 has no strides");
  if (!d.w || !d.x || !d.y) return fail(KQ_E_INVALID, call, "null pointer");
  if (d.w % 16 || d.x % 16 || d.y % 4)
    return fail(KQ_E_INVALID, call, "w and x must be 16-byte aligned, y 4-byte aligned");
  const uint64_t smem = uint64_t(d.k) * 4;
  if (smem > uint64_t(ctx->max_smem))
    return fail(KQ_E_UNSUPPORTED, call, "k " + std::to_string(d.k) + " does not fit in shared memory");
  const uint32_t per_sm = std::max<uint32_t>(1, std::min<uint32_t>(4, uint32_t(ctx->max_smem / std::max<uint64_t>(smem, 1))));
  // a warp per row at a time: enough CTAs for every row, at most per_sm resident per SM
  const uint32_t grid = std::min<uint32_t>(ctx->sm_count * per_sm, (d.rows + 7) / 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTypeThreads);
  cfg.dynamicSmemBytes = static_cast<uint32_t>(smem);
  cfg.stream = stream;
  const uint8_t* W = reinterpret_cast<const uint8_t*>(d.w);
  const float* x = reinterpret_cast<const float*>(d.x);
  float* y = reinterpret_cast<float*>(d.y);
  uint32_t rows = d.rows, nu = d.k / kQK;
  void* params[] = {&W, &x, &y, &rows, &nu};
  const cudaError_t e = cudaLaunchKernelExC(&cfg, unit_fn(t), params);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelExC", "Q2_K/Q3_K/Q8_0 matvec");
  return KQ_OK;
}

}  // namespace kq
