// kq_aux.cu -- verification and synthetic-data kernels: the bit-exact dequantiser and the
// counter-based block generator.
//
// The dequantiser computes every weight in the canonical order of the CPU decode,
//   Q4_K: w = (f32(d) * f32(sc)) * f32(q) - f32(dmin) * f32(m)
//   Q6_K: w = (f32(d) * f32(scale)) * f32(q - 32)
//   Q5_K: as Q4_K, q = nibble | (fifth bit << 4), the fifth bit of element 32g + l in bit g of
//         qh[l]
// with __fmul_rn / __fsub_rn so that nothing contracts into an FMA, the discipline of
// fxeqxmulfx/kernite's scalar references (examples/matmul/src/reference.rs:1-10).
//
// The generator reproduces the oracle's kqo_fill_q4k / q5k / q6k byte for byte: splitmix64
// output number i of the tensor's keyed stream, integer work plus one binary32 multiply, one
// add and a round-to-nearest-even narrowing to fp16 per scale.
//
// Q2_K, Q3_K and Q8_0 (units of 256 weights; a Q8_0 unit is eight 34-byte blocks) decode through
// the __host__ __device__ functions of kq_decode.cuh.
#include <cuda_runtime.h>

#include "kq_decode.cuh"
#include "kq_device.cuh"
#include "kq_internal.h"

namespace kq {
namespace {

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t splitmix_at(uint64_t key, uint64_t i) {
  return mix64(key + (i + 1) * 0x9e3779b97f4a7c15ull);
}

__device__ __forceinline__ uint32_t uniform_fp16(uint64_t word, float lo, float span) {
  const float u = __uint2float_rn(static_cast<uint32_t>(word >> 40)) * 0x1p-24f;  // exact
  const float v = __fadd_rn(lo, __fmul_rn(u, span));
  return __half_as_ushort(__float2half_rn(v));
}

__global__ void fill_q4k_kernel(uint8_t* w, uint64_t b0, uint64_t n, uint64_t key) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t b = b0 + i;
    uint64_t words[18];
#pragma unroll
    for (int t = 0; t < 18; ++t) words[t] = splitmix_at(key, 20 * b + t);
    const uint32_t d = uniform_fp16(splitmix_at(key, 20 * b + 18), 0x1p-10f, 15.0f * 0x1p-10f);
    const uint32_t m = uniform_fp16(splitmix_at(key, 20 * b + 19), 0x1p-10f, 15.0f * 0x1p-10f);
    words[0] = (words[0] & ~0xffffffffull) | d | (uint64_t(m) << 16);
    uint4* out = reinterpret_cast<uint4*>(w + i * kQ4KBytes);  // 144 = 9 x 16, w 16-aligned
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      out[t] = make_uint4(static_cast<uint32_t>(words[2 * t]), static_cast<uint32_t>(words[2 * t] >> 32),
                          static_cast<uint32_t>(words[2 * t + 1]),
                          static_cast<uint32_t>(words[2 * t + 1] >> 32));
    }
  }
}

__global__ void fill_q6k_kernel(uint8_t* w, uint64_t b0, uint64_t n, uint64_t key) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t b = b0 + i;
    uint16_t* out = reinterpret_cast<uint16_t*>(w + i * kQ6KBytes);  // 2-byte aligned
    // bytes 0..191: ql, qh (24 words)
#pragma unroll 4
    for (int t = 0; t < 24; ++t) {
      const uint64_t v = splitmix_at(key, 28 * b + t);
#pragma unroll
      for (int j = 0; j < 4; ++j) out[4 * t + j] = static_cast<uint16_t>(v >> (16 * j));
    }
    // bytes 192..207: scales, each raw byte mapped to (raw & 127) - 64
#pragma unroll
    for (int t = 24; t < 26; ++t) {
      const uint64_t v = splitmix_at(key, 28 * b + t);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t lo = static_cast<uint32_t>((v >> (16 * j)) & 0xff);
        const uint32_t hi = static_cast<uint32_t>((v >> (16 * j + 8)) & 0xff);
        const uint32_t s0 = static_cast<uint8_t>(static_cast<int>(lo & 127) - 64);
        const uint32_t s1 = static_cast<uint8_t>(static_cast<int>(hi & 127) - 64);
        out[96 + 4 * (t - 24) + j] = static_cast<uint16_t>(s0 | (s1 << 8));
      }
    }
    out[104] = static_cast<uint16_t>(
        uniform_fp16(splitmix_at(key, 28 * b + 27), 0x1p-12f, 15.0f * 0x1p-12f));
  }
}

__global__ void fill_q5k_kernel(uint8_t* w, uint64_t b0, uint64_t n, uint64_t key) {
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < n;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t b = b0 + i;
    uint64_t words[22];
#pragma unroll
    for (int t = 0; t < 22; ++t) words[t] = splitmix_at(key, 24 * b + t);
    const uint32_t d = uniform_fp16(splitmix_at(key, 24 * b + 22), 0x1p-11f, 15.0f * 0x1p-11f);
    const uint32_t m = uniform_fp16(splitmix_at(key, 24 * b + 23), 0x1p-11f, 15.0f * 0x1p-11f);
    words[0] = (words[0] & ~0xffffffffull) | d | (uint64_t(m) << 16);
    uint4* out = reinterpret_cast<uint4*>(w + i * kQ5KBytes);  // 176 = 11 x 16, w 16-aligned
#pragma unroll
    for (int t = 0; t < 11; ++t) {
      out[t] = make_uint4(static_cast<uint32_t>(words[2 * t]), static_cast<uint32_t>(words[2 * t] >> 32),
                          static_cast<uint32_t>(words[2 * t + 1]),
                          static_cast<uint32_t>(words[2 * t + 1] >> 32));
    }
  }
}

// One thread per weight.
__global__ void dequant_q4k_kernel(float* out, const uint8_t* w, uint64_t nblocks) {
  const uint64_t total = nblocks * kQK;
  for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
       t += uint64_t(gridDim.x) * blockDim.x) {
    const uint8_t* blk = w + (t / kQK) * kQ4KBytes;
    const uint32_t e = static_cast<uint32_t>(t % kQK);
    const uint32_t j = e / 32, c = e / 64, l = e % 32;
    const uint8_t* s = blk + 4;
    uint32_t sc, m;
    if (j < 4) {
      sc = s[j] & 63u;
      m = s[j + 4] & 63u;
    } else {
      sc = (s[j + 4] & 15u) | ((s[j - 4] >> 6) << 4);
      m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const uint32_t byte = blk[16 + 32 * c + l];
    const uint32_t q = (j & 1) ? (byte >> 4) : (byte & 15u);
    const float d = h2f(blk[0] | (blk[1] << 8));
    const float dmin = h2f(blk[2] | (blk[3] << 8));
    const float ds = __fmul_rn(d, static_cast<float>(sc));
    const float dm = __fmul_rn(dmin, static_cast<float>(m));
    out[t] = __fsub_rn(__fmul_rn(ds, static_cast<float>(q)), dm);
  }
}

__global__ void dequant_q6k_kernel(float* out, const uint8_t* w, uint64_t nblocks) {
  const uint64_t total = nblocks * kQK;
  for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
       t += uint64_t(gridDim.x) * blockDim.x) {
    const uint8_t* blk = w + (t / kQK) * kQ6KBytes;
    const uint32_t e = static_cast<uint32_t>(t % kQK);
    const uint32_t h = e / 128, g = (e % 128) / 32, l = e % 32;
    const uint32_t L0 = blk[64 * h + l], L1 = blk[64 * h + l + 32], H = blk[128 + 32 * h + l];
    uint32_t q;
    switch (g) {
      case 0: q = (L0 & 15u) | ((H & 3u) << 4); break;
      case 1: q = (L1 & 15u) | (((H >> 2) & 3u) << 4); break;
      case 2: q = (L0 >> 4) | (((H >> 4) & 3u) << 4); break;
      default: q = (L1 >> 4) | (((H >> 6) & 3u) << 4); break;
    }
    const int scale = static_cast<int8_t>(blk[192 + e / 16]);
    const float d = h2f(blk[208] | (blk[209] << 8));
    const float ds = __fmul_rn(d, static_cast<float>(scale));
    out[t] = __fmul_rn(ds, static_cast<float>(static_cast<int>(q) - 32));
  }
}

__global__ void dequant_q5k_kernel(float* out, const uint8_t* w, uint64_t nblocks) {
  const uint64_t total = nblocks * kQK;
  for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
       t += uint64_t(gridDim.x) * blockDim.x) {
    const uint8_t* blk = w + (t / kQK) * kQ5KBytes;
    const uint32_t e = static_cast<uint32_t>(t % kQK);
    const uint32_t j = e / 32, c = e / 64, l = e % 32;
    const uint8_t* s = blk + 4;
    uint32_t sc, m;
    if (j < 4) {
      sc = s[j] & 63u;
      m = s[j + 4] & 63u;
    } else {
      sc = (s[j + 4] & 15u) | ((s[j - 4] >> 6) << 4);
      m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const uint32_t byte = blk[48 + 32 * c + l];
    const uint32_t q = ((j & 1) ? (byte >> 4) : (byte & 15u)) | (((blk[16 + l] >> j) & 1u) << 4);
    const float d = h2f(blk[0] | (blk[1] << 8));
    const float dmin = h2f(blk[2] | (blk[3] << 8));
    const float ds = __fmul_rn(d, static_cast<float>(sc));
    const float dm = __fmul_rn(dmin, static_cast<float>(m));
    out[t] = __fsub_rn(__fmul_rn(ds, static_cast<float>(q)), dm);
  }
}

// Q2_K / Q3_K / Q8_0: one thread per weight
template <int T>
__global__ void dequant_unit_kernel(float* out, const uint8_t* w, uint64_t nunits) {
  constexpr uint32_t kUnit = T == 2 ? dec::kQ2KBytes : T == 3 ? dec::kQ3KBytes : dec::kQ8Unit;
  const uint64_t total = nunits * kQK;
  for (uint64_t t = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; t < total;
       t += uint64_t(gridDim.x) * blockDim.x)
    out[t] = dec::weight(T, w + (t / kQK) * kUnit, static_cast<uint32_t>(t % kQK));
}

uint32_t grid_for(uint64_t work, uint32_t threads, int sm_count) {
  const uint64_t want = (work + threads - 1) / threads;
  const uint64_t cap = uint64_t(sm_count) * 16;
  return static_cast<uint32_t>(want < cap ? (want ? want : 1) : cap);
}

}  // namespace

uint64_t stream_key(uint64_t seed, uint64_t tensor) {
  return mix64(mix64(seed * 0xd1342543de82ef95ull + tensor) ^ 0x632be59bd9b4e019ull);
}

__global__ void wait_counter_kernel(unsigned* err, const unsigned long long* cnt,
                                    const unsigned long long* epoch, uint64_t mul, uint64_t add) {
  wait_count(err, cnt, epoch, mul, add);
}

// *epoch += 1 once the kernels before it on the stream are done (a chain of the previous step may
// still read the old value as its CTAs start), launched with programmatic dependent launch so
// that it waits on the device instead of breaking the chains' overlap with a launch gap.
__global__ void epoch_advance_kernel(unsigned long long* epoch) {
  pdl_wait();
  *epoch += 1ull;
  __threadfence();
  pdl_launch_dependents();
}

int aux_prepare(kq_ctx*) { return KQ_OK; }

int epoch_advance(kq_ctx*, uint64_t epoch, cudaStream_t s) {
  if (!epoch || epoch % 8)
    return fail(KQ_E_INVALID, "kq_epoch_advance", "epoch must be a non-null 8-byte aligned address");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, epoch_advance_kernel, reinterpret_cast<unsigned long long*>(epoch));
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx", "kq_epoch_advance");
  return KQ_OK;
}

int wait_counter(kq_ctx* ctx, uint64_t counter, uint64_t epoch, uint64_t mul, uint64_t add,
                 cudaStream_t s) {
  const char* call = "kq_wait_counter";
  if (!counter || !epoch || counter % 8 || epoch % 8)
    return fail(KQ_E_INVALID, call, "counter and epoch must be non-null and 8-byte aligned");
  wait_counter_kernel<<<1, 1, 0, s>>>(ctx->err, reinterpret_cast<const unsigned long long*>(counter),
                                      reinterpret_cast<const unsigned long long*>(epoch), mul, add);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel", call);
  return KQ_OK;
}

namespace {
const char* type_call(const char* verb, int type) {
  static const char* const names[2][9] = {
      {"", "", "kq_dequant_q2k", "kq_dequant_q3k", "kq_dequant_q4k", "kq_dequant_q5k",
       "kq_dequant_q6k", "", "kq_dequant_q8_0"},
      {"", "", "", "", "kq_fill_q4k", "kq_fill_q5k", "kq_fill_q6k", "", ""}};
  return (type >= 2 && type <= 8) ? names[verb[0] == 'f'][type] : "kq_dequant";
}
}  // namespace

int dequant(kq_ctx* ctx, int type, uint64_t out, uint64_t w, uint64_t nblocks, cudaStream_t s) {
  const char* call = type_call("dequant", type);
  if (nblocks == 0) return KQ_OK;
  if (!out || !w) return fail(KQ_E_INVALID, call, "null pointer");
  if (out % 4 || w % 2) return fail(KQ_E_INVALID, call, "out must be 4-byte and w 2-byte aligned");
  const uint32_t threads = 256;
  const uint32_t grid = grid_for(nblocks * kQK, threads, ctx->sm_count);
  if (type == 2)
    dequant_unit_kernel<2><<<grid, threads, 0, s>>>(reinterpret_cast<float*>(out),
                                                    reinterpret_cast<const uint8_t*>(w), nblocks);
  else if (type == 3)
    dequant_unit_kernel<3><<<grid, threads, 0, s>>>(reinterpret_cast<float*>(out),
                                                    reinterpret_cast<const uint8_t*>(w), nblocks);
  else if (type == 8)
    dequant_unit_kernel<8><<<grid, threads, 0, s>>>(reinterpret_cast<float*>(out),
                                                    reinterpret_cast<const uint8_t*>(w), nblocks);
  else if (type == 4)
    dequant_q4k_kernel<<<grid, threads, 0, s>>>(reinterpret_cast<float*>(out),
                                                 reinterpret_cast<const uint8_t*>(w), nblocks);
  else if (type == 5)
    dequant_q5k_kernel<<<grid, threads, 0, s>>>(reinterpret_cast<float*>(out),
                                                 reinterpret_cast<const uint8_t*>(w), nblocks);
  else
    dequant_q6k_kernel<<<grid, threads, 0, s>>>(reinterpret_cast<float*>(out),
                                                 reinterpret_cast<const uint8_t*>(w), nblocks);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel", call);
  return KQ_OK;
}

int fill(kq_ctx* ctx, int type, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
         cudaStream_t s) {
  const char* call = type_call("fill", type);
  if (nblocks == 0) return KQ_OK;
  if (!w) return fail(KQ_E_INVALID, call, "null pointer");
  if ((type == 4 || type == 5) && w % 16) return fail(KQ_E_INVALID, call, "w must be 16-byte aligned");
  if (type == 6 && w % 2) return fail(KQ_E_INVALID, call, "w must be 2-byte aligned");
  const uint32_t threads = 128;
  const uint32_t grid = grid_for(nblocks, threads, ctx->sm_count);
  if (type == 4)
    fill_q4k_kernel<<<grid, threads, 0, s>>>(reinterpret_cast<uint8_t*>(w), block0, nblocks, key);
  else if (type == 5)
    fill_q5k_kernel<<<grid, threads, 0, s>>>(reinterpret_cast<uint8_t*>(w), block0, nblocks, key);
  else
    fill_q6k_kernel<<<grid, threads, 0, s>>>(reinterpret_cast<uint8_t*>(w), block0, nblocks, key);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel", call);
  return KQ_OK;
}

}  // namespace kq
