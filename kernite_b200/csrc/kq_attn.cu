// kq_attn.cu -- the activation side of a Llama decode step around the matvecs: rotary position
// embedding of the step's query and key heads with the key/value cache append, and grouped-query
// attention of the step's queries over the cache.
//
// The functional model is fxeqxmulfx/kernite's microgpt attention (examples/microgpt/src/gpu.rs:
// 130-230): per head, logits q.k scaled, their maximum, exponentials and sum, the weights, and
// the values they weigh, summed. Here the keys and values come from a cache of earlier steps
// (f16, one row of n_kv * head_dim per position), several query heads share a key/value head
// (GQA), the positions are rotated (RoPE, GGML's "norm" mode: adjacent element pairs), and one
// step's attention is split over positions across CTAs (partial maxima, sums and weighted values
// per split, then one combine), because a decode step has one query per head and the cache is
// long.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "kq_device.cuh"
#include "kq_internal.h"

namespace kq {
namespace {

constexpr uint32_t kAttnThreads = 128;
constexpr uint32_t kMaxGroup = 16;    // query heads per key/value head
constexpr uint32_t kMaxHeadDim = 256;
constexpr uint32_t kMaxChunk = 1024;  // positions a CTA of the attention takes
constexpr float kLog2e = 1.4426950408889634f;

// One element pair (2i, 2i+1) of a head rotated by pos * base^(-2i/d), in f64 (the angle of a
// late position is large; its rounding to f32 would cost the rotation's accuracy).
__device__ __forceinline__ void rotate(float x0, float x1, uint32_t i, uint32_t d, uint32_t pos,
                                       double log2_base, double& y0, double& y1) {
  const double inv_freq = exp2(-(2.0 * i / d) * log2_base);
  double s, c;
  sincos(static_cast<double>(pos) * inv_freq, &s, &c);
  y0 = static_cast<double>(x0) * c - static_cast<double>(x1) * s;
  y1 = static_cast<double>(x0) * s + static_cast<double>(x1) * c;
}

// qkv: the step's q (nh heads), k and v (nkv heads each) of head_dim d, back to back (a q|k|v
// matvec's output). q_out <- q rotated; k rotated and v go to row pos of the caches as f16.
__global__ void rope_append_kernel(const float* __restrict__ qkv, float* __restrict__ q_out,
                                   __half* __restrict__ kc, __half* __restrict__ vc, uint32_t nh,
                                   uint32_t nkv, uint32_t d, uint32_t pos, double log2_base) {
  const uint32_t half_d = d / 2;
  const uint32_t nq = nh * half_d, nk = nkv * half_d, nv = nkv * d;
  const uint64_t row = uint64_t(pos) * nkv * d;
  for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < nq + nk + nv; t += gridDim.x * blockDim.x) {
    if (t < nq + nk) {
      const bool is_q = t < nq;
      const uint32_t u = is_q ? t : t - nq;
      const uint32_t head = u / half_d, i = u % half_d;
      const float* src = qkv + (is_q ? 0 : nh * d) + head * d + 2 * i;
      double y0, y1;
      rotate(src[0], src[1], i, d, pos, log2_base, y0, y1);
      if (is_q) {
        q_out[head * d + 2 * i] = static_cast<float>(y0);
        q_out[head * d + 2 * i + 1] = static_cast<float>(y1);
      } else {
        kc[row + head * d + 2 * i] = __double2half(y0);
        kc[row + head * d + 2 * i + 1] = __double2half(y1);
      }
    } else {
      const uint32_t u = t - nq - nk;
      vc[row + u] = __float2half_rn(qkv[(nh + nkv) * d + u]);
    }
  }
}

// Split s of the attention of key/value head g: positions [s * chunk, min(len, (s + 1) * chunk)),
// for the group of query heads g * grp .. g * grp + grp - 1. Writes per head its maximum logit
// (log2 units), the sum of 2^(logit - max) and the weighted sum of the values (unnormalised).
__global__ void __launch_bounds__(kAttnThreads) attention_split_kernel(
    const float* __restrict__ q, const __half* __restrict__ kc, const __half* __restrict__ vc,
    float* __restrict__ part, uint32_t nh, uint32_t nkv, uint32_t d, uint32_t len, uint32_t chunk,
    float scale_log2) {
  const uint32_t g = blockIdx.x, s = blockIdx.y;
  const uint32_t grp = nh / nkv;
  const uint32_t p0 = s * chunk, p1 = min(len, p0 + chunk);
  const uint32_t n = p1 > p0 ? p1 - p0 : 0;
  __shared__ float sq[kMaxGroup * kMaxHeadDim];  // the group's queries, scaled to log2 units
  __shared__ float sw[kMaxGroup * kMaxChunk / 8]; // logits, then weights: [head][position]
  __shared__ float sm[kMaxGroup], sl[kMaxGroup];
  for (uint32_t i = threadIdx.x; i < grp * d; i += blockDim.x)
    sq[i] = q[(g * grp) * d + i] * scale_log2;
  __syncthreads();
  const uint64_t stride = uint64_t(nkv) * d;  // halves between positions
  // logits: a thread per position, its key row read 8 halves at a time
  for (uint32_t p = threadIdx.x; p < n; p += blockDim.x) {
    const __half* kr = kc + uint64_t(p0 + p) * stride + g * d;
    float acc[kMaxGroup];
#pragma unroll
    for (uint32_t h = 0; h < kMaxGroup; ++h) acc[h] = 0.f;
    for (uint32_t j = 0; j < d; j += 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(kr + j);
      const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
      float kv[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h2[e]);
        kv[2 * e] = f.x;
        kv[2 * e + 1] = f.y;
      }
#pragma unroll
      for (uint32_t h = 0; h < kMaxGroup; ++h) {
        if (h < grp) {
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[h] = fmaf(sq[h * d + j + e], kv[e], acc[h]);
        }
      }
    }
#pragma unroll
    for (uint32_t h = 0; h < kMaxGroup; ++h)
      if (h < grp) sw[h * chunk + p] = acc[h];
  }
  __syncthreads();
  // per head: the maximum, the weights 2^(l - max) and their sum (a warp per head)
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t h = warp; h < grp; h += blockDim.x / 32) {
    float m = -INFINITY;
    for (uint32_t p = lane; p < n; p += 32) m = fmaxf(m, sw[h * chunk + p]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (uint32_t p = lane; p < n; p += 32) {
      const float w = n ? exp2f(sw[h * chunk + p] - m) : 0.f;
      sw[h * chunk + p] = w;
      l += w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      sm[h] = m;
      sl[h] = l;
    }
  }
  __syncthreads();
  // the weighted values: a thread per element of the head, over the positions in order
  float* out = part + (uint64_t(s) * nh + g * grp) * (d + 2);
  for (uint32_t j = threadIdx.x; j < d; j += blockDim.x) {
    float acc[kMaxGroup];
#pragma unroll
    for (uint32_t h = 0; h < kMaxGroup; ++h) acc[h] = 0.f;
    const __half* vr = vc + uint64_t(p0) * stride + g * d + j;
    for (uint32_t p = 0; p < n; ++p) {
      const float v = __half2float(vr[uint64_t(p) * stride]);
#pragma unroll
      for (uint32_t h = 0; h < kMaxGroup; ++h)
        if (h < grp) acc[h] = fmaf(sw[h * chunk + p], v, acc[h]);
    }
#pragma unroll
    for (uint32_t h = 0; h < kMaxGroup; ++h)
      if (h < grp) out[h * (d + 2) + 2 + j] = acc[h];
  }
  if (threadIdx.x < grp) {
    out[threadIdx.x * (d + 2)] = sm[threadIdx.x];
    out[threadIdx.x * (d + 2) + 1] = sl[threadIdx.x];
  }
}

// out[h][j] = sum_s 2^(m_s - M) acc_s[j] / sum_s 2^(m_s - M) l_s over the splits, M = max_s m_s
// (splits with no positions carry m = -inf and add nothing).
__global__ void attention_combine_kernel(const float* __restrict__ part, float* __restrict__ out,
                                         uint32_t nh, uint32_t d, uint32_t nsplit) {
  for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < nh * d; t += gridDim.x * blockDim.x) {
    const uint32_t h = t / d, j = t % d;
    float M = -INFINITY;
    for (uint32_t s = 0; s < nsplit; ++s) M = fmaxf(M, part[(uint64_t(s) * nh + h) * (d + 2)]);
    float num = 0.f, den = 0.f;
    for (uint32_t s = 0; s < nsplit; ++s) {
      const float* ps = part + (uint64_t(s) * nh + h) * (d + 2);
      if (ps[0] == -INFINITY) continue;
      const float c = exp2f(ps[0] - M);
      num = fmaf(c, ps[2 + j], num);
      den = fmaf(c, ps[1], den);
    }
    out[t] = num / den;
  }
}

// The split of a cache of len positions over CTAs: at least 64 positions each, at most kMaxChunk,
// about two CTAs per SM over all key/value heads.
void attention_split(uint32_t len, uint32_t nkv, uint32_t grp, int sm_count, uint32_t& chunk,
                     uint32_t& nsplit) {
  const uint32_t cap = std::min<uint32_t>(kMaxChunk, (kMaxGroup * kMaxChunk / 8) / grp);
  const uint32_t want = std::max<uint32_t>(1, (2u * sm_count + nkv - 1) / nkv);
  chunk = std::max<uint32_t>(64, (len + want - 1) / want);
  chunk = std::min<uint32_t>(cap, (chunk + 31) / 32 * 32);
  nsplit = (len + chunk - 1) / chunk;
}

}  // namespace

uint64_t attention_workspace_bytes(kq_ctx* ctx, uint32_t nh, uint32_t nkv, uint32_t d, uint32_t len) {
  uint32_t chunk, nsplit;
  attention_split(len, nkv, nkv ? nh / nkv : 1, ctx->sm_count, chunk, nsplit);
  return uint64_t(nsplit) * nh * (d + 2) * 4;
}

int rope_append(kq_ctx* ctx, uint64_t qkv, uint64_t q_out, uint64_t k_cache, uint64_t v_cache,
                uint32_t nh, uint32_t nkv, uint32_t d, uint32_t pos, double base, cudaStream_t s) {
  const char* call = "kq_rope_append";
  if (!qkv || !q_out || !k_cache || !v_cache) return fail(KQ_E_INVALID, call, "null pointer");
  if (nh == 0 || nkv == 0 || nh % nkv || d == 0 || d % 8 || d > kMaxHeadDim)
    return fail(KQ_E_INVALID, call, "n_heads must be a positive multiple of n_kv and head_dim a "
                                    "multiple of 8 up to 256");
  if (!(base > 1.0)) return fail(KQ_E_INVALID, call, "the rotary base must be above 1");
  if (qkv % 4 || q_out % 4 || k_cache % 16 || v_cache % 16)
    return fail(KQ_E_INVALID, call, "qkv, q_out 4-byte aligned; the caches 16-byte aligned");
  const uint32_t work = nh * d / 2 + nkv * d / 2 + nkv * d;
  const uint32_t threads = 256;
  const uint32_t grid = std::min<uint32_t>((work + threads - 1) / threads, ctx->sm_count * 4);
  rope_append_kernel<<<grid, threads, 0, s>>>(
      reinterpret_cast<const float*>(qkv), reinterpret_cast<float*>(q_out),
      reinterpret_cast<__half*>(k_cache), reinterpret_cast<__half*>(v_cache), nh, nkv, d, pos,
      std::log2(base));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel", call);
  return KQ_OK;
}

int attention_decode(kq_ctx* ctx, uint64_t out, uint64_t q, uint64_t k_cache, uint64_t v_cache,
                     uint32_t nh, uint32_t nkv, uint32_t d, uint32_t len, uint64_t workspace,
                     uint64_t workspace_bytes, cudaStream_t s) {
  const char* call = "kq_attention_decode";
  if (!out || !q || !k_cache || !v_cache || !workspace) return fail(KQ_E_INVALID, call, "null pointer");
  if (nh == 0 || nkv == 0 || nh % nkv || nh / nkv > kMaxGroup || d == 0 || d % 8 || d > kMaxHeadDim)
    return fail(KQ_E_INVALID, call, "n_heads must be 1..16 times n_kv and head_dim a multiple of 8 "
                                    "up to 256");
  if (len == 0) return fail(KQ_E_INVALID, call, "the cache holds no position");
  if (out % 4 || q % 4 || k_cache % 16 || v_cache % 16 || workspace % 16)
    return fail(KQ_E_INVALID, call, "out, q 4-byte aligned; caches and workspace 16-byte aligned");
  const uint32_t grp = nh / nkv;
  uint32_t chunk, nsplit;
  attention_split(len, nkv, grp, ctx->sm_count, chunk, nsplit);
  const uint64_t need = uint64_t(nsplit) * nh * (d + 2) * 4;
  if (workspace_bytes < need)
    return fail(KQ_E_INVALID, call, "workspace of " + std::to_string(workspace_bytes) + " bytes; " +
                                        std::to_string(need) + " needed (kq_attention_workspace)");
  const float scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(d))) * kLog2e;
  attention_split_kernel<<<dim3(nkv, nsplit), kAttnThreads, 0, s>>>(
      reinterpret_cast<const float*>(q), reinterpret_cast<const __half*>(k_cache),
      reinterpret_cast<const __half*>(v_cache), reinterpret_cast<float*>(workspace), nh, nkv, d, len,
      chunk, scale_log2);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel", "attention splits");
  const uint32_t total = nh * d;
  attention_combine_kernel<<<std::min<uint32_t>((total + 255) / 256, ctx->sm_count), 256, 0, s>>>(
      reinterpret_cast<const float*>(workspace), reinterpret_cast<float*>(out), nh, d, nsplit);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel", "attention combine");
  return KQ_OK;
}

}  // namespace kq
