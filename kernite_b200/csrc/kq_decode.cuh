// kq_decode.cuh -- one weight of a Q2_K / Q3_K / Q8_0 unit of 256 weights, as __host__
// __device__ functions. The device's verification kernel (kq_aux.cu) calls them; the same source
// compiled for the host is checked against the CPU oracle and the gguf-py fixtures on a machine
// without a GPU.
//
// Decode order is the canonical one of the CPU oracle, every float operation rounded to binary32
// on its own (no contraction; __fmul_rn / __fsub_rn on the device, and a host build compiled with
// -ffp-contract=off):
//   Q2_K: w = (f32(d) * f32(sc)) * f32(q) - f32(dmin) * f32(m)     (16-weight sub-blocks)
//   Q3_K: w = (f32(d) * f32(scale - 32)) * f32(q)                  (16-weight sub-blocks)
//   Q8_0: w = f32(q) * f32(d)                                        (32-weight blocks)
// following gguf-py/gguf/quants.py (Q2_K, Q3_K, Q8_0 .dequantize_blocks, gguf-py 0.19.0).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#define KQ_HD __host__ __device__ __forceinline__

namespace kq {
namespace dec {

constexpr uint32_t kQ2KBytes = 84;   // u8 scales[16], u8 qs[64], fp16 d, fp16 dmin
constexpr uint32_t kQ3KBytes = 110;  // u8 hmask[32], u8 qs[64], u8 scales[12], fp16 d
constexpr uint32_t kQ8Block = 34;    // fp16 d, i8 qs[32]
constexpr uint32_t kQ8Unit = 272;    // eight Q8_0 blocks = 256 weights

KQ_HD float mul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}

KQ_HD float sub_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  return a - b;
#endif
}

// binary16 bits at p (little endian) widened exactly
KQ_HD float f16_at(const uint8_t* p) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}

// bytes per 256 weights, 0 for a type this header does not decode
KQ_HD uint32_t unit_bytes(int type) {
  return type == 2 ? kQ2KBytes : type == 3 ? kQ3KBytes : type == 8 ? kQ8Unit : 0u;
}

// Q2_K weight e (0..255): bits 2s..2s+1 of qs[32h + l] for e = 128h + 32s + l; sub-block e / 16
// has scale = low nibble and min = high nibble of scales[e / 16]
KQ_HD float q2k_weight(const uint8_t* blk, uint32_t e) {
  const uint32_t h = e >> 7, s = (e >> 5) & 3u, l = e & 31u;
  const uint32_t q = (blk[16 + 32 * h + l] >> (2 * s)) & 3u;
  const uint32_t sm = blk[e >> 4];
  const float dl = mul_rn(f16_at(blk + 80), static_cast<float>(sm & 15u));
  const float ml = mul_rn(f16_at(blk + 82), static_cast<float>(sm >> 4));
  return sub_rn(mul_rn(dl, static_cast<float>(q)), ml);
}

// Q3_K scale i (0..15) minus 32: low 4 bits from nibble i / 8 of byte i % 8, high 2 bits from
// bits 2 (i / 4) of byte 8 + i % 4
KQ_HD int q3k_scale(const uint8_t* s, uint32_t i) {
  const uint32_t lo = (s[i % 8] >> (4 * (i / 8))) & 15u;
  const uint32_t hi = (s[8 + i % 4] >> (2 * (i / 4))) & 3u;
  return static_cast<int>(lo | (hi << 4)) - 32;
}

// Q3_K weight e = 128h + 32s + l: low bits 2s..2s+1 of qs[32h + l], and 4 subtracted unless bit
// 4h + s of hmask[l] is set
KQ_HD float q3k_weight(const uint8_t* blk, uint32_t e) {
  const uint32_t h = e >> 7, s = (e >> 5) & 3u, l = e & 31u;
  const int low = (blk[32 + 32 * h + l] >> (2 * s)) & 3;
  const int high = (blk[l] >> (4 * h + s)) & 1;
  const int q = low - (high ? 0 : 4);
  const float dl = mul_rn(f16_at(blk + 108), static_cast<float>(q3k_scale(blk + 96, e >> 4)));
  return mul_rn(dl, static_cast<float>(q));
}

// Q8_0 weight e of a unit of eight 34-byte blocks
KQ_HD float q8_0_weight(const uint8_t* unit, uint32_t e) {
  const uint8_t* blk = unit + (e >> 5) * kQ8Block;
  const int q = static_cast<int8_t>(blk[2 + (e & 31u)]);
  return mul_rn(static_cast<float>(q), f16_at(blk));
}

KQ_HD float weight(int type, const uint8_t* unit, uint32_t e) {
  return type == 2 ? q2k_weight(unit, e) : type == 3 ? q3k_weight(unit, e) : q8_0_weight(unit, e);
}

}  // namespace dec
}  // namespace kq
