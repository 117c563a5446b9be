// Host build of the device decoder for Q2_K / Q3_K / Q8_0 (kq_decode.cuh), so the
// CPU tests check the same source the verification kernels run against the oracle and the gguf-py
// fixtures. Test infrastructure: compiled by tests/test_decode_host.py into a temporary
// directory, never part of libkq.so. Built with -ffp-contract=off, as the oracle is.
#include "kq_decode.cuh"

extern "C" int kqh_dequant(int type, const uint8_t* units, uint64_t n, float* out) {
  const uint32_t ub = kq::dec::unit_bytes(type);
  if (!ub) return -1;
  for (uint64_t u = 0; u < n; ++u)
    for (uint32_t e = 0; e < 256; ++e) out[u * 256 + e] = kq::dec::weight(type, units + u * ub, e);
  return 0;
}
