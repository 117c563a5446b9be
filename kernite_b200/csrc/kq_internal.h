// kq_internal.h -- what the library's translation units share (host side).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "kq.h"

struct kq_ctx {
  int device = 0;
  int sm_count = 0;
  int max_smem = 0;       // opt-in dynamic shared memory per block
  unsigned* err = nullptr;  // the device error word (a file-scope __device__ variable)
};

namespace kq {

// Records the thread's last error as "<call>: <detail>" and returns `code`.
int fail(int code, const char* call, const std::string& detail);
// Records a CUDA error as "<call>: <NAME> (<n>): <meaning>[: detail]" and returns its number.
int cuda_fail(cudaError_t e, const char* call, const std::string& detail = std::string());
// Makes the ctx's device current if it is not.
int enter(const kq_ctx* ctx);

int matvec_prepare(kq_ctx* ctx);
int matvec(kq_ctx* ctx, const kq_matvec_desc& d, cudaStream_t stream);

int aux_prepare(kq_ctx* ctx);
int dequant(kq_ctx* ctx, int type, uint64_t out, uint64_t w, uint64_t nblocks, cudaStream_t s);
int fill(kq_ctx* ctx, int type, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
         cudaStream_t s);

uint64_t stream_key(uint64_t seed, uint64_t tensor);

}  // namespace kq
