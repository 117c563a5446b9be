// kq_internal.h -- what the library's translation units share (host side).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "kq.h"

struct kq_ctx {
  int device = 0;
  int sm_count = 0;
  int max_smem = 0;       // opt-in dynamic shared memory per block
  unsigned* err = nullptr;  // the ctx's device error word (its own allocation)
  // Scratch the tensor-core path converts X into (allocated once, at creation).
  void* scratch = nullptr;
  uint64_t scratch_bytes = 0;
  // Device staging for kq_matvec_host's x and y (grown on demand).
  void* stage = nullptr;
  uint64_t stage_bytes = 0;
};

namespace kq {

// Scratch bytes a context allocates: the B operand of a k = 32768, batch = 64 tensor-core call.
constexpr uint64_t kCtxScratchBytes = 4ull << 20;

// Records the thread's last error as "<call>: <detail>" and returns `code`.
int fail(int code, const char* call, const std::string& detail);
// Records a CUDA error as "<call>: <NAME> (<n>): <meaning>[: detail]" and returns its number.
int cuda_fail(cudaError_t e, const char* call, const std::string& detail = std::string());
// The current device's address of the library's device error word.
int error_word_address(unsigned** out);
// An entry point's hold on the ctx's device: enter() makes it current if it is not, and the
// destructor makes the caller's device current again, so no entry point leaves the thread on
// another GPU than the one it found.
class DeviceScope {
 public:
  DeviceScope() = default;
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
  ~DeviceScope();
  int enter(const kq_ctx* ctx);

 private:
  int restore_ = -1;
};

int matvec_prepare(kq_ctx* ctx);
int mma_prepare(kq_ctx* ctx);
bool mma_supports(const kq_matvec_desc& d);
int mma_matvec(kq_ctx* ctx, const kq_matvec_desc& d, uint64_t ldx, uint64_t ldy,
               cudaStream_t stream);
uint64_t mma_scratch_bytes(uint32_t k, uint32_t batch);
// cuTensorMapEncodeTiled (through the runtime's driver entry point; the library links only the
// runtime) of a rank-`rank` tiled map over `base`: dims and box innermost first, strides in bytes
// of dims 1.., no interleave, no swizzle, L2 promotion 256 B, zero fill. KQ_OK, or KQ_E_UNSUPPORTED
// when the driver has no such call, KQ_E_INVALID when it refuses the map.
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType type, uint32_t rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                      const char* call);
int matvec(kq_ctx* ctx, const kq_matvec_desc& d, cudaStream_t stream,
           const kq_push_desc* push = nullptr);
// The argument checks every matvec entry point makes before a launch (KQ_E_INVALID on failure).
int check_desc(const kq_matvec_desc& d, const char* call);

int warpmma_prepare(kq_ctx* ctx);
bool warpmma_supports(const kq_matvec_desc& d);
int warpmma_matvec(kq_ctx* ctx, const kq_matvec_desc& d, uint64_t ldx, uint64_t ldy,
                   cudaStream_t stream);
int tagged_unpack(kq_ctx* ctx, uint64_t dst, uint64_t src, uint64_t n, uint64_t epoch, uint64_t mul,
                  uint64_t add, cudaStream_t stream);
int warpmma_plan_launch(kq_ctx* ctx, const kq_matvec_desc& d, kq_launch& out);
int warpmma_push(kq_ctx* ctx, const kq_matvec_desc& d, const kq_push_desc& push, uint64_t ldx,
                 uint64_t ldy, cudaStream_t stream);
int warpmma_chain(kq_ctx* ctx, const kq_chain_job* jobs, uint32_t njobs, uint64_t epoch,
                  cudaStream_t stream);
int epoch_advance(kq_ctx* ctx, uint64_t epoch, cudaStream_t stream);

int aux_prepare(kq_ctx* ctx);
int types_prepare(kq_ctx* ctx);
int types_matvec(kq_ctx* ctx, const kq_matvec_desc& d, cudaStream_t stream);
int wait_counter(kq_ctx* ctx, uint64_t counter, uint64_t epoch, uint64_t mul, uint64_t add,
                 cudaStream_t s);
int dequant(kq_ctx* ctx, int type, uint64_t out, uint64_t w, uint64_t nblocks, cudaStream_t s);
int fill(kq_ctx* ctx, int type, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
         cudaStream_t s);

uint64_t stream_key(uint64_t seed, uint64_t tensor);

int rope_append(kq_ctx* ctx, uint64_t qkv, uint64_t q_out, uint64_t k_cache, uint64_t v_cache,
                uint32_t nh, uint32_t nkv, uint32_t d, uint32_t pos, double base, cudaStream_t s);
uint64_t attention_workspace_bytes(kq_ctx* ctx, uint32_t nh, uint32_t nkv, uint32_t d, uint32_t len);
int attention_decode(kq_ctx* ctx, uint64_t out, uint64_t q, uint64_t k_cache, uint64_t v_cache,
                     uint32_t nh, uint32_t nkv, uint32_t d, uint32_t len, uint64_t workspace,
                     uint64_t workspace_bytes, cudaStream_t s);

}  // namespace kq
