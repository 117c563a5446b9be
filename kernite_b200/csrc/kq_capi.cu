// kq_capi.cu -- the C ABI (include/kq.h): contexts, errors, argument checks, dispatch.
//
// Errors keep the shape of fxeqxmulfx/kernite's kernite_cuda::Error (crates/cuda/src/lib.rs:
// 290-324): the failing call, then "NAME (number): meaning" for a CUDA error, then any detail.
// The message is per thread, as a Rust Result is per call.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>

#include "kq_device.cuh"
#include "kq_internal.h"

// The device error word of kq_matvec_q4k_noalloc, which has no context to hold one: a file-scope
// device variable (zero at load; every GPU that loads the library has its own copy), whose
// address host code takes with cudaGetSymbolAddress per device. A kq_ctx has its own word.
__device__ unsigned g_kq_error_word;

namespace kq {

namespace {
thread_local std::string t_last_error;
}

int fail(int code, const char* call, const std::string& detail) {
  t_last_error = std::string(call) + ": " + detail;
  return code;
}

int cuda_fail(cudaError_t e, const char* call, const std::string& detail) {
  std::string msg = std::string(call) + ": " + cudaGetErrorName(e) + " (" +
                    std::to_string(static_cast<int>(e)) + "): " + cudaGetErrorString(e);
  if (!detail.empty()) msg += ": " + detail;
  t_last_error = msg;
  cudaGetLastError();  // a launch-configuration error is not sticky; do not leave it pending
  return static_cast<int>(e);
}

int error_word_address(unsigned** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_kq_error_word);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress", "device error word");
  *out = static_cast<unsigned*>(p);
  return KQ_OK;
}

int DeviceScope::enter(const kq_ctx* ctx) {
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (cur != ctx->device) {
    e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    restore_ = cur;
  }
  return KQ_OK;
}

DeviceScope::~DeviceScope() {
  if (restore_ >= 0) cudaSetDevice(restore_);
}

}  // namespace kq

using kq::cuda_fail;
using kq::fail;

extern "C" {

int kq_ctx_create(int device, kq_ctx** out) {
  if (!out) return fail(KQ_E_INVALID, "kq_ctx_create", "null out pointer");
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= count)
    return fail(KQ_E_INVALID, "kq_ctx_create",
                "no GPU " + std::to_string(device) + " (the program sees " + std::to_string(count) +
                    ")");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  int major = 0, minor = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute", "compute capability");
  if (major != 10 || minor != 0)
    return fail(KQ_E_UNSUPPORTED, "kq_ctx_create",
                "this library is built for sm_100a (B200); GPU " + std::to_string(device) +
                    " is sm_" + std::to_string(major) + std::to_string(minor));
  kq_ctx* ctx = new kq_ctx();
  ctx->device = device;
  e = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&ctx->max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (e != cudaSuccess) {
    delete ctx;
    return cuda_fail(e, "cudaDeviceGetAttribute", "SM count / shared memory per block");
  }
  // Leave room for the kernels' static shared memory.
  ctx->max_smem -= 2048;
  // The ctx's own error word (in its own 256 bytes, zeroed here and by kq_device_error only), so
  // that no other ctx on the GPU can clear an error this one's launches recorded.
  e = cudaMalloc(reinterpret_cast<void**>(&ctx->err), 256);
  if (e == cudaSuccess) e = cudaMemset(ctx->err, 0, 256);
  if (e != cudaSuccess) {
    if (ctx->err) cudaFree(ctx->err);
    delete ctx;
    return cuda_fail(e, "cudaMalloc", "device error word");
  }
  e = cudaMalloc(&ctx->scratch, kq::kCtxScratchBytes);
  if (e != cudaSuccess) {
    cudaFree(ctx->err);
    delete ctx;
    return cuda_fail(e, "cudaMalloc", "context scratch");
  }
  ctx->scratch_bytes = kq::kCtxScratchBytes;
  int rc = kq::matvec_prepare(ctx);
  if (rc == KQ_OK) rc = kq::mma_prepare(ctx);
  if (rc == KQ_OK) rc = kq::warpmma_prepare(ctx);
  if (rc == KQ_OK) rc = kq::aux_prepare(ctx);
  if (rc == KQ_OK) rc = kq::types_prepare(ctx);
  if (rc != KQ_OK) {
    cudaFree(ctx->scratch);
    cudaFree(ctx->err);
    delete ctx;
    return rc;
  }
  *out = ctx;
  return KQ_OK;
}

int kq_ctx_destroy(kq_ctx* ctx) {
  if (!ctx) return KQ_OK;
  {
    kq::DeviceScope scope;
    scope.enter(ctx);
    // cudaFree waits for the device: no launch still reads what it frees
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->stage) cudaFree(ctx->stage);
    if (ctx->err) cudaFree(ctx->err);
  }
  delete ctx;
  return KQ_OK;
}

size_t kq_last_error(char* buf, size_t len) {
  const std::string& m = kq::t_last_error;
  if (buf && len) {
    const size_t n = m.size() < len - 1 ? m.size() : len - 1;
    std::memcpy(buf, m.data(), n);
    buf[n] = '\0';
  }
  return m.size();
}

int kq_ctx_info(const kq_ctx* ctx, int* device, int* sm_count, int* max_smem_per_block) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_ctx_info", "null ctx");
  if (device) *device = ctx->device;
  if (sm_count) *sm_count = ctx->sm_count;
  if (max_smem_per_block) *max_smem_per_block = ctx->max_smem;
  return KQ_OK;
}

int kq_device_error(kq_ctx* ctx) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_device_error", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned word = 0;
  e = cudaMemcpy(&word, ctx->err, sizeof(word), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy", "device error word");
  if (word == kq::kErrNone) return KQ_OK;
  cudaMemset(ctx->err, 0, sizeof(unsigned));
  const char* what = word == kq::kErrWaitFull    ? "a consumer gave up waiting for a bulk copy"
                     : word == kq::kErrWaitEmpty ? "the producer gave up waiting for a free slot"
                     : word == kq::kErrWaitPeer  ? "a wait on another GPU's flag gave up"
                                                 : "unknown";
  return fail(KQ_E_DEVICE, "kq_device_error",
              "device error word " + std::to_string(word) + ": " + what);
}

static int matvec_simple(kq_ctx* ctx, uint32_t type, uint64_t y, uint64_t w, uint64_t x,
                         uint32_t rows, uint32_t k, uint32_t batch, kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_matvec", "null ctx");
  kq_matvec_desc d = {};
  d.type = type;
  d.rows = rows;
  d.k = k;
  d.batch = batch;
  d.y = y;
  d.w = w;
  d.x = x;
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::matvec(ctx, d, static_cast<cudaStream_t>(stream));
}

int kq_matvec_q4k(kq_ctx* ctx, uint64_t y, uint64_t w, uint64_t x, uint32_t rows, uint32_t k,
                  uint32_t batch, kq_stream stream) {
  return matvec_simple(ctx, KQ_TYPE_Q4_K, y, w, x, rows, k, batch, stream);
}

int kq_matvec_q6k(kq_ctx* ctx, uint64_t y, uint64_t w, uint64_t x, uint32_t rows, uint32_t k,
                  uint32_t batch, kq_stream stream) {
  return matvec_simple(ctx, KQ_TYPE_Q6_K, y, w, x, rows, k, batch, stream);
}

int kq_matvec(kq_ctx* ctx, const kq_matvec_desc* desc, kq_stream stream) {
  if (!ctx || !desc) return fail(KQ_E_INVALID, "kq_matvec", "null ctx or descriptor");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::matvec(ctx, *desc, static_cast<cudaStream_t>(stream));
}

int kq_matvec_host(kq_ctx* ctx, const kq_matvec_desc* desc, float* y_host, const float* x_host,
                   kq_stream stream) {
  const char* call = "kq_matvec_host";
  if (!ctx || !desc || !y_host || !x_host) return fail(KQ_E_INVALID, call, "null argument");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  kq_matvec_desc d = *desc;
  if (d.batch == 0 || d.rows == 0 || d.k == 0)
    return fail(KQ_E_INVALID, call, "rows, k and batch must be positive");
  const bool pair = d.epilogue != KQ_EPILOGUE_NONE;
  const uint64_t ldx = d.ldx ? d.ldx : d.k;
  const uint64_t out_rows = pair ? d.rows / 2 : d.rows;
  const uint64_t ldy = d.ldy ? d.ldy : out_rows;
  if (ldx < d.k || ldy < out_rows)
    return fail(KQ_E_INVALID, call, "ldx must be >= k and ldy >= the output rows");
  // staging: x (batch rows of ldx floats, 256-byte aligned start of y after it), y (batch x ldy)
  const uint64_t xb = (uint64_t(d.batch) * ldx * 4 + 255) / 256 * 256;
  const uint64_t need = xb + uint64_t(d.batch) * ldy * 4;
  if (need > ctx->stage_bytes) {
    if (ctx->stage) {
      cudaError_t e = cudaFree(ctx->stage);  // waits for the device: no launch still uses it
      ctx->stage = nullptr;
      ctx->stage_bytes = 0;
      if (e != cudaSuccess) return cuda_fail(e, "cudaFree", "host-call staging");
    }
    const cudaError_t e = cudaMalloc(&ctx->stage, need);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc", "host-call staging");
    ctx->stage_bytes = need;
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* xs = static_cast<uint8_t*>(ctx->stage);
  float* ys = reinterpret_cast<float*>(xs + xb);
  cudaError_t e = cudaMemcpyAsync(xs, x_host, uint64_t(d.batch) * ldx * 4, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync", "x to the device");
  d.x = reinterpret_cast<uint64_t>(xs);
  d.y = reinterpret_cast<uint64_t>(ys);
  d.ldx = ldx;
  d.ldy = ldy;
  rc = kq::matvec(ctx, d, s);
  if (rc) return rc;
  e = cudaMemcpy2DAsync(y_host, ldy * 4, ys, ldy * 4, out_rows * 4, d.batch, cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy2DAsync", "y to the host");
  return KQ_OK;
}

int kq_dequant_q4k(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_dequant_q4k", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::dequant(ctx, 4, out, w, nblocks, static_cast<cudaStream_t>(stream));
}

int kq_dequant_q6k(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_dequant_q6k", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::dequant(ctx, 6, out, w, nblocks, static_cast<cudaStream_t>(stream));
}

int kq_dequant_q5k(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_dequant_q5k", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::dequant(ctx, 5, out, w, nblocks, static_cast<cudaStream_t>(stream));
}

int kq_fill_q5k(kq_ctx* ctx, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
                kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_fill_q5k", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::fill(ctx, 5, w, block0, nblocks, key, static_cast<cudaStream_t>(stream));
}

#define KQ_DEQUANT_ENTRY(name, type)                                                        \
  int name(kq_ctx* ctx, uint64_t out, uint64_t w, uint64_t nblocks, kq_stream stream) {     \
    if (!ctx) return fail(KQ_E_INVALID, #name, "null ctx");                                \
    kq::DeviceScope scope;                                                                  \
    int rc = scope.enter(ctx);                                                              \
    if (rc) return rc;                                                                      \
    return kq::dequant(ctx, type, out, w, nblocks, static_cast<cudaStream_t>(stream));      \
  }

KQ_DEQUANT_ENTRY(kq_dequant_q2k, 2)
KQ_DEQUANT_ENTRY(kq_dequant_q3k, 3)
KQ_DEQUANT_ENTRY(kq_dequant_q8_0, 8)

int kq_fill_q4k(kq_ctx* ctx, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
                kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_fill_q4k", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::fill(ctx, 4, w, block0, nblocks, key, static_cast<cudaStream_t>(stream));
}

int kq_fill_q6k(kq_ctx* ctx, uint64_t w, uint64_t block0, uint64_t nblocks, uint64_t key,
                kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_fill_q6k", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::fill(ctx, 6, w, block0, nblocks, key, static_cast<cudaStream_t>(stream));
}

uint64_t kq_stream_key(uint64_t seed, uint64_t tensor) { return kq::stream_key(seed, tensor); }

int kq_matvec_push(kq_ctx* ctx, const kq_matvec_desc* desc, const kq_push_desc* push,
                   kq_stream stream) {
  if (!ctx || !desc || !push) return fail(KQ_E_INVALID, "kq_matvec_push", "null ctx, descriptor or push");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::matvec(ctx, *desc, static_cast<cudaStream_t>(stream), push);
}

int kq_rope_append(kq_ctx* ctx, uint64_t qkv, uint64_t q_out, uint64_t k_cache, uint64_t v_cache,
                   uint32_t n_heads, uint32_t n_kv, uint32_t head_dim, uint32_t pos, double base,
                   kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_rope_append", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::rope_append(ctx, qkv, q_out, k_cache, v_cache, n_heads, n_kv, head_dim, pos, base,
                         static_cast<cudaStream_t>(stream));
}

int kq_attention_decode(kq_ctx* ctx, uint64_t out, uint64_t q, uint64_t k_cache, uint64_t v_cache,
                        uint32_t n_heads, uint32_t n_kv, uint32_t head_dim, uint32_t len,
                        uint64_t workspace, uint64_t workspace_bytes, kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_attention_decode", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::attention_decode(ctx, out, q, k_cache, v_cache, n_heads, n_kv, head_dim, len,
                              workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

uint64_t kq_attention_workspace(kq_ctx* ctx, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim,
                                uint32_t len) {
  if (!ctx || !n_kv) return 0;
  return kq::attention_workspace_bytes(ctx, n_heads, n_kv, head_dim, len ? len : 1);
}

// The warp-MMA kernels' cubin, embedded at build time (kernite_b200/build.py).
extern "C" const unsigned char kq_image_warpmma[];
extern "C" const unsigned char kq_image_warpmma_end[];

int kq_module_image(const void** image, size_t* bytes) {
  if (!image || !bytes) return fail(KQ_E_INVALID, "kq_module_image", "null argument");
  *image = kq_image_warpmma;
  *bytes = static_cast<size_t>(kq_image_warpmma_end - kq_image_warpmma);
  return KQ_OK;
}

int kq_matvec_plan(kq_ctx* ctx, const kq_matvec_desc* desc, kq_launch* out) {
  if (!ctx || !desc || !out) return fail(KQ_E_INVALID, "kq_matvec_plan", "null ctx, descriptor or out");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::warpmma_plan_launch(ctx, *desc, *out);
}

int kq_matvec_chain(kq_ctx* ctx, const kq_chain_job* jobs, uint32_t njobs, uint64_t epoch,
                    kq_stream stream) {
  if (!ctx || !jobs) return fail(KQ_E_INVALID, "kq_matvec_chain", "null ctx or jobs");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::warpmma_chain(ctx, jobs, njobs, epoch, static_cast<cudaStream_t>(stream));
}

int kq_epoch_advance(kq_ctx* ctx, uint64_t epoch, kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_epoch_advance", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::epoch_advance(ctx, epoch, static_cast<cudaStream_t>(stream));
}

int kq_tagged_unpack(kq_ctx* ctx, uint64_t dst, uint64_t src, uint64_t n, uint64_t epoch,
                     uint64_t wait_mul, uint64_t wait_add, kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_tagged_unpack", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::tagged_unpack(ctx, dst, src, n, epoch, wait_mul, wait_add, static_cast<cudaStream_t>(stream));
}

int kq_wait_counter(kq_ctx* ctx, uint64_t counter, uint64_t epoch, uint64_t wait_mul,
                    uint64_t wait_add, kq_stream stream) {
  if (!ctx) return fail(KQ_E_INVALID, "kq_wait_counter", "null ctx");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  return kq::wait_counter(ctx, counter, epoch, wait_mul, wait_add, static_cast<cudaStream_t>(stream));
}

int kq_peer_alloc(kq_ctx* ctx, uint64_t bytes, uint64_t* ptr, void* ipc_handle) {
  if (!ctx || !ptr || !ipc_handle || !bytes) return fail(KQ_E_INVALID, "kq_peer_alloc", "null argument or zero size");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc", "peer memory");
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaMemset", "peer memory");
  }
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaIpcGetMemHandle");
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = reinterpret_cast<uint64_t>(p);
  return KQ_OK;
}

int kq_peer_open(kq_ctx* ctx, const void* ipc_handle, uint64_t* ptr) {
  if (!ctx || !ipc_handle || !ptr) return fail(KQ_E_INVALID, "kq_peer_open", "null argument");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *ptr = reinterpret_cast<uint64_t>(p);
  return KQ_OK;
}

int kq_peer_close(kq_ctx* ctx, uint64_t ptr) {
  if (!ctx || !ptr) return fail(KQ_E_INVALID, "kq_peer_close", "null argument");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  const cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return KQ_OK;
}

int kq_peer_free(kq_ctx* ctx, uint64_t ptr) {
  if (!ctx || !ptr) return fail(KQ_E_INVALID, "kq_peer_free", "null argument");
  kq::DeviceScope scope;
  int rc = scope.enter(ctx);
  if (rc) return rc;
  const cudaError_t e = cudaFree(reinterpret_cast<void*>(ptr));
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree", "peer memory");
  return KQ_OK;
}

}  // extern "C"
