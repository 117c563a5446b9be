// kq_device.cuh -- device-side building blocks for sm_100a: block formats, mbarriers, bulk
// (TMA 1-D) copies, programmatic dependent launch, bounded waits.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "kq.h"

namespace kq {

constexpr int kQK = 256;
constexpr int kQ4KBytes = 144;  // fp16 d, fp16 dmin, u8 scales[12], u8 qs[128]
constexpr int kQ6KBytes = 210;  // u8 ql[128], u8 qh[64], i8 scales[16], fp16 d
constexpr int kQ5KBytes = 176;  // fp16 d, fp16 dmin, u8 scales[12], u8 qh[32], u8 qs[128]

// Device error word codes: a bounded wait that gives up writes one (first writer wins) and its
// kernel returns instead of hanging; kq_device_error() reads and clears it.
enum : unsigned {
  kErrNone = 0,
  kErrWaitFull = 1,   // a consumer gave up waiting for a stage's bulk copy
  kErrWaitEmpty = 2,  // the producer gave up waiting for consumers to free a stage
  kErrWaitPeer = 3,   // a wait on another GPU's flag gave up
};

// About two seconds: far above any legitimate wait of these kernels (microseconds).
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(unsigned* err, unsigned code) {
  if (err) atomicCAS(err, 0u, code);
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// This GPU's step counter, written by an earlier kernel on the stream: after pdl_wait() (or a
// kernel boundary) its value is visible, so a relaxed GPU-scope load will do (an acquire at
// system scope costs microseconds on the critical path of every CTA).
__device__ __forceinline__ unsigned long long ld_epoch(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Waits (acquire, system scope) until *cnt >= (*epoch - 1) * mul + add: the arrival count other
// GPUs add to after storing into this GPU's memory. Gives up after kWaitBudgetNs, at once when
// an earlier wait already failed (so one missing rank costs one budget, not one per launch), and
// then records kErrWaitPeer and returns false.
__device__ __forceinline__ bool wait_count(unsigned* err, const unsigned long long* cnt,
                                           const unsigned long long* epoch, uint64_t mul,
                                           uint64_t add) {
  const unsigned long long target = (ld_epoch(epoch) - 1ull) * mul + add;
  if (ld_acquire_sys(cnt) >= target) return true;
  bool ok = false;
  if (!(err && *reinterpret_cast<volatile unsigned*>(err))) {
    const uint64_t t0 = globaltimer();
    while (!(ok = ld_acquire_sys(cnt) >= target)) {
      if (globaltimer() - t0 > kWaitBudgetNs) break;
      __nanosleep(64);
    }
  }
  if (!ok) report_error(err, kErrWaitPeer);
  return ok;
}

// ---------------------------------------------------------------- mbarriers

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread may sleep up to `ns` nanoseconds waiting for the
// phase instead of returning at once.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// The same bounded wait as mbar_wait, sleeping in the barrier between polls.
__device__ __forceinline__ bool mbar_wait_sleep(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 2000u)) return true;
    if (globaltimer() - t0 > kWaitBudgetNs) return false;
  }
}

// Waits for phase `parity` of `bar` to complete; false after kWaitBudgetNs without it.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitBudgetNs) return false;
  }
}

// ---------------------------------------------------------------- bulk copies (TMA, 1-D)

// Creates an L2 policy that evicts streamed weights first, so they do not push x and y out.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Copies `bytes` (multiple of 16) from global `src` (16-byte aligned) to shared `dst` (16-byte
// aligned), completing `bytes` transactions on mbarrier `bar`.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// The same without an L2 policy.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------- per-thread async copies

// 16 bytes global -> shared, asynchronous, cached in L2 only.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits until at most N of this thread's committed groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch

// Waits until the grids this one depends on have completed and their memory is visible.
// A no-op for a kernel launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next kernel on the stream launch (its CTAs then wait in pdl_wait()).
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- epilogues

// The product epilogues of a row pair (v0: the gate row, v1: the up row): v0 v1 s, or
// silu(v0) v1 s with silu(z) = z / (1 + e^-z) (expf: CUDA's accurate exponential).
__device__ __forceinline__ float pair_value(float v0, float v1, uint32_t epilogue, float s) {
  if (epilogue == KQ_EPILOGUE_SILU_PRODUCT) v0 = v0 / (1.f + expf(-v0));
  return v0 * v1 * s;
}

// ---------------------------------------------------------------- misc

__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds_v2(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ int lds_s8(uint32_t addr) {
  int v;
  asm volatile("ld.shared.s8 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ void sts_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

template <int OFF>
__device__ __forceinline__ uint32_t lds_u32_at(uint32_t base) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(base), "n"(OFF));
  return v;
}

template <int I, int N>
struct UnalignedWords {
  __device__ __forceinline__ static void load(uint32_t base, uint32_t (&w)[N + 1]) {
    w[I] = lds_u32_at<4 * I>(base);
    UnalignedWords<I + 1, N>::load(base, w);
  }
};
template <int N>
struct UnalignedWords<N, N> {
  __device__ __forceinline__ static void load(uint32_t base, uint32_t (&w)[N + 1]) {
    w[N] = lds_u32_at<4 * N>(base);
  }
};

// `N` 32-bit words starting at shared address `addr`, which is only 2-byte aligned: N+1 aligned
// loads (immediate offsets from one base) and a funnel shift per word.
template <int N>
__device__ __forceinline__ void lds_words_unaligned(uint32_t addr, uint32_t (&out)[N]) {
  const uint32_t base = addr & ~3u;
  const uint32_t sh = (addr & 3u) * 8u;
  uint32_t w[N + 1];
  UnalignedWords<0, N>::load(base, w);
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// Float whose bits are `bits`, and back.
__device__ __forceinline__ float as_f32(uint32_t u) { return __uint_as_float(u); }

// fp16 bits -> f32 (exact).
__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

}  // namespace kq
