// Shared helpers for the gpb200 CUDA library: status handling, the per-thread
// last-error string, and the small set of sm_100a PTX primitives (mbarrier,
// 1-D bulk-copy TMA, ex2) the tiled kernels use.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <string>

#include "gpb200.h"

namespace gpb {

// ---------------------------------------------------------------------------
// Errors: every C-ABI entry returns an int status; the message is kept per
// thread and read back with gpb_last_error().
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

#define GPB_CHECK_CUDA(expr)                                                     \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess) {                                                     \
      ::gpb::set_error("%s:%d: %s failed: %s", __FILE__, __LINE__, #expr,        \
                       cudaGetErrorString(_e));                                  \
      return GPB_ERR_CUDA;                                                       \
    }                                                                            \
  } while (0)

#define GPB_TRY(expr)                                                            \
  do {                                                                           \
    int _s = (expr);                                                             \
    if (_s != GPB_OK) return _s;                                                 \
  } while (0)

#define GPB_REQUIRE(cond, code, ...)                                             \
  do {                                                                           \
    if (!(cond)) {                                                               \
      ::gpb::set_error(__VA_ARGS__);                                             \
      return (code);                                                             \
    }                                                                            \
  } while (0)

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

// Device error word written by kernels whose bounded waits gave up.
// Codes: 1 = mbarrier wait timed out in a tiled kernel.
enum DeviceErr : int { DEV_OK = 0, DEV_WAIT_TIMEOUT = 1 };

// ---------------------------------------------------------------------------
// PTX primitives (sm_90+/sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// try_wait with a suspend-time hint: the thread may sleep up to `hint_ns`
// inside the instruction until the phase completes.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Suspend-time hint (ns) for the polls of mbar_wait_bounded: a waiting thread
// sleeps inside try_wait until the phase completes or the hint expires,
// instead of re-issuing the poll (measured +1.4 % on the Gram K·V kernel,
// whose 24 issuer and epilogue warps mostly wait); 0 = plain try_wait.
#ifndef GPB_WAIT_HINT_NS
#define GPB_WAIT_HINT_NS 20000
#endif

// Wait on an mbarrier phase for at most about `limit_ns`; returns false on
// timeout. The clock is read once per 32 polls, so a spinning thread costs
// few issue slots.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = 4000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int k = 0; k < 32; ++k) {
      const bool done = GPB_WAIT_HINT_NS > 0 ? mbar_try_wait_hint(bar, parity, GPB_WAIT_HINT_NS)
                                             : mbar_try_wait(bar, parity);
      if (done) return true;
    }
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// Before a producer's CTA may exit: wait (bounded) until every bulk copy it
// issued into a ring of S slots has landed. Tile kt went to slot kt % S with
// phase parity (kt / S) & 1, so the last S tiles cover every copy that can
// still be in flight; on the normal path these phases completed long ago.
template <int S>
__device__ __forceinline__ void drain_ring(uint64_t* full_bar, int issued) {
  for (int kt = issued > S ? issued - S : 0; kt < issued; ++kt)
    (void)mbar_wait_bounded(&full_bar[kt % S], (uint32_t)((kt / S) & 1), 100000000ull);
}

// 1-D bulk copy global -> shared through the TMA engine, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Hardware base-2 exponential (MUFU.EX2), flush-to-zero.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Hardware base-2 logarithm (MUFU.LG2).
__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// e^x through ex2: relative error ~1e-6 for |x| <= 20, enough for the 1e-5
// matvec tolerance.
__device__ __forceinline__ float exp_fast(float x) { return ex2_approx(x * kLog2e); }

}  // namespace gpb
