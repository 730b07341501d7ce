// common.cuh -- sm_100a device helpers shared by every kernel of libugb.
//
// Bulk-copy (TMA) + mbarrier pipeline primitives written as inline PTX, bounded waits that
// report through the device status word instead of hanging, and small integer helpers.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "../../include/ugb.h"

namespace ugb {

// Bits of the device status word (ugb_ctx::status).  Any kernel may OR these in; the host
// reads and clears the word with ugb_status_read().
enum : uint32_t {
  ST_NONFINITE_IN = 1u << 0,   // a non-finite activation reached a quantiser
  ST_NONFINITE_OUT = 1u << 1,  // a kernel produced a non-finite output
  ST_TIMEOUT = 1u << 2,        // a bounded wait gave up (copy or peer never arrived)
  ST_BADARG = 1u << 3,         // a descriptor failed a device-side bounds check
};

__device__ __forceinline__ void status_or(uint32_t *status, uint32_t bits) {
  if (status) atomicOr(status, bits);
}

// ---- shared-memory addressing -----------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ void sts8(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b8 [%0], %1;" ::"r"(addr), "r"(v));
}

__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v));
}

// ---- mbarrier -----------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive without release ordering.  Used to hand a ring stage back to the producer: the
// consumer's shared-memory reads of the stage have completed (their values were consumed by
// the arithmetic that precedes this instruction), and a release arrive would also wait for
// the thread's earlier global stores to become visible -- a full L2 round trip per stage.
__device__ __forceinline__ void mbar_arrive_relaxed(uint32_t bar) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// n arrivals at once (n >= 1).
__device__ __forceinline__ void mbar_arrive_relaxed_n(uint32_t bar, uint32_t n) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}

// Test a phase; if it has not completed, the thread is suspended in hardware until it
// completes or about kSuspendNs pass, so waiting warps do not spin on issue slots.
constexpr uint32_t kSuspendNs = 1000000;
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Default limit of every device-side wait: far above any legitimate copy latency, short
// enough that a lost copy surfaces as UGB_ETIMEOUT instead of a hung GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Wait for phase `parity` of an mbarrier, giving up after kWaitLimitNs.  Returns false on
// timeout (the caller records ST_TIMEOUT and leaves uniformly).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - start > kWaitLimitNs) return false;
  }
}

// ---- bulk copies (TMA, non-tensor) ---------------------------------------------------------

// Global -> shared bulk copy completing on an mbarrier.  dst, src 16-byte aligned; bytes a
// positive multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- programmatic dependent launch -----------------------------------------------------------

// Block until the grids this launch depends on have completed and flushed (no-op when the
// launch carried no programmatic dependency).
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Allow the next grid in the stream to begin launching.
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- numerics ---------------------------------------------------------------------------------

__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xffffu)));
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// The 40 bytes at addr & ~7 as 10 words (five 64-bit loads), shifted down by one word when
// addr & 7 >= 4, so that s[0] holds byte (addr & ~3) onward.  64-bit loads of runs spaced 34
// or 110 bytes apart (GGUF Q8_0 / Q3_K blocks) hit 16 distinct bank pairs per half-warp, so
// they are conflict-free where 32-bit loads of the same runs are 2-way conflicted.
__device__ __forceinline__ void lds_window9(uint32_t addr, uint32_t (&s)[9]) {
  const uint32_t a8 = addr & ~7u;
  uint32_t r[10];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const uint2 v = lds64(a8 + 8u * i);
    r[2 * i] = v.x;
    r[2 * i + 1] = v.y;
  }
  const bool hi = (addr & 4u) != 0;
#pragma unroll
  for (int i = 0; i < 9; ++i) s[i] = hi ? r[i + 1] : r[i];
}

// 32 little-endian bytes starting at a 2-byte aligned shared address, as 8 words:
// word i = bytes [4i, 4i+4) of the run.
__device__ __forceinline__ void lds_words8_u2(uint32_t addr, uint32_t (&w)[8]) {
  uint32_t s[9];
  lds_window9(addr, s);
  const uint32_t sh = (addr & 3u) * 8u;
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = __funnelshift_rc(s[i], s[i + 1], sh);
}

__device__ __forceinline__ uint32_t lds16_u2(uint32_t addr) {
  const uint32_t w = lds32(addr & ~3u);
  return (w >> ((addr & 3u) * 8u)) & 0xffffu;
}

__device__ __forceinline__ uint32_t lds8(uint32_t addr) {
  const uint32_t w = lds32(addr & ~3u);
  return (w >> ((addr & 3u) * 8u)) & 0xffu;
}

__host__ __device__ constexpr inline uint64_t round_up(uint64_t x, uint64_t m) {
  return (x + m - 1) / m * m;
}

}  // namespace ugb
