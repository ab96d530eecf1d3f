// PTX building blocks shared by the library's kernels: shared-memory
// addresses, the global timer, mbarriers with bounded waits, TMA and bulk
// copies, L2 cache policies.  Every wait gives up after WAIT_LIMIT_NS of the
// global timer (2 s), raises the caller's abort flag and records
// NWD_DEVERR_PIPE_TIMEOUT, so no kernel here can spin forever.  A count of
// WAIT_LIMIT_ITERS polls is only a backstop should the timer not advance: a
// poll takes well over 2 s / 2^30 (about 2 ns), so the timer ends every wait
// first.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "nwd.h"

namespace nwd {
namespace ptx {

constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s
constexpr uint32_t WAIT_LIMIT_ITERS = 1u << 30;  // backstop only

// ---------------- PTX wrappers ----------------
static __device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
static __device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
static __device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
static __device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
static __device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
static __device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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
// Atomic add with acquire and release semantics at gpu scope; returns the old value.
static __device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// Non-blocking test of a phase (never suspends the thread).
static __device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait.  Returns false if the CTA is aborting (another thread gave
// up) or this wait ran past its limits (then it raises the abort itself).
static __device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int32_t* abort,
                                          uint32_t* dev_err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31) == 0) {
      if (*abort) return false;
      if (i >= WAIT_LIMIT_ITERS || globaltimer() - t0 > WAIT_LIMIT_NS) {
        *abort = 1;
        atomicOr(dev_err, NWD_DEVERR_PIPE_TIMEOUT);
        return false;
      }
    }
  }
}
// Warp-uniform bounded wait: every lane waits (so every lane acquires the
// barrier's completion), then the warp agrees; if any lane gave up, all do.
static __device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int32_t* abort,
                                          uint32_t* dev_err) {
  const bool ok = mbar_wait(bar, parity, abort, dev_err);
  return __all_sync(0xffffffffu, ok);
}
// L2 prefetch of one tile (no shared memory, no barrier).  L2 is the point of
// coherence, so it is safe even while another kernel may still write the rows.
static __device__ __forceinline__ void tma_prefetch_4d(const CUtensorMap* map, int c0, int c1, int c2,
                                                int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
static __device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "l"(policy)
      : "memory");
}
static __device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
static __device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
static __device__ __forceinline__ uint64_t evict_last_policy() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

}  // namespace ptx
}  // namespace nwd
