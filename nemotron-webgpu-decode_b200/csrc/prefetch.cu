// L2 prefetch of constant buffers (q4 weights) ahead of the launches that read
// them.  An engine issues it on a side stream once the previous kernel's reads
// are done, so that the next projection's weights cross HBM while a latency-
// bound kernel (decode attention of one token) leaves the memory system idle;
// the projection then reads them from L2.  The engine's decode step
// (engine/runtime.js:385-394) runs its projections back to back with nothing
// in between, so there is no counterpart in the reference.
//
// A prefetch moves no data into any SM and orders nothing: L2 is the point of
// coherence, so it is safe whatever else runs, and results never depend on it.
#include <cstdint>

#include "nwd_common.h"

namespace {

constexpr uint32_t PF_MAX_RANGES = 16;
constexpr uint32_t PF_CHUNK = 32768;  // bytes per bulk prefetch

struct PfRanges {
  uint64_t addr[PF_MAX_RANGES];   // 16-byte aligned
  uint64_t bytes[PF_MAX_RANGES];  // multiple of 16
  uint64_t chunk_end[PF_MAX_RANGES];  // running chunk count through range i
  uint32_t n;
};

// One issuing thread per CTA, CTAs spread over the SMs so that each SM's copy
// engine gets a few large requests: chunk c of the ranges laid end to end.
__global__ void prefetch_l2_kernel(const __grid_constant__ PfRanges r) {
  if (threadIdx.x != 0) return;
  const uint64_t total = r.chunk_end[r.n - 1];
  uint32_t i = 0;
  for (uint64_t c = blockIdx.x; c < total; c += gridDim.x) {
    while (c >= r.chunk_end[i]) i++;  // c only grows: ranges are walked once
    const uint64_t first = i ? r.chunk_end[i - 1] : 0;
    const uint64_t off = (c - first) * PF_CHUNK;
    const uint64_t left = r.bytes[i] - off;
    const uint32_t sz = (uint32_t)(left < PF_CHUNK ? left : PF_CHUNK);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(r.addr[i] + off), "r"(sz)
                 : "memory");
  }
}

}  // namespace

using namespace nwd;

extern "C" {

int nwd_prefetch_l2(const void* const* ptrs, const uint64_t* bytes, uint32_t n, void* stream) {
  if (n > PF_MAX_RANGES)
    return fail(NWD_ERR_INVALID, "nwd_prefetch_l2: %u ranges (at most %u)", n, PF_MAX_RANGES);
  if (n && (!ptrs || !bytes)) return fail(NWD_ERR_INVALID, "nwd_prefetch_l2: null pointer");
  PfRanges r = {};
  uint64_t chunks = 0;
  uint32_t m = 0;
  for (uint32_t i = 0; i < n; i++) {
    if (!bytes[i]) continue;
    if (!ptrs[i]) return fail(NWD_ERR_INVALID, "nwd_prefetch_l2: null pointer (range %u)", i);
    // the 16-byte aligned interior of the range (a prefetch is only a hint)
    const uint64_t a = reinterpret_cast<uint64_t>(ptrs[i]);
    const uint64_t a0 = (a + 15) & ~15ull, e = (a + bytes[i]) & ~15ull;
    if (e <= a0) continue;
    r.addr[m] = a0;
    r.bytes[m] = e - a0;
    chunks += (e - a0 + PF_CHUNK - 1) / PF_CHUNK;
    r.chunk_end[m] = chunks;
    m++;
  }
  r.n = m;
  if (!m) return ok();
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st) return st;
  const uint64_t cap = 4ull * (uint64_t)di.sm_count;
  const uint32_t grid = (uint32_t)(chunks < cap ? chunks : cap);
  prefetch_l2_kernel<<<grid, 32, 0, (cudaStream_t)stream>>>(r);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "nwd_prefetch_l2");
  return ok();
}

}  // extern "C"
