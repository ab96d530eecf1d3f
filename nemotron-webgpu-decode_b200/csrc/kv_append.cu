// KV-cache row writes: kernels/kv_append.wgsl restated for fp16 caches.
//
// The WGSL runs one invocation per f32 element (kv_append.wgsl:13-18) and the
// engine dispatches it twice per attention layer (runtime.js:389-390).  Here
// one launch writes K and V, 16 bytes per thread (8 halves), so a 1024-half
// row (n_kv 8 x hd 128) is one 128-thread block.  The copy is a bit-exact
// move of 2-byte patterns.
#include "nwd_common.h"

namespace {

constexpr int kThreads = 128;

// Copies n halves from src[j] to dst[j] (j = which of K/V via blockIdx.y).
// vec: n % 8 == 0 and both pointers 16-byte aligned.
__global__ void __launch_bounds__(kThreads) kv_append_kernel(const uint16_t* __restrict__ k_src,
                                                             const uint16_t* __restrict__ v_src,
                                                             uint16_t* __restrict__ k_dst,
                                                             uint16_t* __restrict__ v_dst,
                                                             uint32_t n, bool vec) {
  const uint16_t* src = blockIdx.y ? v_src : k_src;
  uint16_t* dst = blockIdx.y ? v_dst : k_dst;
  if (vec) {
    uint32_t i = blockIdx.x * kThreads + threadIdx.x;
    if (i < n / 8)
      reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
  } else {
    for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n; i += gridDim.x * kThreads)
      dst[i] = src[i];
  }
}

// One block row per sequence: row = row_offset[b] + pos[b] of the pool.
__global__ void __launch_bounds__(kThreads) kv_append_batched_kernel(
    const uint16_t* __restrict__ k_src, const uint16_t* __restrict__ v_src,
    uint16_t* __restrict__ k_pool, uint16_t* __restrict__ v_pool, uint64_t pool_rows,
    const int64_t* __restrict__ row_offset, const int32_t* __restrict__ pos, uint32_t n,
    uint32_t* err_count) {
  const uint32_t b = blockIdx.y;
  const int64_t row = row_offset[b] + (int64_t)pos[b];
  if (row < 0 || (uint64_t)row >= pool_rows) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && err_count) atomicAdd(err_count, 1u);
    return;
  }
  const uint4* ks = reinterpret_cast<const uint4*>(k_src + (size_t)b * n);
  const uint4* vs = reinterpret_cast<const uint4*>(v_src + (size_t)b * n);
  uint4* kd = reinterpret_cast<uint4*>(k_pool + (size_t)row * n);
  uint4* vd = reinterpret_cast<uint4*>(v_pool + (size_t)row * n);
  for (uint32_t i = blockIdx.x * kThreads + threadIdx.x; i < n / 8; i += gridDim.x * kThreads) {
    kd[i] = __ldg(ks + i);
    vd[i] = __ldg(vs + i);
  }
}

int launch_append(const uint16_t* k_src, const uint16_t* v_src, uint16_t* k_cache,
                  uint16_t* v_cache, uint32_t seq, uint32_t n_kv, uint32_t hd, uint32_t cap,
                  void* stream, const char* who) {
  using namespace nwd;
  if (!k_src || !k_cache || (v_cache && !v_src))
    return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  if (n_kv == 0 || hd == 0) return fail(NWD_ERR_INVALID, "%s: n_kv and hd must be > 0", who);
  if (seq >= cap) return fail(NWD_ERR_RANGE, "seq %u exceeds maxSeq %u", seq, cap);
  const uint64_t n64 = (uint64_t)n_kv * hd;
  if (n64 > (1ull << 30)) return fail(NWD_ERR_INVALID, "%s: row of %llu halves is too large", who,
                                      (unsigned long long)n64);
  const uint32_t n = (uint32_t)n64;
  uint16_t* kd = k_cache + (size_t)seq * n;
  uint16_t* vd = v_cache ? v_cache + (size_t)seq * n : nullptr;
  bool vec = (n % 8 == 0) && aligned16(k_src) && aligned16(kd) &&
             (!vd || (aligned16(v_src) && aligned16(vd)));
  uint32_t blocks = vec ? (n / 8 + kThreads - 1) / kThreads : (n + kThreads - 1) / kThreads;
  if (blocks > 65535u) blocks = 65535u;
  dim3 grid(blocks, vd ? 2 : 1);
  kv_append_kernel<<<grid, kThreads, 0, (cudaStream_t)stream>>>(k_src, v_src, kd, vd, n, vec);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
}

}  // namespace

using namespace nwd;

extern "C" {

int nwd_kv_append(const uint16_t* src, uint16_t* cache, uint32_t seq, uint32_t n_kv, uint32_t hd,
                  uint32_t cap, void* stream) {
  return launch_append(src, nullptr, cache, nullptr, seq, n_kv, hd, cap, stream, "nwd_kv_append");
}

int nwd_kv_append_kv(const uint16_t* k_src, const uint16_t* v_src, uint16_t* k_cache,
                     uint16_t* v_cache, uint32_t seq, uint32_t n_kv, uint32_t hd, uint32_t cap,
                     void* stream) {
  if (!v_src || !v_cache) return fail(NWD_ERR_INVALID, "nwd_kv_append_kv: null pointer");
  return launch_append(k_src, v_src, k_cache, v_cache, seq, n_kv, hd, cap, stream,
                       "nwd_kv_append_kv");
}

int nwd_kv_append_batched(const uint16_t* k_src, const uint16_t* v_src, uint16_t* k_pool,
                          uint16_t* v_pool, uint64_t pool_rows, const int64_t* row_offset,
                          const int32_t* pos, uint32_t batch, uint32_t n_kv, uint32_t hd,
                          uint32_t* err_count, void* stream) {
  if (!k_src || !v_src || !k_pool || !v_pool || !row_offset || !pos)
    return fail(NWD_ERR_INVALID, "nwd_kv_append_batched: null pointer");
  if (batch == 0) return ok();
  if (n_kv == 0 || hd == 0) return fail(NWD_ERR_INVALID, "nwd_kv_append_batched: zero shape");
  if (batch > 65535u) return fail(NWD_ERR_UNSUPPORTED, "nwd_kv_append_batched: batch > 65535");
  const uint32_t n = n_kv * hd;
  if (n % 8 != 0 || !aligned16(k_src) || !aligned16(v_src) || !aligned16(k_pool) ||
      !aligned16(v_pool))
    return fail(NWD_ERR_UNSUPPORTED,
                "nwd_kv_append_batched: rows must be a multiple of 8 halves, pointers 16-byte aligned");
  uint32_t bx = (n / 8 + kThreads - 1) / kThreads;
  kv_append_batched_kernel<<<dim3(bx, batch), kThreads, 0, (cudaStream_t)stream>>>(
      k_src, v_src, k_pool, v_pool, pool_rows, row_offset, pos, n, err_count);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "nwd_kv_append_batched");
  return ok();
}

}  // extern "C"
