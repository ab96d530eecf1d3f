// Cross-shard log-sum-exp merge and the deterministic synthetic-input fill.
#include <cuda_fp16.h>

#include "nwd_common.h"

namespace {

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One block per (b, h) row, one thread per output element.  Shards are
// combined in index order (deterministic):
//   M = max_r m_r,  l = sum_r l_r 2^(m_r - M),  o = sum_r o_r 2^(m_r - M) / l.
__global__ void merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                             __half* __restrict__ out, uint32_t shards, uint32_t rows,
                             uint32_t hd) {
  const uint32_t r = blockIdx.x;
  float M = -INFINITY;
  for (uint32_t s = 0; s < shards; s++) M = fmaxf(M, part_ml[((size_t)s * rows + r) * 2]);
  float l = 0.f;
  for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
    float o = 0.f;
    l = 0.f;
    for (uint32_t s = 0; s < shards; s++) {
      const float m_s = part_ml[((size_t)s * rows + r) * 2];
      const float l_s = part_ml[((size_t)s * rows + r) * 2 + 1];
      if (l_s > 0.f) {
        const float f = ex2(m_s - M);
        l += l_s * f;
        o += part_o[((size_t)s * rows + r) * hd + d] * f;
      }
    }
    out[(size_t)r * hd + d] = __float2half_rn(l > 0.f ? o / l : 0.f);
  }
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Element i of stream `seed`: Irwin-Hall(12) over three splitmix64 outputs;
// the integer steps and the exact power-of-two scale make every element
// bit-identical to the CPU oracle's generator.
__global__ void fill_normal_kernel(__half* __restrict__ dst, uint64_t n, uint64_t seed_mix,
                                   uint64_t offset) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t base = seed_mix + 3ull * (offset + i);
    int64_t s = 0;
#pragma unroll
    for (int j = 0; j < 3; j++) {
      const uint64_t h = splitmix64(base + (uint64_t)j);
      s += (int64_t)(h & 0xffffu) + (int64_t)((h >> 16) & 0xffffu) +
           (int64_t)((h >> 32) & 0xffffu) + (int64_t)(h >> 48);
    }
    const float x = __fmul_rn((float)(s - 393210), 1.0f / 65536.0f);
    dst[i] = __float2half_rn(x);
  }
}

uint64_t host_splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

}  // namespace

using namespace nwd;

extern "C" {

int nwd_attn_merge(const float* part_o, const float* part_ml, uint16_t* o, uint32_t shards,
                   uint32_t batch, uint32_t n_heads, uint32_t head_dim, void* stream) {
  if (!part_o || !part_ml || !o) return fail(NWD_ERR_INVALID, "nwd_attn_merge: null pointer");
  if (shards == 0 || head_dim == 0) return fail(NWD_ERR_INVALID, "nwd_attn_merge: zero shape");
  const uint64_t rows = (uint64_t)batch * n_heads;
  if (rows == 0) return ok();
  if (rows > 0x7fffffffull) return fail(NWD_ERR_UNSUPPORTED, "nwd_attn_merge: too many rows");
  const uint32_t threads = head_dim >= 128 ? 128 : 32 * ((head_dim + 31) / 32);
  merge_kernel<<<(uint32_t)rows, threads, 0, (cudaStream_t)stream>>>(
      part_o, part_ml, reinterpret_cast<__half*>(o), shards, (uint32_t)rows, head_dim);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "nwd_attn_merge");
  return ok();
}

int nwd_fill_normal_f16(uint16_t* dst, uint64_t n, uint64_t seed, uint64_t offset, void* stream) {
  if (!dst && n) return fail(NWD_ERR_INVALID, "nwd_fill_normal_f16: null pointer");
  if (n == 0) return ok();
  uint64_t blocks = (n + 255) / 256;
  if (blocks > 148ull * 64) blocks = 148ull * 64;
  fill_normal_kernel<<<(uint32_t)blocks, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<__half*>(dst), n, host_splitmix64(seed), offset);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "nwd_fill_normal_f16");
  return ok();
}

}  // extern "C"
