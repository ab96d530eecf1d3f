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
// Every shard's (m, l) is read at once into shared memory and the o terms are
// loaded four shards at a time, so a row costs a few memory round trips
// whatever the shard count.  Shard s's o starts at part_o + s * so and its
// (m, l) pairs at part_ml + s * sml; an empty shard (l = 0) contributes
// nothing, whatever its o holds.
constexpr uint32_t MERGE_MAX_SHARDS = 4096;

__global__ void merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                             __half* __restrict__ out, uint32_t shards, uint32_t rows,
                             uint32_t hd, uint64_t so, uint64_t sml) {
  extern __shared__ float sw[];  // [shards] m_s, then weights; [shards] l_s
  const uint32_t r = blockIdx.x;
  for (uint32_t s = threadIdx.x; s < shards; s += blockDim.x) {
    sw[s] = part_ml[s * sml + (uint64_t)r * 2];
    sw[shards + s] = part_ml[s * sml + (uint64_t)r * 2 + 1];
  }
  __syncthreads();
  float M = -INFINITY;
  for (uint32_t s = 0; s < shards; s++) M = fmaxf(M, sw[s]);
  __syncthreads();  // every thread has M before the m values are replaced
  for (uint32_t s = threadIdx.x; s < shards; s += blockDim.x)
    sw[s] = sw[shards + s] > 0.f ? ex2(sw[s] - M) : 0.f;
  __syncthreads();
  float l = 0.f;
  for (uint32_t s = 0; s < shards; s++)
    if (sw[shards + s] > 0.f) l += sw[shards + s] * sw[s];
  const float* po = part_o + (uint64_t)r * hd;
  for (uint32_t d = threadIdx.x; d < hd; d += blockDim.x) {
    float o = 0.f;
    uint32_t s = 0;
    for (; s + 4 <= shards; s += 4) {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; i++) v[i] = po[(s + i) * so + d];
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (sw[shards + s + i] > 0.f) o += v[i] * sw[s + i];
    }
    for (; s < shards; s++)
      if (sw[shards + s] > 0.f) o += po[s * so + d] * sw[s];
    out[(uint64_t)r * hd + d] = __float2half_rn(l > 0.f ? o / l : 0.f);
  }
}

int launch_merge(const float* part_o, const float* part_ml, uint16_t* o, uint32_t shards,
                 uint32_t batch, uint32_t n_heads, uint32_t head_dim, uint64_t so, uint64_t sml,
                 void* stream, const char* who) {
  using namespace nwd;
  if (!part_o || !part_ml || !o) return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  if (shards == 0 || head_dim == 0) return fail(NWD_ERR_INVALID, "%s: zero shape", who);
  if (shards > MERGE_MAX_SHARDS)
    return fail(NWD_ERR_UNSUPPORTED, "%s: %u shards (at most %u)", who, shards, MERGE_MAX_SHARDS);
  const uint64_t rows = (uint64_t)batch * n_heads;
  if (rows == 0) return ok();
  if (rows > 0x7fffffffull) return fail(NWD_ERR_UNSUPPORTED, "%s: too many rows", who);
  const uint32_t threads = head_dim >= 128 ? 128 : 32 * ((head_dim + 31) / 32);
  merge_kernel<<<(uint32_t)rows, threads, 2 * shards * sizeof(float), (cudaStream_t)stream>>>(
      part_o, part_ml, reinterpret_cast<__half*>(o), shards, (uint32_t)rows, head_dim, so, sml);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
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
  const uint64_t rows = (uint64_t)batch * n_heads;
  return launch_merge(part_o, part_ml, o, shards, batch, n_heads, head_dim, rows * head_dim,
                      rows * 2, stream, "nwd_attn_merge");
}

int nwd_attn_merge_packed(const float* packed, uint16_t* o, uint32_t shards, uint32_t batch,
                          uint32_t n_heads, uint32_t head_dim, void* stream) {
  const uint64_t rows = (uint64_t)batch * n_heads;
  const uint64_t stride = rows * ((uint64_t)head_dim + 2);
  return launch_merge(packed, packed ? packed + rows * head_dim : nullptr, o, shards, batch,
                      n_heads, head_dim, stride, stride, stream, "nwd_attn_merge_packed");
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
