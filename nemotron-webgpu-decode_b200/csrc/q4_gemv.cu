// q4 GEMV (decode, one activation vector): the projections either side of
// the attention path.  The engine runs kernels/matmul_nbits_sg.wgsl for an
// attention layer's q/k/v projections (engine/runtime.js:321-329), feeds k/v
// to kv_append and q to attention (:389-391), then runs the same GEMV for
// o_proj and adds it into the hidden state (:330, :392-393, kernels/add.wgsl).
//
// Weights keep the reference's MatMulNBits layout, so the engine's buffers are
// used as they are: per output column n, n_blocks blocks of 32 four-bit values
// (16 bytes: element j of a u32 word is bits [4j, 4j+4)), one f32 scale per
// block ([N][n_blocks]) and one 4-bit zero point per block (packed 8 per u32,
// nibble n*n_blocks + blk).  Element value (q - zero) * scale.
//
// HBM-bound: a column's weights are read once (20.5 bytes per 32 elements).
// A warp takes a group of 4 columns; the 4 lanes of a block each take one
// 8-element word, so for each column the warp's 32 lanes read 8 consecutive
// blocks = 128 contiguous bytes, and a lane keeps 4 block rows x 4 columns of
// words in flight.  The lane's 8 activations are read once from shared memory
// and used for all 4 columns.  A block's term is computed as
//   scale * (sum_j a_j q_j - zero * sum_j a_j),
// with the per-block sums of A formed once per CTA in shared memory, so an
// element costs an integer extract, a float add and one FMA (no conversion
// through the special-function unit).  f32 accumulation throughout; the lanes
// are reduced with shuffles at the end of the column group.
#include <cuda_fp16.h>

#include <algorithm>

#include "nwd_common.h"

namespace {

constexpr int GEMV_THREADS = 128;      // 4 warps
constexpr int CG = 4;                  // columns per warp
constexpr int UNROLL = 4;              // block rows in flight per lane (x 8 block slots per warp)
constexpr uint32_t MAX_BLOCKS = 1024;  // K <= 32768 (shared-memory copy of A and its block sums)
constexpr size_t smem_bytes(uint32_t n_blocks) { return (size_t)n_blocks * 33 * sizeof(float); }

enum OutMode : int {
  OUT_F32 = 0,  // Y[n] (epilogue 0), relu2 (1), Y[n] += (2)
  OUT_QKV = 1,  // columns [0,Nq) -> q fp16, [Nq,Nq+Nk) -> k cache row, then v cache row
};

struct Q4 {
  const uint32_t* B;      // [N][n_blocks][4]
  const float* scales;    // [N][n_blocks]
  const uint32_t* zp;     // [ceil(N*n_blocks/8)]
  uint32_t N;
};

struct GemvArgs {
  Q4 w[3];            // one matrix, or q / k / v
  uint32_t n_mats;
  uint32_t n_total;   // columns over all matrices
  uint32_t n_blocks;
  uint32_t epilogue;  // OUT_F32 only
  float* y;           // OUT_F32
  __half* q_out;      // OUT_QKV
  __half* k_row;      // OUT_QKV: the cache rows the new token's k / v go to
  __half* v_row;
};

template <typename AT>
__device__ __forceinline__ float a_at(const AT* a, uint32_t i);
template <>
__device__ __forceinline__ float a_at<float>(const float* a, uint32_t i) {
  return __ldg(a + i);
}
template <>
__device__ __forceinline__ float a_at<__half>(const __half* a, uint32_t i) {
  return __half2float(a[i]);
}

// float value of the 4-bit field at bit 4j of p: 2^23 + q as a float, minus 2^23 (exact)
__device__ __forceinline__ float nib_f(uint32_t p, int j) {
  return __uint_as_float(((p >> (4 * j)) & 15u) | 0x4B000000u) - 8388608.0f;
}

template <typename AT, int MODE>
__global__ void __launch_bounds__(GEMV_THREADS)
    q4_gemv_kernel(const AT* __restrict__ a, const GemvArgs args) {
  extern __shared__ float sa[];  // A as f32 [K], then the per-block sums of A [n_blocks]
  const uint32_t nb = args.n_blocks, K = nb * 32;
  float* sasum = sa + K;
  for (uint32_t i = threadIdx.x; i < K; i += GEMV_THREADS) sa[i] = a_at<AT>(a, i);
  __syncthreads();
  for (uint32_t b = threadIdx.x; b < nb; b += GEMV_THREADS) {
    float s = 0.f;
#pragma unroll 8
    for (int j = 0; j < 32; j++) s += sa[b * 32 + j];
    sasum[b] = s;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t word = (uint32_t)lane & 3u, slot = (uint32_t)lane >> 2;
  const uint32_t n_groups = (args.n_total + CG - 1) / CG;
  const uint32_t n_warps = gridDim.x * (GEMV_THREADS / 32);
  for (uint32_t g = blockIdx.x * (GEMV_THREADS / 32) + warp; g < n_groups; g += n_warps) {
    // each column of the group: its matrix (selected without indexing the
    // parameter block) and its first block
    const uint32_t* Bp[CG];
    const float* Sp[CG];
    const uint32_t* Zp[CG];
    uint32_t mat[CG], cl[CG];
    uint64_t base[CG];
    bool live[CG];
#pragma unroll
    for (int j = 0; j < CG; j++) {
      const uint32_t col = g * CG + (uint32_t)j;
      live[j] = col < args.n_total;
      uint32_t m = 0, c = live[j] ? col : 0;
      if (c >= args.w[0].N && args.n_mats > 1) {
        c -= args.w[0].N;
        m = 1;
        if (c >= args.w[1].N && args.n_mats > 2) {
          c -= args.w[1].N;
          m = 2;
        }
      }
      Bp[j] = m == 0 ? args.w[0].B : (m == 1 ? args.w[1].B : args.w[2].B);
      Sp[j] = m == 0 ? args.w[0].scales : (m == 1 ? args.w[1].scales : args.w[2].scales);
      Zp[j] = m == 0 ? args.w[0].zp : (m == 1 ? args.w[1].zp : args.w[2].zp);
      mat[j] = m;
      cl[j] = c;
      base[j] = (uint64_t)c * nb;
    }
    float acc[CG];
#pragma unroll
    for (int j = 0; j < CG; j++) acc[j] = 0.f;
    for (uint32_t b0 = 0; b0 < nb; b0 += 8 * UNROLL) {
      uint32_t p[UNROLL][CG], z[UNROLL][CG];
      float s[UNROLL][CG];
#pragma unroll
      for (int u = 0; u < UNROLL; u++) {
        const uint32_t blk = b0 + (uint32_t)u * 8 + slot;
#pragma unroll
        for (int j = 0; j < CG; j++) {
          if (blk < nb && live[j]) {
            const uint64_t i = base[j] + blk;
            p[u][j] = __ldg(Bp[j] + i * 4 + word);
            s[u][j] = __ldg(Sp[j] + i);
            z[u][j] = (__ldg(Zp[j] + (i >> 3)) >> ((uint32_t)(i & 7) * 4)) & 15u;
          } else {
            p[u][j] = 0;
            s[u][j] = 0.f;
            z[u][j] = 0;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < UNROLL; u++) {
        const uint32_t blk = b0 + (uint32_t)u * 8 + slot;
        if (blk < nb) {
          const float4 a0 = *reinterpret_cast<const float4*>(sa + blk * 32 + word * 8);
          const float4 a1 = *reinterpret_cast<const float4*>(sa + blk * 32 + word * 8 + 4);
          const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const float asum = word == 0 ? sasum[blk] : 0.f;  // word 0 carries the zero-point term
#pragma unroll
          for (int j = 0; j < CG; j++) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < 8; e++) d = fmaf(av[e], nib_f(p[u][j], e), d);
            acc[j] = fmaf(s[u][j], d - (float)z[u][j] * asum, acc[j]);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < CG; j++) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    if (lane < CG) {
      // lane j writes column j of the group (static register choices per lane)
      float v = acc[0];
      bool lv = live[0];
      uint32_t m = mat[0], c = cl[0];
#pragma unroll
      for (int jj = 1; jj < CG; jj++)
        if (lane == jj) {
          v = acc[jj];
          lv = live[jj];
          m = mat[jj];
          c = cl[jj];
        }
      if (lv) {
        if (MODE == OUT_F32) {
          const uint32_t col = g * CG + (uint32_t)lane;
          if (args.epilogue == 1) {
            const float r = fmaxf(v, 0.f);
            v = r * r;
          } else if (args.epilogue == 2) {
            v = args.y[col] + v;
          }
          args.y[col] = v;
        } else {
          const __half h = __float2half_rn(v);
          if (m == 0) args.q_out[c] = h;
          else if (m == 1) args.k_row[c] = h;
          else args.v_row[c] = h;
        }
      }
    }
  }
}

int check_q4(const Q4& w, const char* who, const char* name) {
  using namespace nwd;
  if (!w.B || !w.scales || !w.zp) return fail(NWD_ERR_INVALID, "%s: null %s weights", who, name);
  if (reinterpret_cast<uintptr_t>(w.B) & 15u)
    return fail(NWD_ERR_INVALID, "%s: %s packed weights must be 16-byte aligned", who, name);
  return NWD_OK;
}

template <typename AT, int MODE>
int launch_gemv(const AT* a, const GemvArgs& args, void* stream, const char* who) {
  using namespace nwd;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st) return st;
  static bool smem_set[64][2] = {};
  const int slot = (int)sizeof(AT) == 2 ? 1 : 0;
  if (di.device < 64 && !smem_set[di.device][slot]) {
    cudaError_t e = cudaFuncSetAttribute(q4_gemv_kernel<AT, MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_bytes(MAX_BLOCKS));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(q4_gemv_kernel)");
    smem_set[di.device][slot] = true;
  }
  const uint32_t groups = (args.n_total + CG - 1) / CG;
  const uint32_t warps = GEMV_THREADS / 32;
  // enough warps for one column group each, at most 4 CTAs per SM (each CTA
  // reads A once from L2)
  uint64_t grid = (groups + warps - 1) / warps;
  grid = std::min<uint64_t>(grid, (uint64_t)di.sm_count * 4);
  q4_gemv_kernel<AT, MODE><<<(uint32_t)grid, GEMV_THREADS, smem_bytes(args.n_blocks),
                             (cudaStream_t)stream>>>(a, args);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
}

int check_shape(uint32_t K, uint32_t n_blocks, const char* who) {
  using namespace nwd;
  if (n_blocks == 0 || K != n_blocks * 32)
    return fail(NWD_ERR_INVALID, "%s: K (%u) must be 32 * n_blocks (%u)", who, K, n_blocks);
  if (n_blocks > MAX_BLOCKS)
    return fail(NWD_ERR_UNSUPPORTED, "%s: K %u exceeds %u", who, K, MAX_BLOCKS * 32);
  return NWD_OK;
}

}  // namespace

using namespace nwd;

extern "C" {

int nwd_q4_gemv(const float* a, const uint32_t* b, const float* scales, const uint32_t* zp,
                float* y, uint32_t K, uint32_t N, uint32_t n_blocks, uint32_t epilogue,
                void* stream) {
  const char* who = "nwd_q4_gemv";
  if (!a || !y) return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  int st = check_shape(K, n_blocks, who);
  if (st) return st;
  if (epilogue > 2) return fail(NWD_ERR_INVALID, "%s: epilogue %u (0, 1 or 2)", who, epilogue);
  GemvArgs args{};
  args.w[0] = Q4{b, scales, zp, N};
  if ((st = check_q4(args.w[0], who, "the"))) return st;
  if (N == 0) return ok();
  args.n_mats = 1;
  args.n_total = N;
  args.n_blocks = n_blocks;
  args.epilogue = epilogue;
  args.y = y;
  return launch_gemv<float, OUT_F32>(a, args, stream, who);
}

int nwd_q4_gemv_f16a(const uint16_t* a, const uint32_t* b, const float* scales,
                     const uint32_t* zp, float* y, uint32_t K, uint32_t N, uint32_t n_blocks,
                     uint32_t epilogue, void* stream) {
  const char* who = "nwd_q4_gemv_f16a";
  if (!a || !y) return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  int st = check_shape(K, n_blocks, who);
  if (st) return st;
  if (epilogue > 2) return fail(NWD_ERR_INVALID, "%s: epilogue %u (0, 1 or 2)", who, epilogue);
  GemvArgs args{};
  args.w[0] = Q4{b, scales, zp, N};
  if ((st = check_q4(args.w[0], who, "the"))) return st;
  if (N == 0) return ok();
  args.n_mats = 1;
  args.n_total = N;
  args.n_blocks = n_blocks;
  args.epilogue = epilogue;
  args.y = y;
  return launch_gemv<__half, OUT_F32>(reinterpret_cast<const __half*>(a), args, stream, who);
}

int nwd_q4_qkv_append(const float* h, const uint32_t* bq, const float* sq, const uint32_t* zq,
                      const uint32_t* bk, const float* sk, const uint32_t* zk, const uint32_t* bv,
                      const float* sv, const uint32_t* zv, uint16_t* q_out, uint16_t* k_cache,
                      uint16_t* v_cache, uint32_t seq, uint32_t cap, uint32_t K,
                      uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, void* stream) {
  const char* who = "nwd_q4_qkv_append";
  if (!h || !q_out || !k_cache || !v_cache) return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  if (seq >= cap) return fail(NWD_ERR_RANGE, "seq %u exceeds maxSeq %u", seq, cap);
  const uint32_t n_blocks = K / 32;
  int st = check_shape(K, n_blocks, who);
  if (st) return st;
  if (n_heads == 0 || n_kv_heads == 0 || head_dim == 0)
    return fail(NWD_ERR_INVALID, "%s: zero shape", who);
  const uint32_t row = n_kv_heads * head_dim;
  GemvArgs args{};
  args.w[0] = Q4{bq, sq, zq, n_heads * head_dim};
  args.w[1] = Q4{bk, sk, zk, row};
  args.w[2] = Q4{bv, sv, zv, row};
  if ((st = check_q4(args.w[0], who, "q")) || (st = check_q4(args.w[1], who, "k")) ||
      (st = check_q4(args.w[2], who, "v")))
    return st;
  args.n_mats = 3;
  args.n_total = args.w[0].N + 2 * row;
  args.n_blocks = n_blocks;
  args.q_out = reinterpret_cast<__half*>(q_out);
  args.k_row = reinterpret_cast<__half*>(k_cache) + (uint64_t)seq * row;
  args.v_row = reinterpret_cast<__half*>(v_cache) + (uint64_t)seq * row;
  return launch_gemv<float, OUT_QKV>(h, args, stream, who);
}

}  // extern "C"
