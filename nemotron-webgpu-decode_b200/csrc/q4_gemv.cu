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
// A warp takes a group of 4 columns and walks them in rows of 32 blocks, one
// block per lane: for each column a lane loads the block's 16 bytes, its scale
// and its zero point, so a row is 512 contiguous bytes per column.  The loads
// of the next two rows are in flight while a row is computed (software
// pipelining) and the grid is sized to what stays resident.  The lane's 32
// activations come from a shared-memory copy of A (float4s XOR-swizzled by
// block, so the 32 lanes of a warp, reading 32 different blocks, hit distinct
// banks) and serve all 4 columns.  A nibble q becomes the float 1 + q/16 with a
// shift and one logic operation (q placed in the top mantissa bits), so
//   sum_j a_j q_j = 16 * (sum_j a_j (1 + q_j/16) - sum_j a_j)
// and a block contributes scale * (16 * sum_j a_j f_j - (16 + zero) * sum_j a_j):
// three instructions per element, none through the special-function unit.
// f32 accumulation; lanes are reduced with shuffles at the end of the group.
#include <cuda_fp16.h>

#include <algorithm>

#include "nwd_common.h"

namespace {

constexpr int GEMV_THREADS = 128;      // 4 warps
constexpr int CG = 4;                  // columns per warp
constexpr int DEPTH = 2;               // rows of 32 blocks in flight ahead of the one computed
constexpr uint32_t MAX_BLOCKS = 1024;  // K <= 32768 (shared-memory copy of A)
constexpr size_t smem_bytes(uint32_t n_blocks) { return (size_t)n_blocks * 32 * sizeof(float); }

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

// 1 + q/16 for the 4-bit field q at bits [4E, 4E+4) of x: q moved to mantissa
// bits 19-22 under the exponent of 1.0 (exact).  The move is an integer
// multiply (by 2^s, or the high word of a multiply by 2^(32-s)), which runs on
// the FMA pipe; only the mask-and-merge uses the integer ALU, which has half
// the FMA pipe's throughput and would otherwise bound the kernel.
template <int E>
__device__ __forceinline__ float nib16(uint32_t x) {
  constexpr int sh = 19 - 4 * E;
  uint32_t t;
  if (sh >= 0) {
    asm("mul.lo.u32 %0, %1, %2;" : "=r"(t) : "r"(x), "n"(1u << (sh >= 0 ? sh : 0)));
  } else {
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(t) : "r"(x), "n"(1u << (sh < 0 ? 32 + sh : 0)));
  }
  return __uint_as_float((t & 0x00780000u) | 0x3F800000u);
}

// the 8 values of one weight word against 8 activations
__device__ __forceinline__ float word_dot(uint32_t x, const float* a, float d) {
  d = fmaf(a[0], nib16<0>(x), d);
  d = fmaf(a[1], nib16<1>(x), d);
  d = fmaf(a[2], nib16<2>(x), d);
  d = fmaf(a[3], nib16<3>(x), d);
  d = fmaf(a[4], nib16<4>(x), d);
  d = fmaf(a[5], nib16<5>(x), d);
  d = fmaf(a[6], nib16<6>(x), d);
  d = fmaf(a[7], nib16<7>(x), d);
  return d;
}

// shared-memory slot of float4 k (0..7) of block b
__device__ __forceinline__ uint32_t a_slot(uint32_t b, uint32_t k) { return b * 8 + (k ^ (b & 7)); }

template <typename AT>
__device__ __forceinline__ void stage_a(const AT* __restrict__ a, float* sa, uint32_t K);
template <>
__device__ __forceinline__ void stage_a<float>(const float* __restrict__ a, float* sa, uint32_t K) {
  // K is a multiple of 32: float4 copies, every load of a thread issued first
  const float4* a4 = reinterpret_cast<const float4*>(a);
  float4* s4 = reinterpret_cast<float4*>(sa);
  const uint32_t n4 = K / 4;
  for (uint32_t i0 = threadIdx.x; i0 < n4; i0 += 8 * GEMV_THREADS) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const uint32_t i = i0 + (uint32_t)u * GEMV_THREADS;
      if (i < n4) v[u] = __ldg(a4 + i);
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const uint32_t i = i0 + (uint32_t)u * GEMV_THREADS;
      if (i < n4) s4[a_slot(i >> 3, i & 7)] = v[u];
    }
  }
}
template <>
__device__ __forceinline__ void stage_a<__half>(const __half* __restrict__ a, float* sa,
                                                uint32_t K) {
  const uint2* a4 = reinterpret_cast<const uint2*>(a);  // 4 halves
  float4* s4 = reinterpret_cast<float4*>(sa);
  const uint32_t n4 = K / 4;
  for (uint32_t i0 = threadIdx.x; i0 < n4; i0 += 8 * GEMV_THREADS) {
    uint2 v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const uint32_t i = i0 + (uint32_t)u * GEMV_THREADS;
      if (i < n4) v[u] = __ldg(a4 + i);
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const uint32_t i = i0 + (uint32_t)u * GEMV_THREADS;
      if (i < n4) {
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v[u].x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v[u].y));
        s4[a_slot(i >> 3, i & 7)] = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
    }
  }
}

// One row (32 blocks, one per lane) of a column group: the lane's block of
// each of the 4 columns.
struct RowLoad {
  uint4 p[CG];
  float s[CG];
  uint32_t z[CG];
};

template <typename AT, int MODE>
__global__ void __launch_bounds__(GEMV_THREADS)
    q4_gemv_kernel(const AT* __restrict__ a, const GemvArgs args) {
  extern __shared__ float sa[];  // A as f32 [K], float4s swizzled per block
  const uint32_t nb = args.n_blocks;
  stage_a<AT>(a, sa, nb * 32);
  __syncthreads();
  const float4* sa4 = reinterpret_cast<const float4*>(sa);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n_groups = (args.n_total + CG - 1) / CG;
  const uint32_t n_warps = gridDim.x * (GEMV_THREADS / 32);
  const uint32_t rows = (nb + 31) / 32;
  for (uint32_t g = blockIdx.x * (GEMV_THREADS / 32) + warp; g < n_groups; g += n_warps) {
    // each column of the group: its matrix (selected without indexing the
    // parameter block) and its first block
    const uint4* Bp[CG];
    const float* Sp[CG];
    const uint32_t* Zp[CG];
    uint32_t mat[CG], cl[CG], base[CG];
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
      Bp[j] = reinterpret_cast<const uint4*>(m == 0 ? args.w[0].B
                                                    : (m == 1 ? args.w[1].B : args.w[2].B));
      Sp[j] = m == 0 ? args.w[0].scales : (m == 1 ? args.w[1].scales : args.w[2].scales);
      Zp[j] = m == 0 ? args.w[0].zp : (m == 1 ? args.w[1].zp : args.w[2].zp);
      mat[j] = m;
      cl[j] = c;
      base[j] = c * nb;  // < 2^32: N * n_blocks of one matrix fits (checked on the host)
    }
    auto load_row = [&](uint32_t r, RowLoad& L) {
      const uint32_t blk = r * 32 + (uint32_t)lane;
#pragma unroll
      for (int j = 0; j < CG; j++) {
        if (r < rows && blk < nb && live[j]) {
          const uint32_t i = base[j] + blk;
          L.p[j] = __ldg(Bp[j] + i);
          L.s[j] = __ldg(Sp[j] + i);
          L.z[j] = (__ldg(Zp[j] + (i >> 3)) >> ((i & 7) * 4)) & 15u;
        } else {
          L.p[j] = make_uint4(0, 0, 0, 0);
          L.s[j] = 0.f;
          L.z[j] = 0;
        }
      }
    };
    float acc[CG];
#pragma unroll
    for (int j = 0; j < CG; j++) acc[j] = 0.f;
    RowLoad buf[DEPTH + 1];
#pragma unroll
    for (int d = 0; d < DEPTH; d++) load_row((uint32_t)d, buf[d]);
    // rows r, r+1, .., r+DEPTH cycle through the buffers; the loop is unrolled
    // by DEPTH+1 so every buffer index is a compile-time constant
    for (uint32_t r0 = 0; r0 < rows; r0 += DEPTH + 1) {
#pragma unroll
      for (int d = 0; d <= DEPTH; d++) {
        const uint32_t r = r0 + (uint32_t)d;
        load_row(r + DEPTH, buf[(d + DEPTH) % (DEPTH + 1)]);
        const RowLoad& L = buf[d];
        const uint32_t blk = r * 32 + (uint32_t)lane;
        if (r < rows && blk < nb) {
          float av[32];
#pragma unroll
          for (int k = 0; k < 8; k++) {
            const float4 v = sa4[a_slot(blk, (uint32_t)k)];
            av[4 * k] = v.x;
            av[4 * k + 1] = v.y;
            av[4 * k + 2] = v.z;
            av[4 * k + 3] = v.w;
          }
          float t8[8];
#pragma unroll
          for (int k = 0; k < 8; k++) t8[k] = (av[4 * k] + av[4 * k + 1]) + (av[4 * k + 2] + av[4 * k + 3]);
          const float asum = ((t8[0] + t8[1]) + (t8[2] + t8[3])) + ((t8[4] + t8[5]) + (t8[6] + t8[7]));
#pragma unroll
          for (int j = 0; j < CG; j++) {
            float d0 = word_dot(L.p[j].x, av, 0.f);
            float d1 = word_dot(L.p[j].y, av + 8, 0.f);
            d0 = word_dot(L.p[j].z, av + 16, d0);
            d1 = word_dot(L.p[j].w, av + 24, d1);
            const float dsum = d0 + d1;  // sum_j a_j (1 + q_j/16)
            acc[j] = fmaf(L.s[j], fmaf(16.f, dsum, -(16.f + (float)L.z[j]) * asum), acc[j]);
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
            const float rr = fmaxf(v, 0.f);
            v = rr * rr;
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

int check_q4(const Q4& w, uint32_t n_blocks, const char* who, const char* name) {
  using namespace nwd;
  if (!w.B || !w.scales || !w.zp) return fail(NWD_ERR_INVALID, "%s: null %s weights", who, name);
  if ((uint64_t)w.N * n_blocks >= (1ull << 32))
    return fail(NWD_ERR_UNSUPPORTED, "%s: %s has 2^32 blocks or more", who, name);
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
  // one column group per warp where they fit; otherwise as many CTAs as stay
  // resident, each walking several groups
  // resident CTAs per SM for this A size, cached per device, kernel and K (a
  // few K values per process: the engine's projections use two)
  struct Occ {
    uint32_t nb;
    int per_sm;
  };
  static Occ cache[64][2][2][4] = {};
  const int mode_slot = MODE == OUT_F32 ? 0 : 1;
  Occ* line = cache[di.device < 64 ? di.device : 0][slot][mode_slot];
  int per_sm = 0;
  for (int i = 0; i < 4 && !per_sm; i++)
    if (line[i].nb == args.n_blocks) per_sm = line[i].per_sm;
  if (!per_sm) {
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &n, q4_gemv_kernel<AT, MODE>, GEMV_THREADS, smem_bytes(args.n_blocks));
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    per_sm = std::max(1, n);
    for (int i = 3; i > 0; i--) line[i] = line[i - 1];
    line[0] = Occ{args.n_blocks, per_sm};
  }
  const uint32_t groups = (args.n_total + CG - 1) / CG;
  const uint32_t warps = GEMV_THREADS / 32;
  uint64_t grid = (groups + warps - 1) / warps;
  grid = std::min<uint64_t>(grid, (uint64_t)di.sm_count * (uint64_t)per_sm);
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
  if ((st = check_q4(args.w[0], n_blocks, who, "the"))) return st;
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
  if ((st = check_q4(args.w[0], n_blocks, who, "the"))) return st;
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
  if ((st = check_q4(args.w[0], n_blocks, who, "q")) || (st = check_q4(args.w[1], n_blocks, who, "k")) ||
      (st = check_q4(args.w[2], n_blocks, who, "v")))
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
