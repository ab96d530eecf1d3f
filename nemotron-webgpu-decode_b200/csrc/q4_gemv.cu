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
// A column's weights are read once (20.5 bytes per 32 elements); the kernel is
// built so that every byte a CTA needs is in flight at once and the inner loop
// is as short as possible.  The products run on the tensor cores (mma.sync
// m16n8k16, f16 in, f32 accumulate):
//   * A (16 x 16) = the weights of 16 output columns: lane (g, t) = (lane / 4,
//     lane % 4) takes word t of the block of columns g and g + 8 and turns its
//     8 nibbles into exact fp16 integers q - zero: a masked OR against an fp16
//     exponent per nibble pair (1024 + q for the nibbles at bits 0-3 of each
//     half, 64 + q for those at bits 4-7, where the fp16 step is 1/16), then
//     one half2 subtract of (1024 + zero) or (64 + zero).  The reduction index
//     of the MMA is permuted so these pairs are exactly the A fragment's: in
//     step s of a block, k = (2t, 2t+1) holds elements (8t+2s, 8t+2s+4) and
//     k = (2t+8, 2t+9) holds (8t+2s+1, 8t+2s+5).
//   * B (16 x 8) = the activations in the same permuted order: column 0 =
//     fp16(a), column 1 = fp16(a - fp16(a)), the rest zero, so a * (q - zero)
//     keeps ~22 bits and the sum is f32.  Lanes 0-7 supply them.
//   * D row r = output column r of the tile: column 0 its dot with fp16(a),
//     column 1 with the remainder.  Per block both times the block scale go
//     into two f32 accumulators.
// A CTA owns 16 columns.  Its 256 threads first put the tile's constant
// inputs in flight at once with cp.async, lane-dense (a warp copies two whole
// columns): the zero point words, then the weights and scales.  As soon as the
// zero point words are in, they build a table of the fp16 (1024 + zero,
// 64 + zero) pairs per (column, block).  All of this happens before the kernel
// waits for the previous kernel in the stream (programmatic dependent launch),
// so in a layer it overlaps the attention kernel or the previous GEMV.  After
// the wait they load the activations (through L2) and write the B fragments
// into shared memory, then wait for the weights; the 8 warps split the blocks
// (K) in eighths, and the loop body is shared-memory loads, the nibble
// unpacking, two independent MMAs (one per K-step) and four add + FMA pairs.
// The 8 warps' sums meet in shared memory in a fixed order (deterministic).
#include <cuda_fp16.h>

#include <algorithm>

#include "nwd_common.h"

namespace {

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_THREADS = GEMV_WARPS * 32;
constexpr uint32_t TILE_N = 16;       // output columns per CTA (the MMA's M)
constexpr uint32_t MAX_BLOCKS = 440;  // K <= 14080 (a tile's shared memory stays under 227 KB)

// Shared memory of a CTA (all offsets multiples of 16 bytes):
//   W    [16][cs][16 B]  the columns' packed weights; the column stride is an
//                        odd number of blocks, so the 8 columns of a word read
//                        hit distinct banks
//   S    [nb][8] float2  the block scales of columns (g, g + 8)
//   A    [nb][128 B]     per block: the B fragments (uint4 [row][t])
//   ZT   [nb][8] uint2   the fp16 pair (1024 + zero, 64 + zero) of columns
//                        (g, g + 8)
//   ZC   [16][zc]        each column's zero point words as copied
//   COLS [16]            where each column's data starts
//   ZERO 16 bytes        the B fragment of lanes 8-31
//   RED  [warp][16] f32  the warps' sums
struct ColSm {
  const uint8_t* w;   // packed weights of the column
  const float* s;     // its scales
  const uint32_t* z;  // the zero point array of its matrix
  uint32_t c;         // column within its matrix
  uint32_t live;
  uint32_t pad[4];
};
static_assert(sizeof(ColSm) == 48, "ColSm size");

__host__ __device__ constexpr uint32_t col_stride_blocks(uint32_t nb) { return nb | 1u; }
// words spanned by a column's nb nibbles, wherever they start
__host__ __device__ constexpr uint32_t zc_words(uint32_t nb) { return nb / 8 + 2; }
__host__ __device__ constexpr size_t round16(size_t x) { return (x + 15) / 16 * 16; }
__host__ __device__ constexpr size_t off_s(uint32_t nb) { return (size_t)TILE_N * col_stride_blocks(nb) * 16; }
__host__ __device__ constexpr size_t off_a(uint32_t nb) { return off_s(nb) + (size_t)nb * 64; }
__host__ __device__ constexpr size_t off_zt(uint32_t nb) { return off_a(nb) + (size_t)nb * 128; }
__host__ __device__ constexpr size_t off_zc(uint32_t nb) { return off_zt(nb) + (size_t)nb * 64; }
__host__ __device__ constexpr size_t off_cols(uint32_t nb) {
  return off_zc(nb) + round16((size_t)TILE_N * zc_words(nb) * 4);
}
__host__ __device__ constexpr size_t off_zero(uint32_t nb) { return off_cols(nb) + TILE_N * sizeof(ColSm); }
__host__ __device__ constexpr size_t off_red(uint32_t nb) { return off_zero(nb) + 16; }
__host__ __device__ constexpr size_t smem_bytes(uint32_t nb) {
  return off_red(nb) + (size_t)GEMV_WARPS * TILE_N * 4;
}
static_assert(smem_bytes(MAX_BLOCKS) <= 227 * 1024, "tile shared memory");

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

__device__ __forceinline__ uint32_t lop3_or_and(uint32_t x, uint32_t mask, uint32_t magic) {
  uint32_t r;  // (x & mask) | magic
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(mask), "r"(magic));
  return r;
}
__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
  return h2_bits(__halves2half2(lo, hi));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1,
                                         const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most n (0 or 1) of this thread's copy groups are still in flight
__device__ __forceinline__ void cp_async_wait_pending(uint32_t n) {
  if (n == 0) asm volatile("cp.async.wait_group 0;" ::: "memory");
  else asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// a column of the tile resolved to its matrix (selected without indexing the
// parameter block) and local column
__device__ __forceinline__ ColSm col_ref(const GemvArgs& args, uint32_t col) {
  ColSm r{};
  r.live = col < args.n_total;
  uint32_t m = 0, c = r.live ? col : 0;
  if (c >= args.w[0].N && args.n_mats > 1) {
    c -= args.w[0].N;
    m = 1;
    if (c >= args.w[1].N && args.n_mats > 2) {
      c -= args.w[1].N;
      m = 2;
    }
  }
  const uint32_t* B = m == 0 ? args.w[0].B : (m == 1 ? args.w[1].B : args.w[2].B);
  const float* S = m == 0 ? args.w[0].scales : (m == 1 ? args.w[1].scales : args.w[2].scales);
  r.z = m == 0 ? args.w[0].zp : (m == 1 ? args.w[1].zp : args.w[2].zp);
  r.w = reinterpret_cast<const uint8_t*>(B) + (size_t)c * args.n_blocks * 16;
  r.s = S + (size_t)c * args.n_blocks;
  r.c = c;
  return r;
}

// Eight consecutive activations from global memory, through L2 (another
// kernel wrote them).
template <typename AT>
__device__ __forceinline__ void load_act(const AT* p, float (&x)[8]);
template <>
__device__ __forceinline__ void load_act<float>(const float* p, float (&x)[8]) {
  const float4 u = __ldcg(reinterpret_cast<const float4*>(p));
  const float4 v = __ldcg(reinterpret_cast<const float4*>(p) + 1);
  x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w;
  x[4] = v.x; x[5] = v.y; x[6] = v.z; x[7] = v.w;
}
template <>
__device__ __forceinline__ void load_act<__half>(const __half* p, float (&x)[8]) {
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const __half2 h = bits_h2(w[j]);
    x[2 * j] = __low2float(h);
    x[2 * j + 1] = __high2float(h);
  }
}

template <typename AT, int MODE>
__global__ void __launch_bounds__(GEMV_THREADS, 4)
    q4_gemv_kernel(const AT* __restrict__ a, const GemvArgs args) {
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t nb = args.n_blocks, cs = col_stride_blocks(nb), zc = zc_words(nb);
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  ColSm* cols = reinterpret_cast<ColSm*>(smem + off_cols(nb));
  float* red = reinterpret_cast<float*>(smem + off_red(nb));
  const uint32_t* zcw = reinterpret_cast<const uint32_t*>(smem + off_zc(nb));

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = lane >> 2, t = lane & 3;
  const uint32_t tile = blockIdx.x;

  nwd::pdl_trigger();  // the next kernel in the stream may start its own weight copies
  if (threadIdx.x < TILE_N) cols[threadIdx.x] = col_ref(args, tile * TILE_N + threadIdx.x);
  if (threadIdx.x == TILE_N)
    *reinterpret_cast<uint4*>(smem + off_zero(nb)) = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();

  // ---- the constant inputs, all in flight at once: group 0 = the zero point
  // words, group 1 = the weights and scales (warp w: columns w and w + 8, one
  // block per lane)
#pragma unroll
  for (uint32_t h = 0; h < 2; h++) {
    const uint32_t j = warp + 8 * h;
    const ColSm cr = cols[j];
    if (!cr.live) continue;
    const uint32_t w0 = (cr.c * nb) >> 3, n_w = ((cr.c * nb + nb - 1) >> 3) - w0 + 1;
    for (uint32_t k = lane; k < n_w; k += 32)
      cp_async4(sbase + (uint32_t)off_zc(nb) + (j * zc + k) * 4, cr.z + w0 + k);
  }
  cp_async_commit();
#pragma unroll
  for (uint32_t h = 0; h < 2; h++) {
    const uint32_t j = warp + 8 * h;
    const ColSm cr = cols[j];
    if (!cr.live) continue;
    const uint32_t w_dst = sbase + j * cs * 16;
    const uint32_t s_dst = sbase + (uint32_t)off_s(nb) + ((j & 7) * 2 + (j >> 3)) * 4;
    for (uint32_t b = lane; b < nb; b += 32) {
      cp_async16(w_dst + b * 16, cr.w + (size_t)b * 16);
      cp_async4(s_dst + b * 64, cr.s + b);
    }
  }
  cp_async_commit();

  // ---- the zero point table, (block, column) -> fp16 pair (1024 + z, 64 + z),
  // as soon as the words are in (the weights may still be arriving)
  cp_async_wait_pending(1);
  __syncthreads();
  {
    uint32_t* zt = reinterpret_cast<uint32_t*>(smem + off_zt(nb));
    const uint32_t j = threadIdx.x & 15;
    const uint32_t c = cols[j].c, live = cols[j].live, i0 = c * nb;
    for (uint32_t b = threadIdx.x >> 4; b < nb; b += GEMV_THREADS / 16) {
      const uint32_t i = i0 + b;
      const uint32_t z = live ? (zcw[j * zc + (i >> 3) - (i0 >> 3)] >> ((i & 7) * 4)) & 15u : 0u;
      zt[(b * 8 + (j & 7)) * 2 + (j >> 3)] = (0x6400u | z) | ((0x5400u | (z << 4)) << 16);
    }
  }

  // everything above reads only the weights; the activations (and the outputs)
  // belong to the kernels around this one
  nwd::pdl_wait();

  // ---- B fragments straight from the activations in global memory: thread
  // (block, t) loads elements [8t, 8t + 8) and writes uint4 [row][t] of its
  // block; two items' loads are in flight before either is converted
  for (uint32_t item = threadIdx.x; item < nb * 4; item += 2 * GEMV_THREADS) {
    float x[2][8];
    const bool second = item + GEMV_THREADS < nb * 4;
#pragma unroll
    for (uint32_t u = 0; u < 2; u++) {
      const uint32_t it = item + u * GEMV_THREADS;
      if (u == 0 || second) load_act<AT>(a + (size_t)(it >> 2) * 32 + (it & 3) * 8, x[u]);
    }
#pragma unroll
    for (uint32_t u = 0; u < 2; u++) {
      if (u == 1 && !second) break;
      const uint32_t it = item + u * GEMV_THREADS, bb = it >> 2, tt = it & 3;
      __half hi[8], lo[8];
#pragma unroll
      for (int k = 0; k < 8; k++) {
        hi[k] = __float2half_rn(x[u][k]);
        // fp16 activations are exact in the head: the remainder row is zero
        lo[k] = sizeof(AT) == 2 ? __float2half_rn(0.f) : __float2half_rn(x[u][k] - __half2float(hi[k]));
      }
      // step s: {(e, e+4), (e+1, e+5)} with e = 2s
      uint4* blk = reinterpret_cast<uint4*>(smem + off_a(nb) + (size_t)bb * 128);
      blk[tt] = make_uint4(pack_h2(hi[0], hi[4]), pack_h2(hi[1], hi[5]), pack_h2(hi[2], hi[6]),
                           pack_h2(hi[3], hi[7]));
      blk[4 + tt] = make_uint4(pack_h2(lo[0], lo[4]), pack_h2(lo[1], lo[5]), pack_h2(lo[2], lo[6]),
                               pack_h2(lo[3], lo[7]));
    }
  }
  cp_async_wait_pending(0);
  __syncthreads();

  // ---- this warp's eighth of the blocks ----
  const uint32_t b_lo = nb * warp / GEMV_WARPS, b_hi = nb * (warp + 1) / GEMV_WARPS;
  const uint32_t* ws = reinterpret_cast<const uint32_t*>(smem);
  const float2* ss = reinterpret_cast<const float2*>(smem + off_s(nb));
  const uint2* zt2 = reinterpret_cast<const uint2*>(smem + off_zt(nb));
  // lanes 0-7 read their B fragment of each block, lanes 8-31 a zero one
  const uint8_t* fbase = lane < 8 ? smem + off_a(nb) + lane * 16 : smem + off_zero(nb);
  const uint32_t fstride = lane < 8 ? 128u : 0u;
  float accH0 = 0.f, accL0 = 0.f, accH1 = 0.f, accL1 = 0.f;  // columns g and g + 8
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};
  // the two K-steps of a block are independent MMAs (no accumulate chain
  // between them), so several blocks' MMAs are in flight at once
#pragma unroll 4
  for (uint32_t b = b_lo; b < b_hi; b++) {
    const uint32_t x0 = ws[(g * cs + b) * 4 + t];
    const uint32_t x1 = ws[((g + 8) * cs + b) * 4 + t];
    const uint2 zu = zt2[b * 8 + g];
    const uint4 f = *reinterpret_cast<const uint4*>(fbase + b * fstride);
    const float2 sc = ss[b * 8 + g];
    const __half2 zl0 = __low2half2(bits_h2(zu.x)), zh0 = __high2half2(bits_h2(zu.x));
    const __half2 zl1 = __low2half2(bits_h2(zu.y)), zh1 = __high2half2(bits_h2(zu.y));
    const uint32_t x0s = x0 >> 8, x1s = x1 >> 8;
    float d[4], e[4];
    mma16816(d, h2_bits(__hsub2(bits_h2(lop3_or_and(x0, 0x000F000Fu, 0x64006400u)), zl0)),
             h2_bits(__hsub2(bits_h2(lop3_or_and(x1, 0x000F000Fu, 0x64006400u)), zl1)),
             h2_bits(__hsub2(bits_h2(lop3_or_and(x0, 0x00F000F0u, 0x54005400u)), zh0)),
             h2_bits(__hsub2(bits_h2(lop3_or_and(x1, 0x00F000F0u, 0x54005400u)), zh1)), f.x, f.y,
             zero4);
    mma16816(e, h2_bits(__hsub2(bits_h2(lop3_or_and(x0s, 0x000F000Fu, 0x64006400u)), zl0)),
             h2_bits(__hsub2(bits_h2(lop3_or_and(x1s, 0x000F000Fu, 0x64006400u)), zl1)),
             h2_bits(__hsub2(bits_h2(lop3_or_and(x0s, 0x00F000F0u, 0x54005400u)), zh0)),
             h2_bits(__hsub2(bits_h2(lop3_or_and(x1s, 0x00F000F0u, 0x54005400u)), zh1)), f.z, f.w,
             zero4);
    accH0 = fmaf(sc.x, d[0] + e[0], accH0);
    accL0 = fmaf(sc.x, d[1] + e[1], accL0);
    accH1 = fmaf(sc.y, d[2] + e[2], accH1);
    accL1 = fmaf(sc.y, d[3] + e[3], accL1);
  }
  // lanes t == 0 hold columns g and g + 8 (D columns 0 and 1; the rest are zero)
  if (t == 0) {
    red[warp * TILE_N + g] = accH0 + accL0;
    red[warp * TILE_N + g + 8] = accH1 + accL1;
  }
  __syncthreads();
  if (threadIdx.x < TILE_N) {
    const uint32_t j = threadIdx.x;
    float v = red[j];
#pragma unroll
    for (int w = 1; w < GEMV_WARPS; w++) v += red[w * TILE_N + j];
    const ColSm& cr = cols[j];
    if (cr.live) {
      const uint32_t col = tile * TILE_N + j;
      if (MODE == OUT_F32) {
        if (args.epilogue == 1) {
          const float rr = fmaxf(v, 0.f);
          v = rr * rr;
        } else if (args.epilogue == 2) {
          v = args.y[col] + v;
        }
        args.y[col] = v;
      } else {
        const __half h = __float2half_rn(v);
        if (col < args.w[0].N) args.q_out[cr.c] = h;
        else if (col < args.w[0].N + args.w[1].N) args.k_row[cr.c] = h;
        else args.v_row[cr.c] = h;
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
  static bool smem_set[64] = {};  // per instantiation (A type, output mode) and device
  if (di.device < 64 && !smem_set[di.device]) {
    cudaError_t e = cudaFuncSetAttribute(q4_gemv_kernel<AT, MODE>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_bytes(MAX_BLOCKS));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(q4_gemv_kernel)");
    smem_set[di.device] = true;
  }
  // one CTA per 16-column tile (the hardware schedules them as SMs free up)
  const uint64_t grid = (args.n_total + TILE_N - 1) / TILE_N;
  if (grid > 0x7fffffffull) return fail(NWD_ERR_UNSUPPORTED, "%s: too many columns", who);
  cudaError_t e = launch_pdl(q4_gemv_kernel<AT, MODE>, dim3((uint32_t)grid), dim3(GEMV_THREADS),
                             smem_bytes(args.n_blocks), (cudaStream_t)stream, a, args);
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
}

int check_shape(const void* a, uint32_t K, uint32_t n_blocks, const char* who) {
  using namespace nwd;
  if (reinterpret_cast<uintptr_t>(a) & 15u)
    return fail(NWD_ERR_INVALID, "%s: the activation vector must be 16-byte aligned", who);
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
  int st = check_shape(a, K, n_blocks, who);
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
  int st = check_shape(a, K, n_blocks, who);
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
  int st = check_shape(h, K, n_blocks, who);
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
