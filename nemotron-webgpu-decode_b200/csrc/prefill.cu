// Causal chunked prefill attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory).
//
// The reference has no prefill: it feeds the prompt one decode step per token
// (engine/runtime.js:640-643), so prompt token i of a chunk that starts at
// cache row start_pos attends rows 0 .. start_pos + i.  This kernel computes
// exactly that for a whole chunk at once, as a dense contraction.
//
// One CTA per (sequence, query head, 128-query tile), 8 warps:
//   warp 0      TMA producer: the Q tile once, then K and V tiles of 128 rows
//               into 2-stage rings with separate barriers (K(j) is free once
//               S(j) is done, long before V(j)); each 128-row tile as two
//               64-column chunks, 128-byte swizzle: the canonical K-major
//               layout of the tcgen05 shared-memory descriptors.
//   warp 1      MMA issuer (one thread): S(j) = Q K(j)^T into TMEM score
//               buffer j & 1 (M=128 queries, N=128 keys, K=128 = 8 MMAs of
//               K=16), issued one block ahead so it overlaps the softmax of
//               block j-1; then, once P(j) is in TMEM, O += P V into TMEM
//               columns [256,384) with A = P read from tensor memory and
//               B = V an MN-major shared-memory operand.  P is an fp16 head
//               and an fp16 remainder (16 MMAs): one fp16 rounding of P would
//               exceed the parity tolerance on outputs near zero.
//               tcgen05.commit signals S ready, K free, V free and PV done.
//   warp 2      TMEM allocation (512 columns) and release.
//   warps 4-7   softmax: thread r owns query row r (TMEM lane r): loads its
//               128 scores with tcgen05.ld, applies the causal mask, updates
//               the running max with lazy rescaling (O is rescaled in TMEM
//               only when a row's max grows by more than 2^8), and writes
//               P = 2^(s - m) over its own scores: fp16 pairs, head in
//               columns [0,64) of the buffer and remainder in [64,128).  P(j)
//               needs no wait on PV(j-1), which reads the other buffer; the
//               MMAs of one thread run in issue order, so S(j+2) overwrites
//               P(j) only after PV(j) has read it.  At the end the softmax
//               warps divide O by the row sum and store it.
// All waits are bounded; on expiry the kernel records
// NWD_DEVERR_PIPE_TIMEOUT, lets its in-flight copies and MMAs land, frees its
// TMEM and returns.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

#include "nwd_common.h"
#include "ptx.cuh"

namespace {

using namespace nwd::ptx;
using nwd::WsHeader;

constexpr int PHD = 128;          // head_dim
constexpr int BM = 128;           // queries per tile
constexpr int BN = 128;           // keys per block
constexpr int PTHR = 256;         // 8 warps
constexpr int CHUNK = 128 * 128;  // 128 rows x 64 fp16 (one 64-column chunk): 16 KiB
constexpr int TILE = 2 * CHUNK;   // 128 x 128 fp16: 32 KiB
constexpr int KV_ST = 2;          // K/V ring stages

constexpr int O_Q = 0;
constexpr int O_K = O_Q + TILE;
constexpr int O_V = O_K + KV_ST * TILE;
constexpr int O_BAR = O_V + KV_ST * TILE;
// barriers: q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_full,
// pv_done, drain
constexpr int B_QFULL = 0, B_KFULL = 1, B_KEMPTY = 3, B_VFULL = 5, B_VEMPTY = 7, B_SFULL = 9,
              B_PFULL = 11, B_PVDONE = 12, B_DRAIN = 13, NBAR = 14;
constexpr int O_MISC = O_BAR + NBAR * 8;  // tmem base (u32), abort flag (i32)
constexpr int P_SMEM_USED = O_MISC + 16;
constexpr int P_SMEM_BYTES = P_SMEM_USED + 1024;
static_assert(P_SMEM_BYTES <= 227 * 1024, "shared memory");

constexpr uint32_t TMEM_COLS = 512;  // S0 [0,128), S1 [128,256), O [256,384)
constexpr float RESCALE_LOG2 = 8.f;

struct PParams {
  __half* o;
  const int64_t* row_offset;
  uint8_t* ws;
  uint64_t pool_rows;
  uint32_t batch, n_q, start_pos, n_heads, n_kv, group, q_tiles;
  float scale_log2;
};

// ---- tcgen05 wrappers ----
// Shared-memory matrix descriptor: start address, leading / stride byte
// offsets (all >> 4), descriptor version 1 (bits 46-47), 128-byte swizzle
// (layout type 2 in bits 61-63).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// A from tensor memory ([a] is a TMEM address: row i in lane i, fp16 pairs
// along the columns), B from shared memory.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), fp16 A
// and B (bits 7-12 = 0), A K-major, B K-major or MN-major (bit 16), N >> 3 in
// bits 17-22, M >> 4 in bits 24-28.
constexpr uint32_t idesc_f16(uint32_t m, uint32_t n, bool b_mn_major) {
  return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}
constexpr uint32_t IDESC_S = idesc_f16(BM, BN, false);
constexpr uint32_t IDESC_O = idesc_f16(BM, PHD, true);

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// 32 lanes x 32 columns of fp32: thread t of the warp gets row (lane base + t)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(PTHR, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                   const __grid_constant__ CUtensorMap tmv, const __grid_constant__ PParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sb = smem_u32(smem);
  const uint32_t bar = sb + O_BAR;  // + 8 * index
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + O_MISC);
  volatile int32_t* abort_flag = reinterpret_cast<int32_t*>(smem + O_MISC + 4);
  WsHeader* wsh = reinterpret_cast<WsHeader*>(p.ws);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // heavy tiles (late queries see the most keys) get the lowest block indices
  const uint32_t bh_count = p.batch * p.n_heads;
  const uint32_t tile_rank = blockIdx.x / bh_count, bh = blockIdx.x % bh_count;
  const uint32_t qt = p.q_tiles - 1 - tile_rank;
  const uint32_t b = bh / p.n_heads, h = bh % p.n_heads, hkv = h / p.group;
  const uint32_t q0 = qt * BM;
  const uint32_t nq_valid = min((uint32_t)BM, p.n_q - q0);
  const uint32_t last_key = p.start_pos + q0 + nq_valid - 1;  // causal horizon of the tile
  const uint32_t nblk = last_key / BN + 1;

  if (tid == 0) {
    *abort_flag = 0;
    mbar_init(bar + 8 * B_QFULL, 1);
    for (int s = 0; s < KV_ST; s++) {
      mbar_init(bar + 8 * (B_KFULL + s), 1);
      mbar_init(bar + 8 * (B_KEMPTY + s), 1);
      mbar_init(bar + 8 * (B_VFULL + s), 1);
      mbar_init(bar + 8 * (B_VEMPTY + s), 1);
      mbar_init(bar + 8 * (B_SFULL + s), 1);
    }
    mbar_init(bar + 8 * B_PFULL, BM);
    mbar_init(bar + 8 * B_PVDONE, 1);
    mbar_init(bar + 8 * B_DRAIN, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_o = tmem + 256;  // score buffers at tmem + 0 and tmem + 128

  if (warp == 0) {
    // ======================= TMA producer =======================
    const uint64_t pol_q = evict_first_policy(), pol_kv = evict_last_policy();
    const int kv_row0 = (int)p.row_offset[b];
    uint32_t kissued[KV_ST] = {0, 0}, vissued[KV_ST] = {0, 0};
    bool q_issued = false, ok = true;
    if (lane == 0) {
      const uint32_t fb = bar + 8 * B_QFULL;
      mbar_arrive_tx(fb, TILE);
      const int qrow = (int)(b * p.n_q + q0);
      tma_load_4d(sb + O_Q, &tmq, fb, 0, 0, (int)h, qrow, pol_q);
      tma_load_4d(sb + O_Q + CHUNK, &tmq, fb, 0, 1, (int)h, qrow, pol_q);
    }
    q_issued = true;
    __syncwarp();
    for (uint32_t j = 0; j < nblk && ok; j++) {
      const uint32_t st = j & 1, par = ((j >> 1) & 1) ^ 1;
      const int row = kv_row0 + (int)(j * BN);
      // K(j): its stage is free once S(j-2) has completed
      if (!warp_wait(bar + 8 * (B_KEMPTY + st), par, abort_flag, &wsh->error)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        const uint32_t fb = bar + 8 * (B_KFULL + st);
        mbar_arrive_tx(fb, TILE);
        tma_load_4d(sb + O_K + st * TILE, &tmk, fb, 0, 0, (int)hkv, row, pol_kv);
        tma_load_4d(sb + O_K + st * TILE + CHUNK, &tmk, fb, 0, 1, (int)hkv, row, pol_kv);
      }
      __syncwarp();
      kissued[st]++;
      // V(j): its stage is free once PV(j-2) has completed
      if (!warp_wait(bar + 8 * (B_VEMPTY + st), par, abort_flag, &wsh->error)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        const uint32_t fb = bar + 8 * (B_VFULL + st);
        mbar_arrive_tx(fb, TILE);
        tma_load_4d(sb + O_V + st * TILE, &tmv, fb, 0, 0, (int)hkv, row, pol_kv);
        tma_load_4d(sb + O_V + st * TILE + CHUNK, &tmv, fb, 0, 1, (int)hkv, row, pol_kv);
      }
      __syncwarp();
      vissued[st]++;
    }
    if (!ok) {
      // let this CTA's copies in flight land before the CTA can exit
      const uint64_t t0 = globaltimer();
      if (q_issued)
        while (!mbar_try_wait(bar + 8 * B_QFULL, 0) && globaltimer() - t0 < WAIT_LIMIT_NS) {
        }
      for (int s = 0; s < KV_ST; s++) {
        if (kissued[s])
          while (!mbar_try_wait(bar + 8 * (B_KFULL + s), (kissued[s] - 1) & 1) &&
                 globaltimer() - t0 < WAIT_LIMIT_NS) {
          }
        if (vissued[s])
          while (!mbar_try_wait(bar + 8 * (B_VFULL + s), (vissued[s] - 1) & 1) &&
                 globaltimer() - t0 < WAIT_LIMIT_NS) {
          }
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    bool ok = warp_wait(bar + 8 * B_QFULL, 0, abort_flag, &wsh->error);
    // S(i) = Q K(i)^T into score buffer i & 1: 8 K-steps of 16 over head_dim
    auto issue_s = [&](uint32_t i) -> bool {
      const uint32_t st = i & 1;
      if (!warp_wait(bar + 8 * (B_KFULL + st), (i >> 1) & 1, abort_flag, &wsh->error)) return false;
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int k = 0; k < 8; k++) {
          const uint32_t off = (uint32_t)(k >> 2) * CHUNK + (uint32_t)(k & 3) * 32;
          umma(tmem + st * 128, sdesc(sb + O_Q + off, 16, 1024),
               sdesc(sb + O_K + st * TILE + off, 16, 1024), IDESC_S, k > 0);
        }
        umma_commit(bar + 8 * (B_KEMPTY + st));
        umma_commit(bar + 8 * (B_SFULL + st));
      }
      __syncwarp();
      return true;
    };
    if (ok) ok = issue_s(0);
    for (uint32_t j = 0; j < nblk && ok; j++) {
      // one block ahead: S(j+1) overlaps the softmax of block j.  Its score
      // buffer was last read by the softmax of block j-1, which finished
      // before p_full(j-1) released PV(j-1) in the previous iteration.
      if (j + 1 < nblk && !issue_s(j + 1)) {
        ok = false;
        break;
      }
      if (!warp_wait(bar + 8 * B_PFULL, j & 1, abort_flag, &wsh->error) ||
          !warp_wait(bar + 8 * (B_VFULL + (j & 1)), (j >> 1) & 1, abort_flag, &wsh->error)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        // O += P V: 8 K-steps of 16 keys (8 TMEM columns of fp16 pairs)
        // for the P head, then 8 for the P remainder; V MN-major (head_dim
        // contiguous): its 64-column chunks are LBO = 16 KiB apart
        const uint32_t st = j & 1;
        const uint32_t tmem_p = tmem + st * 128;
#pragma unroll
        for (int k = 0; k < 16; k++) {
          const uint32_t kk = (uint32_t)(k & 7);
          umma_ts(tmem_o, tmem_p + (k < 8 ? 0u : 64u) + kk * 8u,
                  sdesc(sb + O_V + st * TILE + kk * 16 * 128, CHUNK, 1024), IDESC_O,
                  (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(bar + 8 * (B_VEMPTY + st));
        umma_commit(bar + 8 * B_PVDONE);
      }
      __syncwarp();
    }
    // every MMA this thread issued has completed before TMEM is released
    if (lane == 0) umma_commit(bar + 8 * B_DRAIN);
    __syncwarp();
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar + 8 * B_DRAIN, 0) && globaltimer() - t0 < WAIT_LIMIT_NS) {
    }
  } else if (warp >= 4) {
    // ======================= softmax / epilogue =======================
    const uint32_t r = (uint32_t)(tid - 128);          // query row = TMEM lane
    const uint32_t lane_base = (uint32_t)(warp - 4) * 32u << 16;
    const uint32_t qpos = p.start_pos + q0 + r;          // this row's last visible key
    const uint32_t key_end = p.start_pos + p.n_q;        // rows past the chunk are never valid
    const uint32_t horizon = min(qpos, key_end - 1);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    float s[128];
    for (uint32_t j = 0; j < nblk; j++) {
      if (!warp_wait(bar + 8 * (B_SFULL + (j & 1)), (j >> 1) & 1, abort_flag, &wsh->error)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tmem_s = tmem + (j & 1) * 128;
#pragma unroll
      for (int c = 0; c < 4; c++) tmem_ld32(tmem_s + lane_base + c * 32, s + c * 32);
      tmem_ld_wait();
      const uint32_t key0 = j * BN;
      if (key0 + BN - 1 > horizon) {
#pragma unroll
        for (int c = 0; c < 128; c++)
          if (key0 + c > horizon) s[c] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; c++) mx = fmaxf(mx, s[c]);
      mx *= p.scale_log2;
      const bool up = mx > m + RESCALE_LOG2;
      if (__any_sync(0xffffffffu, up)) {
        const float alpha = up ? ex2f(m - mx) : 1.f;  // 0 while m is -inf
        if (j > 0) {
          // O is rescaled only after PV(j-1) has accumulated into it.  S(j)
          // was issued after PV(j-2), so PV completions are j-1 or j here and
          // the parity of phase j-1 is unambiguous.
          if (!warp_wait(bar + 8 * B_PVDONE, (j - 1) & 1, abort_flag, &wsh->error)) {
            ok = false;
            break;
          }
          tc_fence_after();
          float ov[32];
#pragma unroll
          for (int c = 0; c < 4; c++) {
            tmem_ld32(tmem_o + lane_base + c * 32, ov);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) ov[i] *= alpha;
            tmem_st32(tmem_o + lane_base + c * 32, ov);
          }
          tmem_st_wait();
        }
        l *= alpha;
        if (up) m = mx;
      }
      const float nb = m == -INFINITY ? 0.f : -m;
      float rs = 0.f;
      // P from the scores just read: the fp16 pair of scores 2c and 2c+1
      // goes to head word c (stored over s[c], already consumed) and
      // remainder word c
      uint32_t* head = reinterpret_cast<uint32_t*>(s);
      uint32_t rem[64];
#pragma unroll
      for (int c = 0; c < 64; c++) {
        const float p0 = ex2f(fmaf(s[2 * c], p.scale_log2, nb));
        const float p1 = ex2f(fmaf(s[2 * c + 1], p.scale_log2, nb));
        rs += p0 + p1;
        __half2 hh = __floats2half2_rn(p0, p1);
        __half2 rr = __floats2half2_rn(p0 - __low2float(hh), p1 - __high2float(hh));
        head[c] = *reinterpret_cast<uint32_t*>(&hh);
        rem[c] = *reinterpret_cast<uint32_t*>(&rr);
      }
      l += rs;
      tmem_st32(tmem_s + lane_base, reinterpret_cast<float*>(head));
      tmem_st32(tmem_s + lane_base + 32, reinterpret_cast<float*>(head + 32));
      tmem_st32(tmem_s + lane_base + 64, reinterpret_cast<float*>(rem));
      tmem_st32(tmem_s + lane_base + 96, reinterpret_cast<float*>(rem + 32));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar + 8 * B_PFULL);
    }
    // every PV has completed once the MMA warp's drain commit has arrived
    if (ok && warp_wait(bar + 8 * B_DRAIN, 0, abort_flag, &wsh->error)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __half* orow = p.o + (((size_t)b * p.n_q + q0 + r) * p.n_heads + h) * PHD;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float ov[32];
        tmem_ld32(tmem_o + lane_base + c * 32, ov);
        tmem_ld_wait();
        if (r < nq_valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            __half2 h0 = __floats2half2_rn(ov[i] * inv, ov[i + 1] * inv);
            __half2 h1 = __floats2half2_rn(ov[i + 2] * inv, ov[i + 3] * inv);
            __half2 h2 = __floats2half2_rn(ov[i + 4] * inv, ov[i + 5] * inv);
            __half2 h3 = __floats2half2_rn(ov[i + 6] * inv, ov[i + 7] * inv);
            v.x = *reinterpret_cast<uint32_t*>(&h0);
            v.y = *reinterpret_cast<uint32_t*>(&h1);
            v.z = *reinterpret_cast<uint32_t*>(&h2);
            v.w = *reinterpret_cast<uint32_t*>(&h3);
            *reinterpret_cast<uint4*>(orow + c * 32 + i) = v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TMEM_COLS)
                 : "memory");
}

// ---- KV-cache rows for a prompt chunk (the kv_append path, many rows) ----
__global__ void kv_append_rows_kernel(const uint4* __restrict__ k_src,
                                      const uint4* __restrict__ v_src, uint4* __restrict__ k_pool,
                                      uint4* __restrict__ v_pool, const int64_t* __restrict__ row_offset,
                                      uint64_t pool_rows, uint32_t start_pos, uint32_t n_rows,
                                      uint32_t row_vec, uint32_t* err) {
  const uint32_t b = blockIdx.y;
  const int64_t base = row_offset[b] + (int64_t)start_pos;
  const uint64_t total = (uint64_t)n_rows * row_vec;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = i / row_vec, c = i % row_vec;
    const int64_t row = base + (int64_t)r;
    if (row < 0 || (uint64_t)row >= pool_rows) {
      if (c == 0 && err) atomicOr(err, NWD_DEVERR_ROW_RANGE);
      continue;
    }
    const uint64_t src = ((uint64_t)b * n_rows + r) * row_vec + c;
    k_pool[(uint64_t)row * row_vec + c] = __ldg(k_src + src);
    v_pool[(uint64_t)row * row_vec + c] = __ldg(v_src + src);
  }
}

bool g_prefill_smem_set[64] = {};

}  // namespace

using namespace nwd;

extern "C" {

int nwd_kv_append_rows(const uint16_t* k_src, const uint16_t* v_src, uint16_t* k_pool,
                       uint16_t* v_pool, uint64_t pool_rows, const int64_t* row_offset,
                       uint32_t start_pos, uint32_t n_rows, uint32_t batch, uint32_t n_kv,
                       uint32_t hd, void* workspace, size_t ws_bytes, void* stream) {
  const char* who = "nwd_kv_append_rows";
  if (!k_src || !v_src || !k_pool || !v_pool || !row_offset)
    return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  if (batch == 0 || n_rows == 0) return ok();
  if (n_kv == 0 || hd == 0) return fail(NWD_ERR_INVALID, "%s: zero shape", who);
  if (batch > 65535u) return fail(NWD_ERR_UNSUPPORTED, "%s: batch > 65535", who);
  const uint64_t row = (uint64_t)n_kv * hd;
  if (row % 8 || !aligned16(k_src) || !aligned16(v_src) || !aligned16(k_pool) || !aligned16(v_pool))
    return fail(NWD_ERR_UNSUPPORTED,
                "%s: rows must be a multiple of 8 halves, pointers 16-byte aligned", who);
  uint32_t* err = (workspace && ws_bytes >= sizeof(WsHeader))
                      ? &reinterpret_cast<WsHeader*>(workspace)->error
                      : nullptr;
  const uint32_t row_vec = (uint32_t)(row / 8);
  const uint64_t total = (uint64_t)n_rows * row_vec;
  uint32_t bx = (uint32_t)std::min<uint64_t>((total + 255) / 256, 1184);
  kv_append_rows_kernel<<<dim3(bx, batch), 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const uint4*>(k_src), reinterpret_cast<const uint4*>(v_src),
      reinterpret_cast<uint4*>(k_pool), reinterpret_cast<uint4*>(v_pool), row_offset, pool_rows,
      start_pos, n_rows, row_vec, err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
}

int nwd_attn_prefill(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                     uint64_t pool_rows, const int64_t* row_offset, uint16_t* o, uint32_t batch,
                     uint32_t n_q, uint32_t start_pos, uint32_t n_heads, uint32_t n_kv_heads,
                     uint32_t head_dim, float scale, void* workspace, size_t ws_bytes,
                     void* stream) {
  const char* who = "nwd_attn_prefill";
  if (!q || !k_pool || !v_pool || !row_offset || !o)
    return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  if (n_heads == 0 || n_kv_heads == 0 || n_heads % n_kv_heads)
    return fail(NWD_ERR_INVALID, "%s: n_heads must be a positive multiple of n_kv_heads", who);
  if (head_dim != PHD) return fail(NWD_ERR_UNSUPPORTED, "%s: head_dim %u (only 128)", who, head_dim);
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(o))
    return fail(NWD_ERR_INVALID, "%s: tensors must be 16-byte aligned", who);
  if (!workspace || ws_bytes < sizeof(WsHeader) || ((uintptr_t)workspace & 255u))
    return fail(NWD_ERR_WORKSPACE, "%s: needs a zeroed, 256-byte aligned workspace of >= %zu bytes",
                who, sizeof(WsHeader));
  if (!(scale >= 0.f) || isinf(scale))
    return fail(NWD_ERR_INVALID, "%s: scale must be finite and >= 0", who);
  if (batch == 0 || n_q == 0) return ok();
  if ((uint64_t)batch * n_q > (1ull << 31) || pool_rows == 0 || pool_rows > (1ull << 31) ||
      (uint64_t)start_pos + n_q > pool_rows)
    return fail(NWD_ERR_RANGE, "%s: rows out of range (batch*n_q %llu, start_pos %u, pool %llu)",
                who, (unsigned long long)batch * n_q, start_pos, (unsigned long long)pool_rows);
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st) return st;
  if (!g_prefill_smem_set[di.device]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         P_SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill_kernel)");
    g_prefill_smem_set[di.device] = true;
  }
  CUtensorMap tq, tk, tv;
  st = kv_tensor_map(&tq, q, (uint64_t)batch * n_q, n_heads, head_dim, BM, 1);
  if (st) return st;
  st = kv_tensor_map(&tk, k_pool, pool_rows, n_kv_heads, head_dim, BN, 1);
  if (st) return st;
  st = kv_tensor_map(&tv, v_pool, pool_rows, n_kv_heads, head_dim, BN, 1);
  if (st) return st;
  PParams p;
  memset(&p, 0, sizeof(p));
  p.o = reinterpret_cast<__half*>(o);
  p.row_offset = row_offset;
  p.ws = reinterpret_cast<uint8_t*>(workspace);
  p.pool_rows = pool_rows;
  p.batch = batch;
  p.n_q = n_q;
  p.start_pos = start_pos;
  p.n_heads = n_heads;
  p.n_kv = n_kv_heads;
  p.group = n_heads / n_kv_heads;
  p.q_tiles = (n_q + BM - 1) / BM;
  const float sc = scale != 0.f ? scale : 1.0f / sqrtf((float)head_dim);
  p.scale_log2 = sc * 1.4426950408889634f;
  const uint64_t grid = (uint64_t)batch * n_heads * p.q_tiles;
  if (grid > 0x7fffffffull) return fail(NWD_ERR_UNSUPPORTED, "%s: too many tiles", who);
  prefill_kernel<<<(uint32_t)grid, PTHR, P_SMEM_BYTES, (cudaStream_t)stream>>>(tq, tk, tv, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
}

}  // extern "C"
