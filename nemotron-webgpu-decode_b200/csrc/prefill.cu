// Causal chunked prefill attention on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory).
//
// The reference has no prefill: it feeds the prompt one decode step per token
// (engine/runtime.js:640-643), so prompt token i of a chunk that starts at
// cache row start_pos attends rows 0 .. start_pos + i.  This kernel computes
// exactly that for a whole chunk at once, as a dense contraction.
//
// Work unit: a tile = (sequence, query head, 128 queries).  The kernel is
// persistent: one CTA per SM walks the tiles heaviest first (late query tiles
// see the most keys) in a snake order over the CTAs, and the roles below
// stream from one tile into the next, so a tile's start (Q load, first scores)
// and end (last P V, O read-out and store) overlap the neighbouring tiles'
// work.  12 warps:
//   warps 0, 3  TMA producers: warp 0 each tile's Q into one of two Q buffers
//               and the K blocks of 128 rows, warp 3 the V blocks, each into
//               a 2-stage ring (K(g) is free once S(g) is done, long before
//               V(g)); each 128-row tile as two 64-column chunks, 128-byte
//               swizzle: the canonical K-major layout of the tcgen05
//               shared-memory descriptors.
//   warp 1      MMA issuer (one thread).  Over the flattened sequence of
//               blocks g of all its tiles: S(g) = Q K(g)^T into TMEM score
//               buffer g mod 3 (M=128 queries, N=128 keys, K=128 = 8 MMAs of
//               K=16), up to two blocks ahead of the P V MMAs so the softmax
//               never waits for them; then, once P(g) is in TMEM, O += P V
//               into the TMEM accumulator with A = P read from tensor memory
//               and B = V an MN-major shared-memory operand.  P is an fp16 head and an fp16 remainder (16 MMAs):
//               one fp16 rounding of P would exceed the parity tolerance on
//               outputs near zero.  tcgen05.commit signals S ready, K/V/Q
//               free, PV done and O complete.
//   warp 2      TMEM allocation (512 columns: S0, S1, S2, O) and release.
//   warps 4-7   softmax: thread r owns query row r (TMEM lane r).  Per block
//               it reads its 128 scores (240 registers per thread: the other
//               warpgroups give theirs up with setmaxnreg), applies the causal
//               mask, updates the running max with lazy rescaling (O is
//               rescaled in TMEM only when a row's max grows by more than
//               2^8), and writes P = 2^(s - m) over its own scores as fp16
//               pairs (per half: head, then remainder).  P(g) needs no wait on
//               PV(g-1), which reads another buffer; the MMAs of one thread
//               run in issue order, so S(g+3) overwrites P(g) only after
//               PV(g) has read it.  At the end of a tile it hands the row sums
//               to the epilogue through shared memory.
//   warps 8-11  epilogue: per tile, once its last PV has completed, divides
//               O by the row sum and stores it as fp16, then frees the O
//               accumulator for the next tile's first PV.
// K/V rows past the chunk's end that a block covers are zeroed in shared
// memory before P V reads them (P is 0 there, but 0 x NaN would not be).
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
constexpr int PTHR = 384;         // 12 warps
constexpr int CHUNK = 128 * 128;  // 128 rows x 64 fp16 (one 64-column chunk): 16 KiB
constexpr int TILE = 2 * CHUNK;   // 128 x 128 fp16: 32 KiB

constexpr int O_Q = 0;                  // 2 Q buffers
constexpr int O_K = O_Q + 2 * TILE;     // 2 K stages
constexpr int O_V = O_K + 2 * TILE;     // 2 V stages
constexpr int O_L = O_V + 2 * TILE;     // row sums handed to the epilogue [2][128] f32
constexpr int O_BAR = O_L + 2 * BM * 4;
// barrier pairs are indexed by buffer (Q, O, L: tile parity; K, V, S, P: block parity)
// Pairs: Q, L by tile parity; K, V by block parity.  Triples: S, P and PV
// done by score buffer (block index mod 3).  V_TMA: completion of a V copy
// whose rows past the chunk's end are zeroed before V_FULL (the producer
// waits for each such copy before it issues the next).
constexpr int B_QFULL = 0, B_QEMPTY = 2, B_KFULL = 4, B_KEMPTY = 6, B_VFULL = 8, B_VEMPTY = 10,
              B_VTMA = 12, B_LFULL = 13, B_LEMPTY = 15, B_SFULL = 17, B_PFULL = 20,
              B_PVDONE = 23, B_OFULL = 26, B_OEMPTY = 27, B_DRAIN = 28, NBAR = 29;
constexpr int O_MISC = O_BAR + NBAR * 8;  // tmem base (u32), abort flag (i32)
constexpr int P_SMEM_USED = O_MISC + 16;
constexpr int P_SMEM_BYTES = P_SMEM_USED + 1024;
static_assert(P_SMEM_BYTES <= 227 * 1024, "shared memory");

constexpr uint32_t TMEM_COLS = 512;  // S0, S1, S2 (128 columns each), then O at 384
constexpr uint32_t TMEM_O = 384;
constexpr uint32_t NSBUF = 3;        // score / P buffers
constexpr uint32_t GROUP_THREADS = 128;  // softmax / epilogue warpgroups
constexpr float RESCALE_LOG2 = 8.f;

struct PParams {
  __half* o;
  const int64_t* row_offset;
  uint8_t* ws;
  uint64_t pool_rows;
  uint32_t batch, n_q, start_pos, n_heads, n_kv, group, q_tiles, n_tiles;
  float scale_log2;
};

// One tile of the heaviest-first snake schedule: round k of CTA c takes tile
// k * G + c (k even) or k * G + G - 1 - c (k odd); tile index t covers query
// tile q_tiles - 1 - t / (batch * n_heads) of (sequence, head) t % (batch * n_heads).
struct Tile {
  uint32_t b, h, hkv, q0, nq, nblk;
  int kv_row0;
};
__device__ __forceinline__ bool get_tile(const PParams& p, uint32_t k, Tile& t) {
  const uint32_t G = gridDim.x, c = blockIdx.x;
  const uint64_t idx = (uint64_t)k * G + ((k & 1u) ? (G - 1 - c) : c);
  if (idx >= p.n_tiles) return false;
  const uint32_t bh_count = p.batch * p.n_heads;
  const uint32_t rank = (uint32_t)(idx / bh_count), bh = (uint32_t)(idx % bh_count);
  const uint32_t qt = p.q_tiles - 1 - rank;
  t.b = bh / p.n_heads;
  t.h = bh % p.n_heads;
  t.hkv = t.h / p.group;
  t.q0 = qt * BM;
  t.nq = min((uint32_t)BM, p.n_q - t.q0);
  t.nblk = (p.start_pos + t.q0 + t.nq - 1) / BN + 1;  // causal horizon of the tile
  t.kv_row0 = (int)p.row_offset[t.b];
  return true;
}

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

// P for one half row: the fp16 pair of scores 2c and 2c+1 becomes head word
// c and remainder word c; they are written back over the half's own score
// columns (head at +0, remainder at +32).  Returns the half's sum of P.
__device__ __forceinline__ float store_p_half(uint32_t taddr, float* s, float scale_log2,
                                              float nb) {
  float rsv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float head[32], rem[32];
#pragma unroll
  for (int c = 0; c < 32; c++) {
    const float p0 = ex2f(fmaf(s[2 * c], scale_log2, nb));
    const float p1 = ex2f(fmaf(s[2 * c + 1], scale_log2, nb));
    rsv[c & 7] += p0 + p1;
    __half2 hh = __floats2half2_rn(p0, p1);
    __half2 rr = __floats2half2_rn(p0 - __low2float(hh), p1 - __high2float(hh));
    head[c] = __uint_as_float(*reinterpret_cast<uint32_t*>(&hh));
    rem[c] = __uint_as_float(*reinterpret_cast<uint32_t*>(&rr));
  }
  tmem_st32(taddr, head);
  tmem_st32(taddr + 32, rem);
  return ((rsv[0] + rsv[4]) + (rsv[1] + rsv[5])) + ((rsv[2] + rsv[6]) + (rsv[3] + rsv[7]));
}

// Position in a ring of 3 buffers: the buffer and the parity of its use.
struct Ring3 {
  uint32_t buf = 0, phase = 0;
  __device__ __forceinline__ void next() {
    if (++buf == NSBUF) {
      buf = 0;
      phase ^= 1u;
    }
  }
};

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
  const uint32_t key_end = p.start_pos + p.n_q;  // rows past the chunk are never valid

  if (tid == 0) {
    *abort_flag = 0;
    for (int s = 0; s < 2; s++) {
      mbar_init(bar + 8 * (B_QFULL + s), 1);
      mbar_init(bar + 8 * (B_QEMPTY + s), 1);
      mbar_init(bar + 8 * (B_KFULL + s), 1);
      mbar_init(bar + 8 * (B_KEMPTY + s), 1);
      mbar_init(bar + 8 * (B_VFULL + s), 1);
      mbar_init(bar + 8 * (B_VEMPTY + s), 1);
      mbar_init(bar + 8 * (B_LFULL + s), GROUP_THREADS);
      mbar_init(bar + 8 * (B_LEMPTY + s), GROUP_THREADS);
    }
    for (int s = 0; s < (int)NSBUF; s++) {
      mbar_init(bar + 8 * (B_SFULL + s), 1);
      mbar_init(bar + 8 * (B_PFULL + s), GROUP_THREADS);
      mbar_init(bar + 8 * (B_PVDONE + s), 1);
    }
    mbar_init(bar + 8 * B_VTMA, 1);
    mbar_init(bar + 8 * B_OFULL, 1);
    mbar_init(bar + 8 * B_OEMPTY, GROUP_THREADS);
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
  // Register split (per thread), set at the top of each role: producer/MMA
  // warpgroup 56, softmax 240, epilogue 120.  128 * (56 + 240 + 120) = 53248
  // registers, within the 384 * 168 = 64512 this kernel is launched with.
  if (warp == 0 || warp == 3) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");
    // ================ TMA producers: warp 0 Q and K, warp 3 V ================
    // K and V come from separate warps so that K(g+1), needed early for the
    // look-ahead S, never queues behind V(g), whose stage frees only when
    // PV(g-2) completes.
    const bool kq = warp == 0;
    const uint64_t pol_q = evict_first_policy(), pol_kv = evict_last_policy();
    // loads issued so far (buffer i of a pair got the ones with index parity i)
    uint32_t nq = 0, nkv = 0, ntma = 0;
    bool ok = true;
    uint32_t g = 0, u = 0;
    Tile t;
    const int kv_full = kq ? B_KFULL : B_VFULL, kv_empty = kq ? B_KEMPTY : B_VEMPTY;
    const uint32_t kv_smem = sb + (kq ? O_K : O_V);
    const CUtensorMap* kv_map = kq ? &tmk : &tmv;
    for (uint32_t k = 0; ok && get_tile(p, k, t); k++, u++) {
      if (kq) {
        const uint32_t qs = u & 1;
        // Q buffer qs is free once the last S of tile u-2 has completed
        if (!warp_wait(bar + 8 * (B_QEMPTY + qs), ((u >> 1) & 1) ^ 1, abort_flag, &wsh->error)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t fb = bar + 8 * (B_QFULL + qs);
          mbar_arrive_tx(fb, TILE);
          const int qrow = (int)(t.b * p.n_q + t.q0);
          tma_load_4d(sb + O_Q + qs * TILE, &tmq, fb, 0, 0, (int)t.h, qrow, pol_q);
          tma_load_4d(sb + O_Q + qs * TILE + CHUNK, &tmq, fb, 0, 1, (int)t.h, qrow, pol_q);
        }
        __syncwarp();
        nq++;
      }
      for (uint32_t j = 0; j < t.nblk; j++, g++) {
        const uint32_t st = g & 1;
        // K(g) is free once S(g-2) has completed, V(g) once PV(g-2) has
        if (!warp_wait(bar + 8 * (kv_empty + st), ((g >> 1) & 1) ^ 1, abort_flag,
                       &wsh->error)) {
          ok = false;
          break;
        }
        const int row = t.kv_row0 + (int)(j * BN);
        // V rows past the chunk's end (P is 0 there, but 0 x NaN would not
        // be): the copy completes on V_TMA, this warp zeroes them, then
        // releases the stage on V_FULL
        const uint32_t valid = key_end - j * BN;
        const bool tail = !kq && valid < (uint32_t)BN;
        const uint32_t fb = bar + 8 * (tail ? B_VTMA : kv_full + st);
        if (lane == 0) {
          mbar_arrive_tx(fb, TILE);
          tma_load_4d(kv_smem + st * TILE, kv_map, fb, 0, 0, (int)t.hkv, row, pol_kv);
          tma_load_4d(kv_smem + st * TILE + CHUNK, kv_map, fb, 0, 1, (int)t.hkv, row, pol_kv);
        }
        __syncwarp();
        if (tail) {
          ntma++;
          if (!warp_wait(fb, (ntma - 1) & 1, abort_flag, &wsh->error)) {
            ok = false;
            break;
          }
          // rows [valid, 128) of both 64-column chunks: 128 bytes each
          const uint4 z = make_uint4(0u, 0u, 0u, 0u);
          for (uint32_t i = valid * 8 + (uint32_t)lane; i < (uint32_t)BN * 8; i += 32) {
            reinterpret_cast<uint4*>(smem + O_V + st * TILE)[i] = z;
            reinterpret_cast<uint4*>(smem + O_V + st * TILE + CHUNK)[i] = z;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive(bar + 8 * (kv_full + st));
        }
        nkv++;
      }
    }
    if (!ok) {
      // let this warp's copies in flight land before the CTA can exit
      const uint64_t t0 = globaltimer();
      auto land = [&](int base, uint32_t n) {
#pragma unroll
        for (uint32_t s = 0; s < 2; s++) {
          const uint32_t cnt = (n + 1 - s) / 2;  // loads that went to buffer s
          if (cnt)
            while (!mbar_try_wait(bar + 8 * (base + s), (cnt - 1) & 1) &&
                   globaltimer() - t0 < WAIT_LIMIT_NS) {
            }
        }
      };
      if (kq) {
        land(B_QFULL, nq);
        land(B_KFULL, nkv);
      } else {
        // a V copy completes on V_FULL (counted by nkv once released) or, for
        // a tail block, on V_TMA (its last phase covers one still in flight)
        land(B_VFULL, nkv);
        if (ntma)
          while (!mbar_try_wait(bar + 8 * B_VTMA, (ntma - 1) & 1) &&
                 globaltimer() - t0 < WAIT_LIMIT_NS) {
          }
      }
    }
  } else if (warp == 1) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");
    // ======================= MMA issuer =======================
    // Over the flattened blocks of all its tiles, the issuer polls for the
    // next S and the next PV and issues whichever is ready, S first:
    //   S(gs)  needs K(gs) (and the tile's Q at its first block) and
    //          gs <= gp + 2, i.e. PV(gs-3), which reads P from the score
    //          buffer S(gs) overwrites, already issued (the MMAs of one
    //          thread run in order);
    //   PV(gp) needs gp < gs, P(gp) and V(gp), and at a tile's first block
    //          the O accumulator released by the epilogue.
    // S thus runs up to two blocks ahead of PV: the softmax of a block never
    // waits for the PV two blocks back.
    // The scheduler runs on lane 0 alone (an MMA issue blocks while the
    // tensor pipe's queue is full, so every cycle between issues is idle
    // tensor time): no warp-collective operation in the loop, and the clock
    // is read only while nothing can be issued.
    if (lane == 0) {
      Tile ts, tp;
      uint32_t ks = 0, us = 0, js = 0, gs = 0;  // next S
      uint32_t kp = 0, up = 0, jp = 0, gp = 0;  // next PV
      Ring3 rs, rp;                             // their score buffers
      bool have_s = get_tile(p, 0, ts);
      bool have_p = get_tile(p, 0, tp);
      uint32_t idle = 0;
      uint64_t idle_since = 0;
      while (have_p) {
        if (have_s && gs <= gp + 2 &&
            (js != 0 || mbar_test_wait(bar + 8 * (B_QFULL + (us & 1)), (us >> 1) & 1)) &&
            mbar_test_wait(bar + 8 * (B_KFULL + (gs & 1)), (gs >> 1) & 1)) {
          const uint32_t st = gs & 1, qs = us & 1;
          tc_fence_after();
          // 8 K-steps of 16 over head_dim (32 bytes apart in a 64-column chunk)
          const uint64_t da = sdesc(sb + O_Q + qs * TILE, 16, 1024);
          const uint64_t db = sdesc(sb + O_K + st * TILE, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < 8; kk++) {
            // the start address field is addr >> 4: offsets add directly
            const uint32_t off = ((uint32_t)(kk >> 2) * CHUNK + (uint32_t)(kk & 3) * 32) >> 4;
            umma(tmem + rs.buf * 128, da + off, db + off, IDESC_S, kk > 0);
          }
          umma_commit(bar + 8 * (B_KEMPTY + st));
          umma_commit(bar + 8 * (B_SFULL + rs.buf));
          if (js + 1 == ts.nblk) umma_commit(bar + 8 * (B_QEMPTY + qs));
          gs++;
          rs.next();
          if (++js == ts.nblk) {
            js = 0;
            us++;
            have_s = get_tile(p, ++ks, ts);
          }
          idle = 0;
        } else if (gp < gs && (jp != 0 || mbar_test_wait(bar + 8 * B_OEMPTY, (up & 1) ^ 1)) &&
                   mbar_test_wait(bar + 8 * (B_PFULL + rp.buf), rp.phase) &&
                   mbar_test_wait(bar + 8 * (B_VFULL + (gp & 1)), (gp >> 1) & 1)) {
          const uint32_t st = gp & 1;
          tc_fence_after();
          // O += P V: 8 K-steps of 16 keys (8 TMEM columns of fp16 pairs) for
          // the P head, then 8 for the P remainder.  P columns: keys [0,64)
          // head at +0 and remainder at +32, keys [64,128) head at +64 and
          // remainder at +96.  V MN-major (head_dim contiguous): its
          // 64-column chunks are LBO = 16 KiB apart; 16 keys are 2 KiB.
          const uint32_t tmem_p = tmem + rp.buf * 128;
          const uint64_t dv = sdesc(sb + O_V + st * TILE, CHUNK, 1024);
#pragma unroll
          for (int kstep = 0; kstep < 16; kstep++) {
            const uint32_t kk = (uint32_t)(kstep & 7);
            umma_ts(tmem + TMEM_O,
                    tmem_p + (kk >> 2) * 64u + (kstep < 8 ? 0u : 32u) + (kk & 3u) * 8u,
                    dv + ((kk * 16 * 128) >> 4), IDESC_O, (jp > 0 || kstep > 0) ? 1u : 0u);
          }
          umma_commit(bar + 8 * (B_VEMPTY + st));
          umma_commit(bar + 8 * (B_PVDONE + rp.buf));
          if (jp + 1 == tp.nblk) umma_commit(bar + 8 * B_OFULL);
          gp++;
          rp.next();
          if (++jp == tp.nblk) {
            jp = 0;
            up++;
            have_p = get_tile(p, ++kp, tp);
          }
          idle = 0;
        } else if ((++idle & 63) == 0) {
          // nothing ready: give up after WAIT_LIMIT_NS without progress
          if (*abort_flag) break;
          const uint64_t now = globaltimer();
          if (idle == 64) {
            idle_since = now;
          } else if (now - idle_since > WAIT_LIMIT_NS) {
            atomicOr(&wsh->error, NWD_DEVERR_PIPE_TIMEOUT);
            *abort_flag = 1;
            break;
          }
        }
      }
    }
    __syncwarp();
    // every MMA this thread issued has completed before TMEM is released
    if (lane == 0) umma_commit(bar + 8 * B_DRAIN);
    __syncwarp();
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar + 8 * B_DRAIN, 0) && globaltimer() - t0 < WAIT_LIMIT_NS) {
    }
  } else if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;" ::: "memory");  // TMEM owner, idle
  } else if (warp < 8) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 240;" ::: "memory");
    // ======================= softmax =======================
    const uint32_t r = (uint32_t)(tid - 128);                 // query row = TMEM lane
    const uint32_t lane_base = (uint32_t)(warp - 4) * 32u << 16;
    const uint32_t tmem_o = tmem + TMEM_O + lane_base;
    float* lsum = reinterpret_cast<float*>(smem + O_L);
    bool ok = true;
    uint32_t u = 0;
    Ring3 rb;        // score buffer of the current block
    Ring3 rprev;     // score buffer of the block before it
    Tile t;
    float s[128];
    for (uint32_t k = 0; ok && get_tile(p, k, t); k++, u++) {
      const uint32_t horizon = min(p.start_pos + t.q0 + r, key_end - 1);
      float m = -INFINITY, l = 0.f;
      for (uint32_t j = 0; j < t.nblk; j++) {
        if (!warp_wait(bar + 8 * (B_SFULL + rb.buf), rb.phase, abort_flag, &wsh->error)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tmem_s = tmem + rb.buf * 128 + lane_base;
        const uint32_t key0 = j * BN;
#pragma unroll
        for (int c = 0; c < 4; c++) tmem_ld32(tmem_s + c * 32, s + c * 32);
        tmem_ld_wait();
        if (key0 + BN - 1 > horizon) {
#pragma unroll
          for (int c = 0; c < 128; c++)
            if (key0 + c > horizon) s[c] = -INFINITY;
        }
        // eight independent max chains, then a tree
        float mv[8];
#pragma unroll
        for (int i = 0; i < 8; i++) mv[i] = s[i];
#pragma unroll
        for (int c = 8; c < 128; c++) mv[c & 7] = fmaxf(mv[c & 7], s[c]);
#pragma unroll
        for (int i = 0; i < 4; i++) mv[i] = fmaxf(mv[i], mv[i + 4]);
        const float mx = fmaxf(fmaxf(mv[0], mv[1]), fmaxf(mv[2], mv[3])) * p.scale_log2;
        const bool up = mx > m + RESCALE_LOG2;
        if (__any_sync(0xffffffffu, up)) {
          const float alpha = up ? ex2f(m - mx) : 1.f;  // 0 while m is -inf
          if (j > 0) {
            // O is rescaled only after PV of the block before has accumulated
            // into it.  Its PV_DONE barrier (one per score buffer) last
            // completed for the block three before that, which finished
            // before S of this block was issued: the parity is unambiguous.
            if (!warp_wait(bar + 8 * (B_PVDONE + rprev.buf), rprev.phase, abort_flag,
                           &wsh->error)) {
              ok = false;
              break;
            }
            tc_fence_after();
            float ov[32];
#pragma unroll
            for (int c = 0; c < 4; c++) {
              tmem_ld32(tmem_o + c * 32, ov);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; i++) ov[i] *= alpha;
              tmem_st32(tmem_o + c * 32, ov);
            }
          }
          l *= alpha;
          if (up) m = mx;
        }
        const float nb = m == -INFINITY ? 0.f : -m;
        l += store_p_half(tmem_s, s, p.scale_log2, nb) +
             store_p_half(tmem_s + 64, s + 64, p.scale_log2, nb);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(bar + 8 * (B_PFULL + rb.buf));
        rprev = rb;
        rb.next();
      }
      if (!ok) break;
      // hand the row sums of tile u to the epilogue
      const uint32_t ls = u & 1;
      if (!warp_wait(bar + 8 * (B_LEMPTY + ls), ((u >> 1) & 1) ^ 1, abort_flag, &wsh->error))
        break;
      lsum[ls * BM + r] = l;
      mbar_arrive(bar + 8 * (B_LFULL + ls));
    }
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 120;" ::: "memory");
    // ======================= epilogue =======================
    // Per tile: once its last PV has completed, O is read out of TMEM as
    // fp16 (normalised by the row sum) and the accumulator is released for
    // the next tile's first PV before the rows are stored.
    const uint32_t quad = (uint32_t)warp & 3u;
    const uint32_t r = quad * 32u + (uint32_t)lane;
    const uint32_t lane_base = quad * 32u << 16;
    const float* lsum = reinterpret_cast<const float*>(smem + O_L);
    uint32_t u = 0;
    Tile t;
    for (uint32_t k = 0; get_tile(p, k, t); k++, u++) {
      const uint32_t ls = u & 1;
      if (!warp_wait(bar + 8 * (B_LFULL + ls), (u >> 1) & 1, abort_flag, &wsh->error) ||
          !warp_wait(bar + 8 * B_OFULL, u & 1, abort_flag, &wsh->error))
        break;
      tc_fence_after();
      const float lt = lsum[ls * BM + r];
      mbar_arrive(bar + 8 * (B_LEMPTY + ls));
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      uint32_t packed[64];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float ov[32];
        tmem_ld32(tmem + TMEM_O + lane_base + c * 32, ov);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          __half2 h2 = __floats2half2_rn(ov[i] * inv, ov[i + 1] * inv);
          packed[c * 16 + i / 2] = *reinterpret_cast<uint32_t*>(&h2);
        }
      }
      tc_fence_before();
      mbar_arrive(bar + 8 * B_OEMPTY);
      if (r < t.nq) {
        uint4* orow = reinterpret_cast<uint4*>(
            p.o + (((size_t)t.b * p.n_q + t.q0 + r) * p.n_heads + t.h) * PHD);
#pragma unroll
        for (int i = 0; i < 16; i++)
          orow[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                               packed[4 * i + 3]);
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
  const uint64_t tiles = (uint64_t)batch * n_heads * p.q_tiles;
  if (tiles > 0x7fffffffull) return fail(NWD_ERR_UNSUPPORTED, "%s: too many tiles", who);
  p.n_tiles = (uint32_t)tiles;
  // persistent: one CTA per SM (shared memory and TMEM allow no second one)
  const uint32_t grid = (uint32_t)std::min<uint64_t>(tiles, (uint64_t)di.sm_count);
  prefill_kernel<<<grid, PTHR, P_SMEM_BYTES, (cudaStream_t)stream>>>(tq, tk, tv, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
}

}  // extern "C"
