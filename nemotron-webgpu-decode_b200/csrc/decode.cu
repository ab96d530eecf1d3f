// Split-KV flash-decode for GQA attention over a token-major fp16 KV cache.
//
// Restates kernels/sparse_attn.wgsl:32-113 (O = softmax(scale q.K^T) V per
// query head, kv head = h / group) for B200:
//
//  * Work split (stream-K style): the (sequence, kv head, row) space of the
//    whole call is flattened, pair by pair, and every persistent CTA (one per
//    SM) takes one equal contiguous range of it.  A range is cut at pair
//    boundaries into pieces: pieces covering a whole pair write O directly;
//    only the pieces at the two ends of a range are partial, so a CTA has at
//    most two partials to merge and every SM streams the same number of bytes
//    whatever the length distribution (ragged batches, one long sequence).
//  * Per CTA: one producer warp streams 64-row K and V tiles of the piece's kv
//    head into a 5-stage shared-memory ring with TMA (4-D tensor map over the
//    [rows, n_kv, 128] cache, 128-byte swizzle, no multicast) and mbarrier
//    transaction counts.  A piece's first stage also carries the G query rows
//    of its kv head (1-D bulk copy).
//  * Four consumer warps each take 16 rows of every stage.  All G <= 8 query
//    heads of the kv head share each loaded K/V tile: S^T = K Q^T and
//    O^T += V^T P^T are m16n8k16 tensor-core MMAs with rows (tokens) on M and
//    query heads on N, fp32 accumulation.  Online softmax in the log2 domain
//    with shuffle max reductions and lazy rescaling; P is handed from the score
//    accumulators to the PV operand with movmatrix (no shared-memory round
//    trip), as an fp16 head + fp16 remainder pair (two MMAs) so P keeps ~22
//    bits.
//  * End of piece: the four warps merge their (m, l, acc) in shared memory.
//    A partial piece writes its (m, l, acc) to a workspace slot and takes a
//    ticket on its pair; the CTA holding the pair's last ticket merges the
//    pieces in range order (deterministic) and writes the result.  No CTA
//    ever waits for another.
//  * Optional append mode fuses kernels/kv_append.wgsl: the piece that ends
//    at the new row writes it (generic stores + proxy fence) before its TMA
//    loads read it.
//
// Every mbarrier wait is bounded (time and iteration limits); on expiry the
// kernel records NWD_DEVERR_PIPE_TIMEOUT in the workspace and leaves after
// its own copies in flight have landed.
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>

#include "nwd_common.h"
#include "ptx.cuh"

namespace {

using namespace nwd::ptx;

using nwd::WsHeader;

constexpr int HD = 128;                  // head_dim supported by the tiles
constexpr int WPG = 4;                   // consumer warps per group (16 rows each)
constexpr int TOK = 16 * WPG;            // rows per stage
constexpr int NST = 5;                   // pipeline stages
constexpr int GMAX = 8;                  // query heads per kv head (mma N)
constexpr int KV_BYTES = TOK * HD * 2;   // one K (or V) stage: 16 KiB
constexpr int Q_BYTES = GMAX * HD * 2;   // query rows of one kv head
constexpr int MAXB = 4096;               // sequences per launch

// stage header flags
constexpr int32_t F_FIRST = 1, F_LAST = 2, F_COMPLETE = 4, F_TERM = 8;

// Written by the producer for every stage; `f`..`l` are the CTAs whose ranges
// cover the stage's (b, hkv) pair, `slot` the workspace slot of a partial piece.
struct StageHdr {
  int32_t b, hkv, t0, ntok, flags, slot, f, l;
};

struct Params {
  const __half* q;
  const __half* k_new;
  const __half* v_new;
  __half* k_pool;
  __half* v_pool;
  __half* o;
  float* part_o;    // partial mode: user outputs
  float* part_ml;
  const int64_t* row_offset;  // null => 0
  const int32_t* seq_len;     // null => single_len for b = 0
  uint8_t* ws;
  uint64_t pool_rows;
  uint64_t tickets_off, ml_off, o_off;
  uint32_t nslots;  // partial slots in the workspace (2 per CTA)
  int32_t single_len;
  uint32_t batch, n_heads, n_kv, group;
  float scale_log2;
  uint32_t append;   // seq_len holds the row to write; attend row + 1 rows
  uint32_t partial;  // write (m, l, o) partials instead of O
  uint32_t min_chunk;  // least rows (x kv heads) per CTA range
  uint32_t pair_max;   // one CTA per (sequence, kv head) when every pair is this short
  uint32_t split_k;    // > 0: CTA i takes piece i % k of pair i / k (k equal pieces per pair)
  uint32_t prefetch;   // single sequence: K/V tiles per CTA prefetched into L2 before the wait
  uint32_t prefetch_div;  // ... at most 1 / prefetch_div of the CTA's range
  uint32_t cluster;    // > 0: launched as clusters of this many CTAs, one cluster per kv
                       // head (split_k == cluster); the pieces merge over DSMEM
  nwd::XchgDesc x;     // partial mode, x.world > 0: push each pair's partial to every rank
  // Flattened split of a batch: each non-empty (sequence, kv head) pair of L
  // rows takes roundup(L + pair_cost, pair_pad) items of the range space
  // (pair_pad 1, pair_cost 0: L items).
  uint32_t pair_pad;
  uint32_t pair_cost;
};

// ---- shared memory layout (offsets from a 1024-aligned base) ----
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + NST * KV_BYTES;
constexpr int OFF_Q = OFF_V + NST * KV_BYTES;
constexpr int OFF_MRG = OFF_Q + NST * Q_BYTES;

// Configuration by number of consumer groups NG: one group of four warps, or
// two groups taking alternate stages (two warps per SM sub-partition, which
// hides the MMA / shuffle latency of the softmax chain when streaming).
template <int NG>
struct Cfg {
  static constexpr int NCW = WPG * NG;                  // consumer warps
  static constexpr int NTHR = (NCW + 1) * 32;           // + producer warp
  static constexpr int MRG_FLOATS = NCW * GMAX * (HD + 2);
  static constexpr int OFF_PFX = OFF_MRG + MRG_FLOATS * 4;
  static constexpr int OFF_HDR = OFF_PFX + ((MAXB + 1) * 4 + 15) / 16 * 16;
  static constexpr int OFF_BAR = OFF_HDR + NST * (int)sizeof(StageHdr);
  static constexpr int OFF_MISC = OFF_BAR + 2 * NST * 8 + 8;  // + consumer-sync barrier
  static constexpr int SMEM_USED = OFF_MISC + 64;
  static constexpr int SMEM_BYTES = SMEM_USED + 1024;  // slack for manual 1024-byte alignment
  static constexpr int DPT = GMAX * HD / (NCW * 32);   // epilogue dims per thread (8 or 4)
  static_assert(SMEM_BYTES <= 227 * 1024, "exceeds the 227 KiB per-CTA shared memory of sm_100");
  static_assert(NG == 1 || NG == 2, "one or two consumer groups");
};

struct Misc {
  int32_t abort;
  int32_t last;
  uint32_t warp_sum[10];
  uint32_t max_rows;
  uint64_t total_rows;
};
static_assert(sizeof(Misc) <= 64, "misc block");

constexpr float RESCALE_LOG2 = 8.f;  // lazy-rescale threshold (log2 units)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Barrier among the 128 consumer threads on an mbarrier, so that it is
// bounded like every other wait (a named barrier cannot time out).
__device__ __forceinline__ bool consumer_sync(uint32_t bar, uint32_t& ph, volatile int32_t* abort,
                                              uint32_t* dev_err) {
  mbar_arrive(bar);
  const bool ok = warp_wait(bar, ph, abort, dev_err);
  ph ^= 1u;
  return ok;
}

// This step's exchange row `row` of the source rank (this rank) in
// destination rank r's buffer.
__device__ __forceinline__ float* xchg_row(const nwd::XchgDesc& x, uint32_t r, uint32_t row) {
  const uint32_t par = x.epoch & 1u;
  return x.data[r] + ((size_t)(par * x.world + x.rank) * x.R + row) * nwd::XCH_ROW;
}
// Marks pair `pair` of this rank as written on every rank: one system-scope
// fence orders the partial's stores (made by this CTA's threads before a
// barrier) before the flag stores, which are relaxed (fence + relaxed store is
// a release; a release store per rank would wait on its own fence, world
// times over NVLink, on the step's critical path).
__device__ __forceinline__ void xchg_publish(const nwd::XchgDesc& x, uint32_t pair) {
  const uint32_t par = x.epoch & 1u;
  __threadfence_system();
  for (uint32_t r = 0; r < x.world; r++) {
    uint32_t* f = x.flags[r] + (size_t)(par * x.world + x.rank) * x.P + pair;
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(x.epoch) : "memory");
  }
}

// Cluster-wide barrier over every thread of every CTA of the cluster (release
// / acquire: shared-memory writes before it are visible to the cluster's
// distributed-shared-memory loads after it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Loads from CTA `rank`'s shared memory at the offset `local` has in this CTA.
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(remote)
               : "r"(smem_u32(local)), "r"(rank));
  return remote;
}
__device__ __forceinline__ float2 ld_cluster_f2(const float* local, uint32_t rank) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];"
               : "=f"(v.x), "=f"(v.y)
               : "r"(cluster_addr(local, rank))
               : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_cluster_f4(const float* local, uint32_t rank) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr(local, rank))
               : "memory");
  return v;
}

// Byte offset of 16-byte chunk `chunk16` of 128-byte row R inside a stage
// written by TMA with 128-byte swizzle (stage base 1024-aligned).
__device__ __forceinline__ uint32_t swz(uint32_t R, uint32_t chunk16) {
  return R * 128u + ((chunk16 ^ (R & 7u)) << 4);
}

// ---------------- work plan ----------------
// Rows attended by sequence b (clamped to the pool so every sum below fits).
__device__ __forceinline__ uint32_t seq_rows(const Params& p, uint32_t b) {
  int64_t v;
  if (!p.seq_len) v = p.single_len;
  else v = p.append ? (int64_t)p.seq_len[b] + 1 : (int64_t)p.seq_len[b];
  if (v <= 0) return 0u;
  return (uint64_t)v > p.pool_rows ? (uint32_t)p.pool_rows : (uint32_t)v;
}
// Range items of one (sequence, kv head) pair of L rows, the flattened
// split's unit: none for an empty pair; for a batch L + pair_cost rounded up
// to pair_pad, for a single sequence L.
__device__ __forceinline__ uint32_t pair_items(const Params& p, uint32_t L) {
  if (L == 0 || !p.seq_len) return L;
  return (uint32_t)(((uint64_t)L + p.pair_cost + p.pair_pad - 1) / p.pair_pad * p.pair_pad);
}
__device__ __forceinline__ int64_t seq_off(const Params& p, uint32_t b) {
  return p.row_offset ? p.row_offset[b] : 0;
}
__device__ __forceinline__ uint32_t cdiv(uint64_t a, uint64_t b) { return (uint32_t)((a + b - 1) / b); }

// Block-wide exclusive scan of per-thread values; returns this thread's
// offset, writes the grand total to *total (all threads see it after return).
template <int NTHR>
__device__ uint32_t block_scan(uint32_t v, Misc* misc, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) misc->warp_sum[warp] = x;
  __syncthreads();
  uint32_t before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < NTHR / 32; w++) {
    const uint32_t s = misc->warp_sum[w];
    if (w < warp) before += s;
    all += s;
  }
  __syncthreads();
  *total = all;
  return before + x - v;
}

// Largest b < batch with S[b] <= y (S non-decreasing, S[batch] > y): the
// sequence whose rows contain flattened row y.  Empty sequences never match.
__device__ __forceinline__ uint32_t find_seq(const uint32_t* S, uint32_t batch, uint64_t y) {
  uint32_t lo = 0, hi = batch;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if ((uint64_t)S[mid] <= y) lo = mid; else hi = mid;
  }
  return lo;
}

// ---------------- kernel ----------------
// 64-bit quotient with a 32-bit fast path (most operands fit).
__device__ __forceinline__ uint64_t udiv64(uint64_t a, uint64_t b) {
  if ((a >> 32) == 0 && (b >> 32) == 0) return (uint32_t)a / (uint32_t)b;
  return a / b;
}

template <int NG>
__global__ void __launch_bounds__(Cfg<NG>::NTHR, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const __grid_constant__ Params p) {
  using C = Cfg<NG>;
  constexpr int NCW = C::NCW, NTHR = C::NTHR, NGRP = NG;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint32_t* S = reinterpret_cast<uint32_t*>(smem + C::OFF_PFX);  // row prefix over sequences
  StageHdr* hdr = reinterpret_cast<StageHdr*>(smem + C::OFF_HDR);
  Misc* misc = reinterpret_cast<Misc*>(smem + C::OFF_MISC);
  volatile int32_t* abort_flag = &misc->abort;
  const uint32_t bar_full = sbase + C::OFF_BAR;            // + 8*s
  const uint32_t bar_empty = sbase + C::OFF_BAR + 8 * NST; // + 8*s
  const uint32_t bar_csync = sbase + C::OFF_BAR + 16 * NST;
  WsHeader* wsh = reinterpret_cast<WsHeader*>(p.ws);
  uint32_t* tickets = reinterpret_cast<uint32_t*>(p.ws + p.tickets_off);
  float* ws_ml = reinterpret_cast<float*>(p.ws + p.ml_off);
  float* ws_o = reinterpret_cast<float*>(p.ws + p.o_off);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t B = p.seq_len ? p.batch : 1u;
  const uint32_t G = p.group;
  // launched as a programmatic dependent launch: let the next kernel start
  // early, and wait for the previous one before touching any memory.  A
  // single sequence's plan reads only the parameters, so it (with the barrier
  // set-up and the tensor-map prefetch) runs while the previous kernel drains;
  // a batch's plan reads seq_len, which the previous kernel may write.
  nwd::pdl_trigger();
  const bool early_plan = p.seq_len == nullptr;
  if (!early_plan) nwd::pdl_wait();

  // ---- plan: row prefix S over sequences (S[b] = rows before b) ----
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
    misc->abort = 0;
    misc->last = 0;
    misc->total_rows = 0;
    misc->max_rows = 0;
#pragma unroll
    for (int s = 0; s < NST; s++) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, WPG);
    }
    mbar_init(bar_csync, NCW * 32);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint32_t seg = (B + NTHR - 1) / NTHR;
  const uint32_t beg = min(B, tid * seg), end = min(B, beg + seg);
  uint64_t rows_local = 0;  // range items of this thread's sequences (one kv head)
  uint32_t max_local = 0;
  for (uint32_t b = beg; b < end; b++) {
    const uint32_t L = seq_rows(p, b);
    rows_local += pair_items(p, L);
    max_local = max(max_local, L);
  }
  {
    // reduce within the warp first: one shared-memory atomic per warp (every
    // thread's atomics on the same two words serialised to 13 us at 256
    // sequences)
    unsigned long long ws = rows_local;
    uint32_t wm = max_local;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ws += __shfl_xor_sync(0xffffffffu, ws, o);
      wm = max(wm, __shfl_xor_sync(0xffffffffu, wm, o));
    }
    if (lane == 0 && ws) atomicAdd(reinterpret_cast<unsigned long long*>(&misc->total_rows), ws);
    if (lane == 0 && wm) atomicMax(&misc->max_rows, wm);
  }
  uint32_t total32;
  uint32_t run = block_scan<NTHR>((uint32_t)rows_local, misc, &total32);  // syncs: sums final
  if (misc->total_rows >= (1ull << 32)) {
    // more than 2^32 rows (range items) in one call: refuse (uniform across the block)
    if (early_plan) nwd::pdl_wait();
    if (tid == 0 && blockIdx.x == 0) atomicOr(&wsh->error, NWD_DEVERR_ROW_RANGE);
    return;
  }
  for (uint32_t b = beg; b < end; b++) {
    S[b] = run;
    run += pair_items(p, seq_rows(p, b));
  }
  if (tid == 0) S[B] = total32;
  __syncthreads();
  // Work split.  Pair mode (small problems): CTA i takes the whole pair i, no
  // partials.  Otherwise every CTA takes an equal range [x0, x1) of the
  // flattened (pair, row) space, T = n_kv * all rows.
  // Aligned split: CTA i takes piece i % k of pair i / k, the pair's rows cut
  // into k equal pieces (k = 1: one CTA per pair, no partials).  Chosen by the
  // host for a single sequence, or here for small problems.
  uint32_t split_k = p.split_k;
  if (split_k == 0 && (uint64_t)B * p.n_kv <= gridDim.x && misc->max_rows <= p.pair_max)
    split_k = 1;
  const uint64_t T = (uint64_t)p.n_kv * total32;
  uint64_t W = udiv64(T + gridDim.x - 1, gridDim.x);
  if (W < p.min_chunk) W = p.min_chunk;
  // range ends on a multiple of pair_pad inside every pair: each piece but a
  // pair's last holds whole stages, an even number of them
  W = udiv64(W + p.pair_pad - 1, p.pair_pad) * p.pair_pad;
  const uint64_t x0 = min(T, (uint64_t)blockIdx.x * W);
  const uint64_t x1 = min(T, x0 + W);

  if (early_plan) {
    // A single sequence: start this CTA's first K/V tiles on their way into L2
    // while the previous kernel drains (the rows are read again by TMA after
    // the wait; a row the previous kernel is still writing is updated in L2).
    // At most 1 / p.prefetch_div of the range's tiles and p.prefetch: measured
    // on back-to-back single-sequence steps, prefetching more (or at all for
    // ranges of a few tiles) floods DRAM while the previous kernel's
    // latency-bound merge still runs, and costs more than it hides.
    if (warp == NCW && lane == 0 && !p.row_offset && total32 > 0 && p.prefetch > 0) {
      const uint32_t L = total32;
      uint64_t x = x0, xe = x1;
      if (split_k) {
        const uint32_t j = blockIdx.x % split_k, hkv = blockIdx.x / split_k;
        x = (uint64_t)hkv * L + (uint64_t)j * L / split_k;
        xe = hkv < p.n_kv ? (uint64_t)hkv * L + (uint64_t)(j + 1) * L / split_k : x;
      }
      uint32_t budget = min(p.prefetch, (uint32_t)(udiv64(xe - x, TOK) / p.prefetch_div));
      while (x < xe && budget > 0) {
        const uint32_t hkv = (uint32_t)udiv64(x, L), t = (uint32_t)(x - (uint64_t)hkv * L);
        const uint32_t n = (uint32_t)min((uint64_t)(L - t), xe - x);
        for (uint32_t r = 0; r < n && budget > 0; r += TOK, budget--) {
          tma_prefetch_4d(&tmk, 0, 0, (int)hkv, (int)(t + r));
          tma_prefetch_4d(&tmv, 0, 0, (int)hkv, (int)(t + r));
        }
        x += n;
      }
    }
    nwd::pdl_wait();
  }

  // Empty sequences produce no rows, so no range covers them: CTA b % grid
  // writes their result (zeros, as the WGSL's untouched accumulator; or an
  // empty partial m = -inf, l = 0, o = 0).
  for (uint32_t b = blockIdx.x; b < B; b += gridDim.x) {
    if (S[b + 1] != S[b]) continue;
    if (p.append && tid == 0) atomicOr(&wsh->error, NWD_DEVERR_ROW_RANGE);  // pos < 0
    const size_t row0 = (size_t)b * p.n_heads;
    for (uint32_t i = tid; i < p.n_heads * (HD / 8); i += NTHR) {
      const size_t row = row0 + i / (HD / 8), d = (i % (HD / 8)) * 8;
      if (p.partial && p.x.world) {
        for (uint32_t r = 0; r < p.x.world; r++) {
          float* dst = xchg_row(p.x, r, (uint32_t)row);
          *reinterpret_cast<float4*>(dst + d) = make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(dst + d + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
          if (d == 0) *reinterpret_cast<float2*>(dst + HD) = make_float2(-INFINITY, 0.f);
        }
      } else if (p.partial) {
        float4* dst = reinterpret_cast<float4*>(p.part_o + row * HD + d);
        dst[0] = dst[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (d == 0) *reinterpret_cast<float2*>(p.part_ml + row * 2) = make_float2(-INFINITY, 0.f);
      } else {
        *reinterpret_cast<uint4*>(p.o + row * HD + d) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    if (p.partial && p.x.world) {
      __syncthreads();  // every thread's empty partials are written
      if (tid == 0)
        for (uint32_t hkv = 0; hkv < p.n_kv; hkv++) xchg_publish(p.x, b * p.n_kv + hkv);
    }
  }

  if (warp == NCW) {
    // ======================= producer warp =======================
    // Stages are numbered c = 0, 1, 2, ... (ring slot c % NST); consumer group
    // c & 1 takes stage c.  Every piece gets an even number of stages (an
    // empty one pads odd counts), so both groups see a first and a last stage
    // of every piece.
    const uint64_t policy = evict_first_policy();
    int slot = 0;
    uint32_t phase = 0;
    uint32_t n_issued = 0;  // stages armed so far (slot s armed ceil((n-s)/NST) times)
    bool aborted = false;

    // emits one piece: rows [t0, t1) of pair (b, hkv)
    // fused kv_append: the new row L-1 of kv head hkv of sequence b (lanes
    // 0-15: K, 16-31: V), written with generic stores; the TMA load of the
    // tile holding it must come after a proxy fence by the same lanes.  Any
    // wait in this warp stops this SM's stream, so the row's load is issued
    // one piece ahead, stored once the piece before has issued its stages,
    // and the fence sits just before the one tile that reads the row.
    struct PendRow {
      uint4 v;
      uint4* dst;
      bool valid, stored;
    };
    auto load_row = [&](uint32_t b, uint32_t hkv, uint32_t L, PendRow& r) {
      r.valid = r.stored = false;
      const int64_t row = seq_off(p, b) + (int64_t)L - 1;
      if (row >= 0 && (uint64_t)row < p.pool_rows) {
        const size_t dst = ((size_t)row * p.n_kv + hkv) * HD;
        const size_t src = ((size_t)b * p.n_kv + hkv) * HD;
        const int half = lane >> 4, j = lane & 15;
        r.dst = reinterpret_cast<uint4*>((half ? p.v_pool : p.k_pool) + dst) + j;
        r.v = __ldg(reinterpret_cast<const uint4*>((half ? p.v_new : p.k_new) + src) + j);
        r.valid = true;
      } else if (lane == 0) {
        atomicOr(&wsh->error, NWD_DEVERR_ROW_RANGE);
      }
    };
    auto store_row = [&](PendRow& r) {
      if (r.valid && !r.stored) {
        *r.dst = r.v;
        r.stored = true;
      }
    };

    // emits one piece: rows [t0, t1) of pair (b, hkv).  own: this piece's new
    // row (append mode, t1 == L), possibly loaded and stored by the piece
    // before; next: the next piece's new row (nb >= 0), loaded here and
    // stored after this piece's stages.
    auto emit_piece = [&](uint32_t b, uint32_t hkv, uint32_t L, uint32_t t0, uint32_t t1,
                          bool complete, int32_t f, int32_t l, PendRow& own, int32_t nb,
                          uint32_t nhkv, uint32_t nL, PendRow& next) {
      const int32_t pslot = (int32_t)(2u * blockIdx.x + (t0 > 0 ? 0u : 1u));
      const int64_t off = seq_off(p, b);
      if (lane == 0 && t0 == 0 && hkv == 0 && (off < 0 || (uint64_t)off + L > p.pool_rows))
        atomicOr(&wsh->error, NWD_DEVERR_ROW_RANGE);
      const bool ends = p.append && t1 == L;
      if (ends && !own.valid) load_row(b, hkv, L, own);
      if (nb >= 0) load_row((uint32_t)nb, nhkv, nL, next);
      const uint32_t nreal = cdiv(t1 - t0, TOK);
      const uint32_t nstages = (nreal + NGRP - 1u) / NGRP * NGRP;
      for (uint32_t s = 0; s < nstages && !aborted; s++) {
        if (!warp_wait(bar_empty + 8 * slot, phase ^ 1u, abort_flag, &wsh->error)) {
          aborted = true;
          break;
        }
        if (ends && s + 1 == nreal) {
          // the tile holding row L-1: the row's stores first, then the fence
          store_row(own);
          asm volatile("fence.proxy.async;" ::: "memory");
          __syncwarp();
        }
        if (lane == 0) {
          StageHdr h;
          h.b = (int32_t)b;
          h.hkv = (int32_t)hkv;
          h.t0 = (int32_t)(t0 + s * TOK);
          h.ntok = s < nreal ? (int32_t)min((uint32_t)TOK, t1 - (t0 + s * TOK)) : 0;
          h.flags = (s < (uint32_t)NGRP ? F_FIRST : 0) | (s + NGRP >= nstages ? F_LAST : 0) |
                    (complete ? F_COMPLETE : 0);
          h.slot = pslot;
          h.f = f;
          h.l = l;
          hdr[slot] = h;
          const uint32_t fb = bar_full + 8 * slot;
          if (h.ntok > 0) {
            const uint32_t qbytes = (s < (uint32_t)NGRP) ? G * HD * 2 : 0u;
            mbar_arrive_tx(fb, 2 * KV_BYTES + qbytes);
            const int row = (int)(off + (int64_t)h.t0);
            tma_load_4d(sbase + OFF_K + slot * KV_BYTES, &tmk, fb, 0, 0, (int)hkv, row, policy);
            tma_load_4d(sbase + OFF_V + slot * KV_BYTES, &tmv, fb, 0, 0, (int)hkv, row, policy);
            if (qbytes)
              bulk_load(sbase + OFF_Q + slot * Q_BYTES,
                        p.q + ((size_t)b * p.n_heads + (size_t)hkv * G) * HD, qbytes, fb);
          } else {
            mbar_arrive(fb);
          }
        }
        __syncwarp();
        n_issued++;
        if (++slot == NST) {
          slot = 0;
          phase ^= 1u;
        }
      }
      if (nb >= 0) store_row(next);  // long before the next piece's fence
    };

    if (split_k) {
      const uint32_t pair = blockIdx.x / split_k, j = blockIdx.x % split_k;
      if (pair < B * p.n_kv) {
        const uint32_t b = pair / p.n_kv, hkv = pair % p.n_kv;
        const uint32_t L = seq_rows(p, b);
        const uint32_t t0 = (uint32_t)((uint64_t)j * L / split_k);
        const uint32_t t1 = (uint32_t)((uint64_t)(j + 1) * L / split_k);
        PendRow own{}, next{};
        if (t1 > t0)
          emit_piece(b, hkv, L, t0, t1, split_k == 1, (int32_t)(pair * split_k),
                     (int32_t)(pair * split_k + split_k - 1), own, -1, 0u, 0u, next);
      }
    } else if (x0 < x1) {
      // Locate the first pair, then walk pairs forward.  A pair spans V range
      // items (pair_items) of which the first L are its rows; a range that
      // starts or ends in the remaining V - L items has no rows there.
      uint32_t b = find_seq(S, B, udiv64(x0, p.n_kv));
      uint32_t V = S[b + 1] - S[b];
      uint32_t L = seq_rows(p, b);
      const uint64_t r = x0 - (uint64_t)p.n_kv * S[b];
      uint32_t hkv = (uint32_t)udiv64(r, V);
      uint32_t t0 = (uint32_t)(r - (uint64_t)hkv * V);
      uint64_t pstart = x0 - t0;  // range position of the pair's row 0
      uint64_t x = x0;
      // the next pair of the walk (next kv head, or the next non-empty
      // sequence); only called while the range holds more items, so one exists
      auto next_pair = [&]() {
        if (++hkv == p.n_kv) {
          hkv = 0;
          do {
            b++;
          } while (b + 1 < B && S[b + 1] == S[b]);
          V = S[b + 1] - S[b];
          L = seq_rows(p, b);
        }
      };
      if (t0 >= L) {  // the range starts past the pair's rows
        x = pstart + V;
        if (x < x1) next_pair();
        pstart = x;
        t0 = 0;
      }
      int32_t f = (int32_t)udiv64(pstart, W);
      PendRow cur{}, nxt{};  // this piece's new row (set up by the piece before), the next one's
      while (x < x1 && !aborted) {
        const uint64_t len = min((uint64_t)(L - t0), x1 - x);
        const uint32_t t1 = t0 + (uint32_t)len;
        const bool complete = (t0 == 0 && t1 == L);
        const int32_t l = (t1 == L) ? (int32_t)blockIdx.x : (int32_t)udiv64(pstart + L - 1, W);
        // append mode: the next piece (the next non-empty pair, from its row
        // 0) ends at its new row if the range holds all of its rows
        int32_t nb = -1;
        uint32_t nhkv = 0, nL = 0;
        if (p.append && pstart + V < x1) {
          uint32_t b2 = b, h2 = hkv + 1, L2 = L;
          if (h2 == p.n_kv) {
            h2 = 0;
            do {
              b2++;
            } while (b2 + 1 < B && S[b2 + 1] == S[b2]);
            L2 = seq_rows(p, b2);
          }
          if (L2 > 0 && pstart + V + L2 <= x1) {
            nb = (int32_t)b2;
            nhkv = h2;
            nL = L2;
          }
        }
        nxt.valid = nxt.stored = false;
        emit_piece(b, hkv, L, t0, t1, complete, f, l, cur, nb, nhkv, nL, nxt);
        cur = nxt;
        // the range ends inside the pair's rows, or the pair is done: the
        // next pair starts V items after this one
        x = pstart + V;
        if (t1 < L || x >= x1) break;
        next_pair();
        pstart = x;
        t0 = 0;
        f = (int32_t)blockIdx.x;
      }
    }
    if (!aborted) {
      // one terminator stage per consumer group (the stage count is even here)
      for (int k = 0; k < NGRP && !aborted; k++) {
        if (warp_wait(bar_empty + 8 * slot, phase ^ 1u, abort_flag, &wsh->error)) {
          if (lane == 0) {
            hdr[slot].flags = F_TERM;
            mbar_arrive(bar_full + 8 * slot);
          }
          __syncwarp();
          n_issued++;
          if (++slot == NST) {
            slot = 0;
            phase ^= 1u;
          }
        } else {
          aborted = true;
        }
      }
    }
    if (aborted) {
      // leave only after this CTA's copies in flight have landed
      for (uint32_t s = 0; s < (uint32_t)NST; s++)
        if (n_issued > s) {
          const uint32_t times = (n_issued - s - 1u) / NST + 1u;
          const uint32_t par = (times - 1u) & 1u;
          const uint64_t t0 = globaltimer();
          while (!mbar_try_wait(bar_full + 8 * s, par) && globaltimer() - t0 < WAIT_LIMIT_NS) {
          }
        }
    }
    if (!p.cluster) return;
  } else {
  // ======================= consumer warps =======================
  const uint32_t grp = warp / WPG, wig = warp % WPG;  // group; 16-row slice of a stage
  const uint32_t g0 = 2u * (lane & 3);      // this lane's two heads (C/B fragment cols)
  const uint32_t rowq = lane >> 2;          // fragment row
  // ldmatrix lane roles
  const uint32_t li = lane >> 3, lr = lane & 7;
  const uint32_t tokK = wig * 16 + (li & 1) * 8 + lr;  // K: matrices (rows 0-7/8-15) x (k lo/hi)
  const uint32_t tokV = wig * 16 + (li >> 1) * 8 + lr; // V^T: (d lo/hi) x (tokens lo/hi)

  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float acc[8][4];
  uint32_t qf[8][2];
  // this group's stages: c = grp, grp + 2, ... -> ring slot and phase
  uint32_t slot = grp, phase = 0, cph = 0;
  float* mrg = reinterpret_cast<float*>(smem + OFF_MRG);
  float* mrg_m = mrg;                       // [NCW][GMAX]
  float* mrg_l = mrg + NCW * GMAX;          // [NCW][GMAX]
  float* mrg_acc = mrg + 2 * NCW * GMAX;    // [NCW][GMAX][HD]

  while (true) {
    // Consecutive uses of a ring slot alternate between the two groups (NST
    // is odd).  A parity wait cannot tell phase k from phase k+2, so first
    // wait until the slot's previous use (the other group's stage) has been
    // released: then the full barrier is at most one phase behind this wait.
    if (NGRP > 1 && !warp_wait(bar_empty + 8 * slot, phase ^ 1u, abort_flag, &wsh->error)) break;
    if (!warp_wait(bar_full + 8 * slot, phase, abort_flag, &wsh->error)) break;
    const StageHdr h = hdr[slot];
    if (h.flags & F_TERM) break;
    if (h.flags & F_FIRST) {
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; mt++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[mt][j] = 0.f;
      if (h.ntok > 0) {
        const uint8_t* qs = smem + OFF_Q + slot * Q_BYTES + rowq * (HD * 2) + g0 * 2;
        const bool live = rowq < G;
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          qf[ks][0] = live ? *reinterpret_cast<const uint32_t*>(qs + ks * 32) : 0u;
          qf[ks][1] = live ? *reinterpret_cast<const uint32_t*>(qs + ks * 32 + 16) : 0u;
        }
      }
    }
    const int valid = min(16, h.ntok - (int)wig * 16);
    if (valid > 0) {
      const uint32_t kb = sbase + OFF_K + slot * KV_BYTES;
      const uint32_t vb = sbase + OFF_V + slot * KV_BYTES;
      // Issue every shared-memory fragment load of the tile up front (K for
      // S^T = K Q^T, V^T for O^T += V^T P^T) so their latency overlaps the
      // QK MMAs and the softmax instead of sitting on the critical path.
      uint32_t ka[8][4], va[8][4];
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        const uint32_t R = 2u * tokK + (uint32_t)(ks >> 2);
        const uint32_t ch = (uint32_t)(ks & 3) * 2u + (li >> 1);
        ldsm_x4(kb + swz(R, ch), ka[ks][0], ka[ks][1], ka[ks][2], ka[ks][3]);
      }
#pragma unroll
      for (int mt = 0; mt < 8; mt++) {
        const uint32_t R = 2u * tokV + (uint32_t)(mt >> 2);
        const uint32_t ch = (uint32_t)(mt & 3) * 2u + (li & 1);
        ldsm_x4_t(vb + swz(R, ch), va[mt][0], va[mt][1], va[mt][2], va[mt][3]);
      }
      // ---- S^T[16 tokens][8 heads] = K Q^T (two accumulator chains) ----
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 8; ks++)
        mma16816((ks & 1) ? s1 : s0, ka[ks][0], ka[ks][1], ka[ks][2], ka[ks][3], qf[ks][0],
                 qf[ks][1]);
      float sr[4];
#pragma unroll
      for (int j = 0; j < 4; j++) sr[j] = s0[j] + s1[j];
      if ((int)rowq >= valid) sr[0] = sr[1] = -INFINITY;
      if ((int)rowq + 8 >= valid) sr[2] = sr[3] = -INFINITY;
      // ---- online softmax in the log2 domain, per head column ----
      // tile max of the raw scores; the scale is positive, so it commutes
      float mx0 = fmaxf(sr[0], sr[2]), mx1 = fmaxf(sr[1], sr[3]);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      mx0 *= p.scale_log2;
      mx1 *= p.scale_log2;
      // Lazy rescale: the reference max m only moves when a head's tile max
      // exceeds it by more than 2^RESCALE_LOG2, so P stays <= 2^8 and the
      // accumulators are rescaled rarely (the result o / l does not depend
      // on which m is used).
      const bool up0 = mx0 > m0 + RESCALE_LOG2, up1 = mx1 > m1 + RESCALE_LOG2;
      if (__any_sync(0xffffffffu, up0 || up1)) {
        const float al0 = up0 ? ex2(m0 - mx0) : 1.f;  // 0 while m is -inf
        const float al1 = up1 ? ex2(m1 - mx1) : 1.f;
        if (up0) m0 = mx0;
        if (up1) m1 = mx1;
        l0 *= al0;
        l1 *= al1;
#pragma unroll
        for (int mt = 0; mt < 8; mt++) {
          acc[mt][0] *= al0;
          acc[mt][1] *= al1;
          acc[mt][2] *= al0;
          acc[mt][3] *= al1;
        }
      }
      const float nb0 = m0 == -INFINITY ? 0.f : -m0;
      const float nb1 = m1 == -INFINITY ? 0.f : -m1;
      const float p0 = ex2(fmaf(sr[0], p.scale_log2, nb0));
      const float p1 = ex2(fmaf(sr[1], p.scale_log2, nb1));
      const float p2 = ex2(fmaf(sr[2], p.scale_log2, nb0));
      const float p3 = ex2(fmaf(sr[3], p.scale_log2, nb1));
      l0 += p0 + p2;
      l1 += p1 + p3;
      // ---- P^T fragments for the PV MMA ----
      // P is split into an fp16 head and an fp16 remainder (p = hi + lo to
      // ~22 bits): a single fp16 rounding of P (2^-11 relative) would exceed
      // the parity tolerance on outputs near zero.
      const __half2 h01 = __floats2half2_rn(p0, p1), h23 = __floats2half2_rn(p2, p3);
      const __half2 r01 = __floats2half2_rn(p0 - __low2float(h01), p1 - __high2float(h01));
      const __half2 r23 = __floats2half2_rn(p2 - __low2float(h23), p3 - __high2float(h23));
      const uint32_t pb0 = movmatrix_t(*reinterpret_cast<const uint32_t*>(&h01));
      const uint32_t pb1 = movmatrix_t(*reinterpret_cast<const uint32_t*>(&h23));
      const uint32_t pl0 = movmatrix_t(*reinterpret_cast<const uint32_t*>(&r01));
      const uint32_t pl1 = movmatrix_t(*reinterpret_cast<const uint32_t*>(&r23));
      if (valid < 16) {
        // rows past `valid` may hold stale or foreign data: zero them in V^T
        const int te = (int)g0;  // tokens te, te+1 (regs 0,1) and te+8, te+9 (regs 2,3)
        const uint32_t mlo = (te < valid ? 0x0000ffffu : 0u) | (te + 1 < valid ? 0xffff0000u : 0u);
        const uint32_t mhi =
            (te + 8 < valid ? 0x0000ffffu : 0u) | (te + 9 < valid ? 0xffff0000u : 0u);
#pragma unroll
        for (int mt = 0; mt < 8; mt++) {
          va[mt][0] &= mlo;
          va[mt][1] &= mlo;
          va[mt][2] &= mhi;
          va[mt][3] &= mhi;
        }
      }
      // ---- O^T[128 dims][8 heads] += V^T P^T ----
#pragma unroll
      for (int mt = 0; mt < 8; mt++)
        mma16816(acc[mt], va[mt][0], va[mt][1], va[mt][2], va[mt][3], pb0, pb1);
#pragma unroll
      for (int mt = 0; mt < 8; mt++)
        mma16816(acc[mt], va[mt][0], va[mt][1], va[mt][2], va[mt][3], pl0, pl1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * slot);
    slot += NGRP;
    if (slot >= NST) {
      slot -= NST;
      phase ^= 1u;
    }
    if (!(h.flags & F_LAST)) continue;

    // ======== end of piece: merge the eight warps, then emit ========
    float lt0 = l0, lt1 = l1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      lt0 += __shfl_xor_sync(0xffffffffu, lt0, o);
      lt1 += __shfl_xor_sync(0xffffffffu, lt1, o);
    }
    if (lane < 4) {
      mrg_m[warp * GMAX + g0] = m0;
      mrg_m[warp * GMAX + g0 + 1] = m1;
      mrg_l[warp * GMAX + g0] = lt0;
      mrg_l[warp * GMAX + g0 + 1] = lt1;
    }
    {
      float* a = mrg_acc + (size_t)warp * GMAX * HD;
#pragma unroll
      for (int mt = 0; mt < 8; mt++) {
        const uint32_t d = mt * 16 + rowq;
        a[g0 * HD + d] = acc[mt][0];
        a[(g0 + 1) * HD + d] = acc[mt][1];
        a[g0 * HD + d + 8] = acc[mt][2];
        a[(g0 + 1) * HD + d + 8] = acc[mt][3];
      }
    }
    if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;
    // NCW*32 threads: head g, dims d0 .. d0+DPT-1
    constexpr int DPT = C::DPT, NV = DPT / 4;
    const uint32_t ct = warp * 32 + lane;
    const uint32_t g = ct / (HD / DPT), d0 = (ct % (HD / DPT)) * DPT;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NCW; w++) M = fmaxf(M, mrg_m[w * GMAX + g]);
    float Ls = 0.f;
    float4 o4[NV];
#pragma unroll
    for (int j = 0; j < NV; j++) o4[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < NCW; w++) {
      const float mw = mrg_m[w * GMAX + g];
      const float f = mw == -INFINITY ? 0.f : ex2(mw - M);
      Ls += f * mrg_l[w * GMAX + g];
      const float4* a = reinterpret_cast<const float4*>(mrg_acc + ((size_t)w * GMAX + g) * HD + d0);
#pragma unroll
      for (int j = 0; j < NV; j++) {
        const float4 x = a[j];
        o4[j].x += f * x.x;
        o4[j].y += f * x.y;
        o4[j].z += f * x.z;
        o4[j].w += f * x.w;
      }
    }
    if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;  // scratch free again

    if (p.cluster) {
      // one piece per CTA: keep its (m, l, o) per head in shared memory at the
      // same offsets in every CTA of the cluster (row g of [GMAX][HD + 4]:
      // o, then m, l); the cluster merges them after the loop
      if (g < G) {
        float* row = mrg + (size_t)g * (HD + 4);
        float4* dst = reinterpret_cast<float4*>(row + d0);
#pragma unroll
        for (int j = 0; j < NV; j++) dst[j] = o4[j];
        if (d0 == 0) *reinterpret_cast<float2*>(row + HD) = make_float2(M, Ls);
      }
      continue;
    }

    const uint32_t b = (uint32_t)h.b, hkv = (uint32_t)h.hkv;
    bool emit = (h.flags & F_COMPLETE) != 0;
    if (!emit) {
      // partial piece: publish it, take a ticket on the pair; the last of the
      // pair's l - f + 1 pieces merges them in range order
      if (g < G) {
        const size_t sl = (size_t)h.slot * G + g;
        if (d0 == 0) *reinterpret_cast<float2*>(ws_ml + sl * 2) = make_float2(M, Ls);
        float4* dst = reinterpret_cast<float4*>(ws_o + sl * HD + d0);
#pragma unroll
        for (int j = 0; j < NV; j++) dst[j] = o4[j];
      }
      // The consumer barrier orders every thread's partial before thread 0's
      // ticket, whose release (gpu scope, cumulative) publishes them; the
      // ticket's acquire and the barrier after it order the last CTA's loads
      // of the other pieces after their publication.
      if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;
      if (ct == 0) {
        const uint32_t t = atom_add_acq_rel_gpu(&tickets[b * p.n_kv + hkv], 1u);
        misc->last = (t == (uint32_t)(h.l - h.f)) ? 1 : 0;
      }
      if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;
      emit = misc->last != 0;
      if (emit) {
        if (g < G) {
          // one online pass over the pieces, MB pieces' loads in flight per
          // thread (the merge is L2-latency bound, not bandwidth bound, so
          // every batch is one round trip): a single sequence over 8 kv heads
          // has at most 20 pieces per pair, two batches; MB is the most that
          // stays within registers
          constexpr int MB = NV == 1 ? 12 : 10;
          M = -INFINITY;
          Ls = 0.f;
#pragma unroll
          for (int j = 0; j < NV; j++) o4[j] = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int32_t c0 = h.f; c0 <= h.l; c0 += MB) {
            float2 ml[MB];
            float4 x[MB][NV];
#pragma unroll
            for (int j = 0; j < MB; j++) {
              const int32_t c = c0 + j;
              if (c <= h.l) {
                // CTA f holds the pair's head in its tail slot; later CTAs in their head slot
                const size_t sl = (size_t)(2 * c + (c == h.f ? 1 : 0)) * G + g;
                ml[j] = __ldcg(reinterpret_cast<const float2*>(ws_ml + sl * 2));
                const float4* src = reinterpret_cast<const float4*>(ws_o + sl * HD + d0);
#pragma unroll
                for (int v = 0; v < NV; v++) x[j][v] = __ldcg(src + v);
              } else {
                ml[j] = make_float2(-INFINITY, 0.f);
#pragma unroll
                for (int v = 0; v < NV; v++) x[j][v] = make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
#pragma unroll
            for (int j = 0; j < MB; j++) {
              if (ml[j].x == -INFINITY) continue;  // empty piece
              const float Mn = fmaxf(M, ml[j].x);
              const float a = ex2(M - Mn);  // 0 while M is -inf
              const float f = ex2(ml[j].x - Mn);
              Ls = Ls * a + f * ml[j].y;
#pragma unroll
              for (int v = 0; v < NV; v++) {
                o4[v].x = o4[v].x * a + f * x[j][v].x;
                o4[v].y = o4[v].y * a + f * x[j][v].y;
                o4[v].z = o4[v].z * a + f * x[j][v].z;
                o4[v].w = o4[v].w * a + f * x[j][v].w;
              }
              M = Mn;
            }
          }
        }
        if (ct == 0) tickets[b * p.n_kv + hkv] = 0u;
      }
      // misc->last is reused by the next piece
      if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;
    }
    if (emit && g < G) {
      const size_t row = (size_t)b * p.n_heads + (size_t)hkv * G + g;
      if (p.partial && p.x.world) {
        // the pair's partial straight into every rank's exchange slot
        for (uint32_t r = 0; r < p.x.world; r++) {
          float* dst = xchg_row(p.x, r, (uint32_t)row);
          if (d0 == 0) *reinterpret_cast<float2*>(dst + HD) = make_float2(M, Ls);
#pragma unroll
          for (int j = 0; j < NV; j++) *reinterpret_cast<float4*>(dst + d0 + 4 * j) = o4[j];
        }
      } else if (p.partial) {
        if (d0 == 0) *reinterpret_cast<float2*>(p.part_ml + row * 2) = make_float2(M, Ls);
        float4* dst = reinterpret_cast<float4*>(p.part_o + row * HD + d0);
#pragma unroll
        for (int j = 0; j < NV; j++) dst[j] = o4[j];
      } else {
        const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
#pragma unroll
        for (int j = 0; j < NV; j++) {
          uint2 v;
          v.x = pack_half2(o4[j].x * inv, o4[j].y * inv);
          v.y = pack_half2(o4[j].z * inv, o4[j].w * inv);
          *reinterpret_cast<uint2*>(p.o + row * HD + d0 + 4 * j) = v;
        }
      }
    }
    if (emit && p.partial && p.x.world) {
      // every thread's stores of the pair's partial, then its flag on every rank
      if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;
      if (ct == 0) xchg_publish(p.x, b * p.n_kv + hkv);
    }
  }
  }  // consumer warps

  if (p.cluster) {
    // ======== the cluster's pieces meet over distributed shared memory ========
    // Every thread of every CTA of the cluster (producer warp included) comes
    // here exactly once, whether its loop ended normally or gave up on a wait
    // (then the partial is stale, and the workspace's error word says so).
    // The first barrier publishes each CTA's partial to the cluster; the
    // second keeps every CTA resident until the others have read it.
    cluster_sync_all();
    const uint32_t C = p.cluster, rank = blockIdx.x % C, hkv = blockIdx.x / C;
    const float* mrg = reinterpret_cast<const float*>(smem + OFF_MRG);
    for (uint32_t i = rank * NTHR + tid; i < G * (HD / 4); i += C * NTHR) {
      const uint32_t g = i / (HD / 4), d = (i % (HD / 4)) * 4;
      const float* row = mrg + (size_t)g * (HD + 4);
      float2 ml[16];
      float M = -INFINITY;
#pragma unroll
      for (uint32_t c = 0; c < 16; c++) {
        ml[c] = c < C ? ld_cluster_f2(row + HD, c) : make_float2(-INFINITY, 0.f);
        M = fmaxf(M, ml[c].x);
      }
      float Ls = 0.f;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      // pieces in rank order (= row order): deterministic
#pragma unroll
      for (uint32_t c = 0; c < 16; c++) {
        if (c >= C || ml[c].x == -INFINITY) continue;
        const float w = ex2(ml[c].x - M);
        const float4 x = ld_cluster_f4(row + d, c);
        Ls += w * ml[c].y;
        o.x += w * x.x;
        o.y += w * x.y;
        o.z += w * x.z;
        o.w += w * x.w;
      }
      const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
      uint2 v;
      v.x = pack_half2(o.x * inv, o.y * inv);
      v.y = pack_half2(o.z * inv, o.w * inv);
      *reinterpret_cast<uint2*>(p.o + ((size_t)hkv * G + g) * HD + d) = v;
    }
    cluster_sync_all();
  }
}

// ---------------- host side ----------------
// Work-split policy.  When every (sequence, kv head) pair has at most
// pair_max rows and there are no more pairs than SMs, each pair gets its own
// CTA (no partials, lowest latency).  Otherwise each CTA's range holds at
// least min_chunk (row, kv head) items, so small problems use fewer CTAs
// instead of many tiny partials.
struct Tuning {
  uint32_t min_chunk = 256;
  uint32_t pair_max = 512;
  uint32_t groups = 0;  // consumer groups: 0 = by problem size, else 1 or 2
  // single sequence: two consumer groups from this many rows (config 2 at
  // 4 096 rows, clustered: 10.07 us with two groups, 10.32 with one)
  uint32_t two_group_rows = 4096;
  uint32_t short_rows = 2048;  // single sequence of at most this many rows: decode_short.cu
  uint32_t short_cta_rows = 128;  // past 256 rows: rows per CTA of a kv head's cluster
  // Single sequence: K/V tiles per CTA prefetched into L2 under PDL, at most
  // prefetch and 1 / prefetch_div of the CTA's tiles (clustered launches: 8
  // and a quarter).  Config 2, per step: a quarter / 8 gave 10.30, 17.45 and
  // 25.28 us at 4 096, 16 384 and 32 768 rows; half / 16 gave 10.39, 17.09
  // and 25.02 us (4 096 rows runs clustered); all / 32: 10.73, 18.21, 26.93.
  uint32_t prefetch = 16;
  uint32_t prefetch_div = 2;
  // single sequence split into k pieces per kv head: run each kv head's pieces
  // as one thread-block cluster (at most cluster_max CTAs, 16 needs the
  // non-portable opt-in) that merges over distributed shared memory; 0 turns
  // it off.  Up to cluster_rows rows any size whose clusters all fit at once
  // is taken (the merge it saves outweighs fewer CTAs: 8 kv heads at 4 096
  // rows, 80 CTAs in clusters of 10 against 128 unclustered, 10.5 against
  // 11.6 us); above, only one keeping cluster_keep / 8 of the k CTAs (16 384
  // rows in clusters of 10: 18.2 against 17.8 us, 32 768: 29.5 against 26.0).
  uint32_t cluster_max = 16;
  uint32_t cluster_rows = 8192;
  uint32_t cluster_keep = 7;
  // Batches: the flattened split charges each (sequence, kv head) pair its
  // rows plus pair_cost, rounded up to whole pairs of stages (pair_pad 1), so
  // every CTA issues the same number of stages and a CTA whose range holds
  // many pairs takes fewer rows for their fixed costs (first stage, epilogue,
  // output or partial write).  Config 3 (256 sequences of 512-8 192 rows) per
  // step: 708 us cut at any row (pair_pad 0: equal rows, up to 4 % more
  // stages on a CTA holding many pair ends), 702 us padded, 688-691 us with
  // a cost of 192-384 rows, 697 / 711 us at 512 / 1 024.
  uint32_t pair_cost = 256;
  uint32_t pair_pad = 1;
};

uint32_t env_u32(const char* name, uint32_t dflt) {
  const char* s = getenv(name);
  if (!s || !*s) return dflt;
  long v = strtol(s, nullptr, 10);
  return v > 0 ? (uint32_t)v : dflt;
}

const Tuning& tuning() {
  static Tuning t = [] {
    Tuning x;
    x.min_chunk = env_u32("NWD_DECODE_MIN_CHUNK", x.min_chunk);
    x.pair_max = env_u32("NWD_DECODE_PAIR_MAX", x.pair_max);
    // 0 charges pairs their rows alone
    const char* pc = getenv("NWD_DECODE_PAIR_COST");
    if (pc && *pc) x.pair_cost = (uint32_t)std::min<unsigned long>(strtoul(pc, nullptr, 10), 65536ul);
    const char* pp = getenv("NWD_DECODE_PAIR_PAD");
    if (pp && *pp) x.pair_pad = strtoul(pp, nullptr, 10) ? 1u : 0u;
    x.groups = env_u32("NWD_DECODE_GROUPS", x.groups);
    if (x.groups > 2) x.groups = 2;
    x.two_group_rows = env_u32("NWD_DECODE_TWO_GROUP_ROWS", x.two_group_rows);
    // 0 turns the short-sequence kernel off
    const char* sr = getenv("NWD_DECODE_SHORT_ROWS");
    if (sr && *sr) x.short_rows = (uint32_t)strtoul(sr, nullptr, 10);
    if (x.short_rows > nwd::decode_short_max_rows()) x.short_rows = nwd::decode_short_max_rows();
    x.short_cta_rows = env_u32("NWD_DECODE_SHORT_CTA_ROWS", x.short_cta_rows);
    // 0 turns the prefetch off
    const char* pf = getenv("NWD_DECODE_PREFETCH");
    if (pf && *pf) x.prefetch = (uint32_t)strtoul(pf, nullptr, 10);
    x.prefetch_div = env_u32("NWD_DECODE_PREFETCH_DIV", x.prefetch_div);
    // 0 turns the cluster merge off
    const char* cl = getenv("NWD_DECODE_CLUSTER");
    if (cl && *cl) x.cluster_max = (uint32_t)strtoul(cl, nullptr, 10);
    if (x.cluster_max > 16) x.cluster_max = 16;
    x.cluster_rows = env_u32("NWD_DECODE_CLUSTER_ROWS", x.cluster_rows);
    const char* ck = getenv("NWD_DECODE_CLUSTER_KEEP");
    if (ck && *ck) x.cluster_keep = (uint32_t)strtoul(ck, nullptr, 10);
    if (x.cluster_keep > 8) x.cluster_keep = 8;
    return x;
  }();
  return t;
}

// Partial slots: two per CTA (a range has at most a head and a tail piece).
uint32_t slots_for(const nwd::DeviceInfo& di) { return 2u * (uint32_t)di.sm_count; }

bool g_smem_set[64][3] = {};

// Clusters of c CTAs of decode_kernel<NG> that can be resident at once on
// the current device (cudaOccupancyMaxActiveClusters), cached per device;
// 0 if the size cannot be launched.
int g_cluster_fit[64][3][17];
bool g_cluster_known[64][3][17] = {};
std::mutex g_cluster_mu;

template <int NG>
int cluster_fit(int device, uint32_t c, uint32_t n_kv) {
  std::lock_guard<std::mutex> lk(g_cluster_mu);
  if (g_cluster_known[device][NG][c]) return g_cluster_fit[device][NG][c];
  int n = 0;
  cudaError_t e = cudaSuccess;
  if (c > 8)
    e = cudaFuncSetAttribute(decode_kernel<NG>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c * n_kv);
    cfg.blockDim = dim3(Cfg<NG>::NTHR);
    cfg.dynamicSmemBytes = Cfg<NG>::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaOccupancyMaxActiveClusters(&n, decode_kernel<NG>, &cfg);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();  // not launchable at this size: clear the sticky-free error
    n = 0;
  }
  g_cluster_fit[device][NG][c] = n;
  g_cluster_known[device][NG][c] = true;
  return n;
}

template <int NG>
cudaError_t launch_cluster(uint32_t grid, uint32_t c, cudaStream_t stream, const CUtensorMap& tmk,
                           const CUtensorMap& tmv, const Params& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg<NG>::NTHR);
  cfg.dynamicSmemBytes = Cfg<NG>::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = c;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, decode_kernel<NG>, tmk, tmv, p);
}

struct Call {
  const uint16_t* q;
  const uint16_t* k_new;
  const uint16_t* v_new;
  const uint16_t* k_pool;
  const uint16_t* v_pool;
  uint64_t pool_rows;
  const int64_t* row_offset;
  const int32_t* seq_len;
  int32_t single_len;
  uint16_t* o;
  float* part_o;
  float* part_ml;
  uint32_t batch, n_heads, n_kv, hd;
  float scale;
  bool append, partial;
  void* ws;
  size_t ws_bytes;
  void* stream;
  const char* who;
  const nwd::XchgDesc* x;  // partial mode only: push to the exchange buffers
};

int check_shape(uint32_t n_heads, uint32_t n_kv, uint32_t hd, const char* who) {
  using namespace nwd;
  if (n_heads == 0 || n_kv == 0 || hd == 0)
    return fail(NWD_ERR_INVALID, "%s: n_heads, n_kv_heads and head_dim must be > 0", who);
  if (n_heads % n_kv != 0)
    return fail(NWD_ERR_INVALID, "%s: n_heads %u is not a multiple of n_kv_heads %u", who, n_heads,
                n_kv);
  if (hd != HD) return fail(NWD_ERR_UNSUPPORTED, "%s: head_dim %u (only 128 is supported)", who, hd);
  if (n_heads / n_kv > GMAX)
    return fail(NWD_ERR_UNSUPPORTED, "%s: group %u > %d", who, n_heads / n_kv, GMAX);
  return NWD_OK;
}

// A single sequence of at most tu.short_rows rows (not a shard partial) runs
// on decode_short_kernel, which uses no workspace.
bool takes_short_path(const Call& c, const Tuning& tu) {
  return !c.seq_len && !c.partial && c.single_len >= 1 &&
         (uint32_t)c.single_len <= tu.short_rows;
}

// How a split-KV launch is cut: grid, pieces per kv head of a single
// sequence (0 = the flattened stream-K split), CTAs per cluster (0 = none),
// consumer groups.  Sets the kernel's shared-memory attribute on first use.
struct Plan {
  uint32_t grid, split_k, cluster, ng;
};

int plan_split(const Call& c, const nwd::DeviceInfo& di, const Tuning& tu, Plan* out) {
  using namespace nwd;
  const uint32_t grid_max = (uint32_t)di.sm_count;
  // grid: one CTA per SM; for a single sequence (rows known here) one CTA per
  // kv head when the sequence is short, else only as many CTAs as ranges of
  // min_chunk items
  uint32_t grid = grid_max;
  uint32_t split_k = 0;
  if (!c.seq_len) {
    // single sequence: cut each kv head's rows into k equal pieces, one CTA
    // each (k = 1 for short sequences: no partials), so no CTA straddles two
    // heads; fall back to the flattened split when there are more kv heads
    // than SMs
    const uint64_t rows = (uint64_t)(c.single_len > 0 ? c.single_len : 0);
    if (c.n_kv <= grid_max) {
      uint64_t k = 1;
      if (rows > tu.pair_max) {
        k = std::min<uint64_t>(grid_max / c.n_kv, (rows + tu.min_chunk - 1) / tu.min_chunk);
        if (k < 1) k = 1;
      }
      split_k = (uint32_t)k;
      grid = c.n_kv * (uint32_t)k;
    } else {
      const uint64_t need = (c.n_kv * rows + tu.min_chunk - 1) / tu.min_chunk;
      if (need < grid) grid = (uint32_t)need;
    }
  }
  if (grid == 0) grid = 1;
  // Consumer groups: two (latency hiding) for batched calls and long single
  // sequences, one for short single sequences (its epilogue is shorter).
  uint32_t ng = tu.groups;
  if (ng == 0) ng = (c.seq_len || (uint64_t)c.single_len >= tu.two_group_rows) ? 2u : 1u;
  if (!g_smem_set[di.device][ng]) {
    cudaError_t e = ng == 2 ? cudaFuncSetAttribute(decode_kernel<2>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   Cfg<2>::SMEM_BYTES)
                            : cudaFuncSetAttribute(decode_kernel<1>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   Cfg<1>::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_kernel)");
    g_smem_set[di.device][ng] = true;
  }
  // A single sequence cut into k >= 2 pieces per kv head (not a shard
  // partial): each kv head's pieces run as one cluster and merge over
  // distributed shared memory instead of workspace partials and a ticket.
  // The largest size (at most k) whose n_kv clusters can all be resident at
  // once; past cluster_rows rows only if it keeps at least cluster_keep / 8
  // of the k CTAs per kv head (long sequences stream faster on more CTAs);
  // none fits, the split stays as it is.
  uint32_t cluster = 0;
  if (!c.seq_len && !c.partial && split_k >= 2 && tu.cluster_max >= 2) {
    const uint32_t keep = (uint64_t)c.single_len <= tu.cluster_rows ? 0u : tu.cluster_keep;
    uint32_t C = std::min(split_k, tu.cluster_max);
    while (C >= 2 && 8u * C >= keep * split_k) {
      const int fit = ng == 2 ? cluster_fit<2>(di.device, C, c.n_kv)
                              : cluster_fit<1>(di.device, C, c.n_kv);
      if (fit >= (int)c.n_kv) break;
      C--;
    }
    if (C >= 2 && 8u * C >= keep * split_k) {
      cluster = C;
      split_k = C;
      grid = c.n_kv * C;
    }
  }
  out->grid = grid;
  out->split_k = split_k;
  out->cluster = cluster;
  out->ng = ng;
  return NWD_OK;
}

int launch(const Call& c) {
  using namespace nwd;
  int st = check_shape(c.n_heads, c.n_kv, c.hd, c.who);
  if (st) return st;
  if (!c.q || !c.k_pool || !c.v_pool || (!c.partial && !c.o) ||
      (c.partial && !c.x && (!c.part_o || !c.part_ml)) || (c.append && (!c.k_new || !c.v_new)))
    return fail(NWD_ERR_INVALID, "%s: null pointer", c.who);
  if (!aligned16(c.q) || !aligned16(c.k_pool) || !aligned16(c.v_pool) ||
      (c.o && !aligned16(c.o)) || (c.part_o && !aligned16(c.part_o)) ||
      (c.part_ml && ((uintptr_t)c.part_ml & 7u)) || (c.k_new && !aligned16(c.k_new)) ||
      (c.v_new && !aligned16(c.v_new)))
    return fail(NWD_ERR_INVALID, "%s: tensors must be 16-byte aligned", c.who);
  if (c.batch > (uint32_t)MAXB)
    return fail(NWD_ERR_UNSUPPORTED, "%s: batch %u > %d per call", c.who, c.batch, MAXB);
  if (c.pool_rows == 0 || c.pool_rows > (1ull << 31))
    return fail(NWD_ERR_INVALID, "%s: pool rows %llu outside [1, 2^31]", c.who,
                (unsigned long long)c.pool_rows);
  DeviceInfo di;
  st = current_device_info(&di);
  if (st) return st;
  const Tuning& tu = tuning();
  const uint32_t G = c.n_heads / c.n_kv;
  const WsLayout lay = ws_layout(c.batch, c.n_kv, G, c.hd, slots_for(di));
  if (!c.ws) return fail(NWD_ERR_WORKSPACE, "%s: workspace is NULL", c.who);
  if (c.ws_bytes < lay.total)
    return fail(NWD_ERR_WORKSPACE, "%s: workspace of %zu bytes < %zu required", c.who, c.ws_bytes,
                lay.total);
  if ((uintptr_t)c.ws & 255u)
    return fail(NWD_ERR_WORKSPACE, "%s: workspace must be 256-byte aligned", c.who);
  if (c.batch == 0) return ok();
  if (!(c.scale >= 0.f) || isinf(c.scale))
    return fail(NWD_ERR_INVALID, "%s: scale must be finite and >= 0 (0 = 1/sqrt(head_dim))", c.who);

  // one short sequence: a cluster of CTAs per kv head (no workspace use)
  if (takes_short_path(c, tu)) {
    const float sc = c.scale != 0.f ? c.scale : 1.0f / sqrtf((float)c.hd);
    return launch_decode_short(c.q, c.k_new, c.v_new, const_cast<uint16_t*>(c.k_pool),
                               const_cast<uint16_t*>(c.v_pool), c.o, (uint32_t)c.single_len,
                               c.n_kv, G, sc * 1.4426950408889634f, c.append, tu.short_cta_rows,
                               c.stream, c.who);
  }

  CUtensorMap tmk, tmv;
  st = kv_tensor_map(&tmk, c.k_pool, c.pool_rows, c.n_kv, c.hd, TOK);
  if (st) return st;
  st = kv_tensor_map(&tmv, c.v_pool, c.pool_rows, c.n_kv, c.hd, TOK);
  if (st) return st;

  Params p;
  memset(&p, 0, sizeof(p));
  p.q = reinterpret_cast<const __half*>(c.q);
  p.k_new = reinterpret_cast<const __half*>(c.k_new);
  p.v_new = reinterpret_cast<const __half*>(c.v_new);
  p.k_pool = const_cast<__half*>(reinterpret_cast<const __half*>(c.k_pool));
  p.v_pool = const_cast<__half*>(reinterpret_cast<const __half*>(c.v_pool));
  p.o = reinterpret_cast<__half*>(c.o);
  p.part_o = c.part_o;
  p.part_ml = c.part_ml;
  p.row_offset = c.row_offset;
  p.seq_len = c.seq_len;
  p.single_len = c.single_len;
  p.ws = reinterpret_cast<uint8_t*>(c.ws);
  p.pool_rows = c.pool_rows;
  p.tickets_off = lay.tickets_off;
  p.ml_off = lay.ml_off;
  p.o_off = lay.o_off;
  p.nslots = lay.max_units;
  p.batch = c.batch;
  p.n_heads = c.n_heads;
  p.n_kv = c.n_kv;
  p.group = G;
  if (!(c.scale >= 0.f) || isinf(c.scale))
    return fail(NWD_ERR_INVALID, "%s: scale must be finite and >= 0 (0 = 1/sqrt(head_dim))", c.who);
  const float scale = c.scale != 0.f ? c.scale : 1.0f / sqrtf((float)c.hd);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.append = c.append ? 1u : 0u;
  p.partial = c.partial ? 1u : 0u;
  if (c.x) p.x = *c.x;  // memset above leaves world = 0 otherwise
  p.min_chunk = tu.min_chunk;

  p.pair_max = tu.pair_max;

  Plan pl;
  st = plan_split(c, di, tu, &pl);
  if (st) return st;
  p.split_k = pl.split_k;
  p.cluster = pl.cluster;
  p.prefetch = pl.cluster ? std::min(tu.prefetch, 8u) : tu.prefetch;
  p.prefetch_div = pl.cluster ? 4u : tu.prefetch_div;
  // batches: pieces cut at whole pairs of stages (NG stages: one per group),
  // each pair charged pair_cost items on top of its rows
  p.pair_pad = c.seq_len && tu.pair_pad ? (uint32_t)TOK * pl.ng : 1u;
  p.pair_cost = c.seq_len ? tu.pair_cost : 0u;
  const uint32_t grid = pl.grid, ng = pl.ng;
  cudaError_t e;
  if (p.cluster)
    e = ng == 2 ? launch_cluster<2>(grid, p.cluster, (cudaStream_t)c.stream, tmk, tmv, p)
                : launch_cluster<1>(grid, p.cluster, (cudaStream_t)c.stream, tmk, tmv, p);
  else
    e = ng == 2 ? launch_pdl(decode_kernel<2>, dim3(grid), dim3(Cfg<2>::NTHR), Cfg<2>::SMEM_BYTES,
                             (cudaStream_t)c.stream, tmk, tmv, p)
                : launch_pdl(decode_kernel<1>, dim3(grid), dim3(Cfg<1>::NTHR), Cfg<1>::SMEM_BYTES,
                             (cudaStream_t)c.stream, tmk, tmv, p);
  if (e != cudaSuccess) return cuda_fail(e, c.who);
  return ok();
}

// ---- scratch for nwd_attn_decode_noalloc ----
// Callers that cannot allocate device memory get the decode's scratch (work
// header, merge tickets, partial slots) from this file-scope array instead of
// a caller workspace.  Its size covers one sequence with up to
// NOALLOC_MAX_KV_HEADS kv heads, a GQA group up to GMAX and up to
// NOALLOC_MAX_SMS SMs (two partial slots per SM).  Every GPU that loads the
// library holds it until the process exits.
constexpr uint32_t NOALLOC_MAX_KV_HEADS = 64;
constexpr uint32_t NOALLOC_MAX_SMS = 160;
constexpr size_t NOALLOC_BYTES =
    256 /* header */ + 256 /* tickets: 64 kv heads x 4 B */ +
    (size_t)2 * NOALLOC_MAX_SMS * GMAX * 2 * sizeof(float) /* (m, l) per slot and head */ +
    (size_t)2 * NOALLOC_MAX_SMS * GMAX * HD * sizeof(float) /* o per slot and head */;
__device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch on the current device.  Host code only sees
// a host-side stand-in for a __device__ array, so the address is looked up
// with the device current.  It is looked up again on every call made outside
// stream capture (a cheap query once the module is loaded, and it stays right
// after a cudaDeviceReset reloads the module); a call made while `stream` is
// being captured reuses the address of the device's last uncaptured call,
// since the first lookup may load the module, which capture does not allow.
int noalloc_scratch(int device, void* stream, void** out) {
  using namespace nwd;
  if (device < 0 || device >= NOALLOC_MAX_DEVICES)
    return fail(NWD_ERR_UNSUPPORTED, "built-in decode scratch: device %d >= %d", device,
                NOALLOC_MAX_DEVICES);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing((cudaStream_t)stream, &cap);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
    g_noalloc_ptr[device] = ptr;
  } else if (!g_noalloc_ptr[device]) {
    return fail(NWD_ERR_CUDA,
                "built-in decode scratch: the first call on device %d was made during stream "
                "capture; make one call before capturing",
                device);
  }
  *out = g_noalloc_ptr[device];
  return NWD_OK;
}

}  // namespace

using namespace nwd;

namespace nwd {

int decode_partial_xchg(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                        uint64_t pool_rows, const int64_t* row_offset, const int32_t* seq_len,
                        uint32_t batch, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim,
                        float scale, void* workspace, size_t ws_bytes, void* stream,
                        const XchgDesc& x) {
  if (!row_offset || !seq_len) return fail(NWD_ERR_INVALID, "decode_partial_xchg: null pointer");
  if (x.world == 0 || x.world > (uint32_t)XCH_MAX_RANKS || x.rank >= x.world || x.epoch == 0 ||
      x.R != batch * n_heads || x.P != batch * n_kv)
    return fail(NWD_ERR_INVALID, "decode_partial_xchg: exchange descriptor does not match");
  for (uint32_t r = 0; r < x.world; r++)
    if (!x.data[r] || !x.flags[r] || !aligned16(x.data[r]))
      return fail(NWD_ERR_INVALID, "decode_partial_xchg: exchange buffer %u missing", r);
  Call c{};
  c.q = q; c.k_pool = k_pool; c.v_pool = v_pool; c.pool_rows = pool_rows;
  c.row_offset = row_offset; c.seq_len = seq_len; c.batch = batch; c.n_heads = n_heads;
  c.n_kv = n_kv; c.hd = head_dim; c.scale = scale; c.partial = true; c.ws = workspace;
  c.ws_bytes = ws_bytes; c.stream = stream; c.who = "nwd_mgpu_decode_step"; c.x = &x;
  return launch(c);
}

}  // namespace nwd

extern "C" {

int nwd_attn_decode_workspace_size(uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                                   uint32_t head_dim, size_t* bytes) {
  if (!bytes) return fail(NWD_ERR_INVALID, "nwd_attn_decode_workspace_size: bytes is NULL");
  int st = check_shape(n_heads, n_kv_heads, head_dim, "nwd_attn_decode_workspace_size");
  if (st) return st;
  DeviceInfo di;
  st = current_device_info(&di);
  if (st) return st;
  *bytes = ws_layout(batch ? batch : 1u, n_kv_heads, n_heads / n_kv_heads, head_dim,
                     slots_for(di)).total;
  return ok();
}

int nwd_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                    uint16_t* o, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                    uint32_t seq, uint32_t cap, float scale, void* workspace, size_t ws_bytes,
                    void* stream) {
  if (seq > cap) return fail(NWD_ERR_RANGE, "seq %u exceeds maxSeq %u", seq, cap);
  Call c{};
  c.q = q; c.k_pool = k_cache; c.v_pool = v_cache; c.pool_rows = cap;
  c.single_len = (int32_t)seq; c.o = o; c.batch = 1;
  c.n_heads = n_heads; c.n_kv = n_kv_heads; c.hd = head_dim; c.scale = scale;
  c.ws = workspace; c.ws_bytes = ws_bytes; c.stream = stream; c.who = "nwd_attn_decode";
  return launch(c);
}

int nwd_attn_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                            uint16_t* o, uint32_t n_heads, uint32_t n_kv_heads,
                            uint32_t head_dim, uint32_t seq, uint32_t cap, float scale,
                            void* stream) {
  const char* who = "nwd_attn_decode_noalloc";
  if (seq > cap) return fail(NWD_ERR_RANGE, "seq %u exceeds maxSeq %u", seq, cap);
  int st = check_shape(n_heads, n_kv_heads, head_dim, who);
  if (st) return st;
  if (n_kv_heads > NOALLOC_MAX_KV_HEADS)
    return fail(NWD_ERR_UNSUPPORTED, "%s: n_kv_heads %u exceeds the built-in scratch limit of %u",
                who, n_kv_heads, NOALLOC_MAX_KV_HEADS);
  DeviceInfo di;
  st = current_device_info(&di);
  if (st) return st;
  const WsLayout lay = ws_layout(1, n_kv_heads, n_heads / n_kv_heads, head_dim, slots_for(di));
  if ((uint32_t)di.sm_count > NOALLOC_MAX_SMS || lay.total > NOALLOC_BYTES)
    return fail(NWD_ERR_UNSUPPORTED,
                "%s: needs %zu bytes of scratch on this device (%d SMs); the built-in scratch "
                "holds %zu",
                who, lay.total, di.sm_count, NOALLOC_BYTES);
  void* scratch = nullptr;
  st = noalloc_scratch(di.device, stream, &scratch);
  if (st) return st;
  Call c{};
  c.q = q; c.k_pool = k_cache; c.v_pool = v_cache; c.pool_rows = cap;
  c.single_len = (int32_t)seq; c.o = o; c.batch = 1;
  c.n_heads = n_heads; c.n_kv = n_kv_heads; c.hd = head_dim; c.scale = scale;
  c.ws = scratch; c.ws_bytes = NOALLOC_BYTES; c.stream = stream; c.who = who;
  if (!takes_short_path(c, tuning()) && seq > 0) {
    // The scratch keeps the previous call's contents.  The merge tickets must
    // start at zero; a completed call leaves them so, one that gave up on a
    // wait may not, so clear them (a memset, no allocation).  The header's
    // error word is left for nwd_noalloc_check to read.
    cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + lay.tickets_off, 0,
                                    lay.ml_off - lay.tickets_off, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "clearing the decode scratch's merge tickets");
  }
  return launch(c);
}

int nwd_attn_decode_plan(uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                         uint32_t head_dim, uint32_t seq, int* kernel, int* grid, int* split,
                         int* cluster, int* groups) {
  const char* who = "nwd_attn_decode_plan";
  if (!kernel || !grid || !split || !cluster || !groups)
    return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  int st = check_shape(n_heads, n_kv_heads, head_dim, who);
  if (st) return st;
  if (batch == 0 || batch > (uint32_t)MAXB)
    return fail(NWD_ERR_UNSUPPORTED, "%s: batch %u outside [1, %d]", who, batch, MAXB);
  DeviceInfo di;
  st = current_device_info(&di);
  if (st) return st;
  const Tuning& tu = tuning();
  static const int32_t kLens = 0;  // stands for a device seq_len array (batch > 1)
  Call c{};
  c.batch = batch;
  c.n_heads = n_heads;
  c.n_kv = n_kv_heads;
  c.hd = head_dim;
  c.single_len = (int32_t)seq;
  c.seq_len = batch > 1 ? &kLens : nullptr;
  c.who = who;
  if (takes_short_path(c, tu)) {
    const uint32_t C = nwd::decode_short_cluster(seq, tu.short_cta_rows);
    *kernel = 1;
    *grid = (int)(n_kv_heads * C);
    *split = (int)C;
    *cluster = C > 1 ? (int)C : 0;
    *groups = 0;
    return ok();
  }
  Plan pl;
  st = plan_split(c, di, tu, &pl);
  if (st) return st;
  *kernel = 0;
  *grid = (int)pl.grid;
  *split = (int)pl.split_k;
  *cluster = (int)pl.cluster;
  *groups = (int)pl.ng;
  return ok();
}

int nwd_noalloc_check(uint32_t* device_error, void* stream) {
  if (!device_error) return fail(NWD_ERR_INVALID, "nwd_noalloc_check: device_error is NULL");
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st) return st;
  void* scratch = nullptr;
  st = noalloc_scratch(di.device, stream, &scratch);
  if (st) return st;
  // the error word is the scratch header's first word, as in a caller workspace
  return nwd_workspace_check(scratch, sizeof(WsHeader), device_error, stream);
}

int nwd_kv_append_attn_decode(const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                              uint16_t* k_cache, uint16_t* v_cache, uint16_t* o,
                              uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                              uint32_t seq, uint32_t cap, float scale, void* workspace,
                              size_t ws_bytes, void* stream) {
  if (seq >= cap) return fail(NWD_ERR_RANGE, "seq %u exceeds maxSeq %u", seq, cap);
  Call c{};
  c.q = q; c.k_new = k_new; c.v_new = v_new; c.k_pool = k_cache; c.v_pool = v_cache;
  c.pool_rows = cap; c.single_len = (int32_t)seq + 1; c.o = o; c.batch = 1;
  c.n_heads = n_heads; c.n_kv = n_kv_heads; c.hd = head_dim; c.scale = scale; c.append = true;
  c.ws = workspace; c.ws_bytes = ws_bytes; c.stream = stream; c.who = "nwd_kv_append_attn_decode";
  return launch(c);
}

int nwd_attn_decode_batched(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                            uint64_t pool_rows, const int64_t* row_offset,
                            const int32_t* seq_len, uint16_t* o, uint32_t batch,
                            uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                            float scale, void* workspace, size_t ws_bytes, void* stream) {
  if (!row_offset || !seq_len) return fail(NWD_ERR_INVALID, "nwd_attn_decode_batched: null pointer");
  Call c{};
  c.q = q; c.k_pool = k_pool; c.v_pool = v_pool; c.pool_rows = pool_rows;
  c.row_offset = row_offset; c.seq_len = seq_len; c.o = o; c.batch = batch;
  c.n_heads = n_heads; c.n_kv = n_kv_heads; c.hd = head_dim; c.scale = scale;
  c.ws = workspace; c.ws_bytes = ws_bytes; c.stream = stream; c.who = "nwd_attn_decode_batched";
  return launch(c);
}

int nwd_kv_append_attn_decode_batched(const uint16_t* q, const uint16_t* k_new,
                                      const uint16_t* v_new, uint16_t* k_pool, uint16_t* v_pool,
                                      uint64_t pool_rows, const int64_t* row_offset,
                                      const int32_t* pos, uint16_t* o, uint32_t batch,
                                      uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                      float scale, void* workspace, size_t ws_bytes,
                                      void* stream) {
  if (!row_offset || !pos)
    return fail(NWD_ERR_INVALID, "nwd_kv_append_attn_decode_batched: null pointer");
  Call c{};
  c.q = q; c.k_new = k_new; c.v_new = v_new; c.k_pool = k_pool; c.v_pool = v_pool;
  c.pool_rows = pool_rows; c.row_offset = row_offset; c.seq_len = pos; c.o = o; c.batch = batch;
  c.n_heads = n_heads; c.n_kv = n_kv_heads; c.hd = head_dim; c.scale = scale; c.append = true;
  c.ws = workspace; c.ws_bytes = ws_bytes; c.stream = stream;
  c.who = "nwd_kv_append_attn_decode_batched";
  return launch(c);
}

int nwd_attn_decode_partial(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                            uint64_t pool_rows, const int64_t* row_offset,
                            const int32_t* seq_len, float* part_o, float* part_ml,
                            uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                            uint32_t head_dim, float scale, void* workspace, size_t ws_bytes,
                            void* stream) {
  if (!row_offset || !seq_len) return fail(NWD_ERR_INVALID, "nwd_attn_decode_partial: null pointer");
  Call c{};
  c.q = q; c.k_pool = k_pool; c.v_pool = v_pool; c.pool_rows = pool_rows;
  c.row_offset = row_offset; c.seq_len = seq_len; c.part_o = part_o; c.part_ml = part_ml;
  c.batch = batch; c.n_heads = n_heads; c.n_kv = n_kv_heads; c.hd = head_dim; c.scale = scale;
  c.partial = true; c.ws = workspace; c.ws_bytes = ws_bytes; c.stream = stream;
  c.who = "nwd_attn_decode_partial";
  return launch(c);
}

}  // extern "C"
