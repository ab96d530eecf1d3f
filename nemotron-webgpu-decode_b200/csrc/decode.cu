// Split-KV flash-decode for GQA attention over a token-major fp16 KV cache.
//
// Restates kernels/sparse_attn.wgsl:32-113 (O = softmax(scale q.K^T) V per
// query head, kv head = h / group) for B200:
//
//  * Work is cut into units (sequence b, kv head, chunk of C rows).  One
//    persistent CTA per SM pulls units from an atomic queue in the workspace.
//  * Per CTA: one producer warp streams 64-row K and V tiles of the unit's kv
//    head into a 5-stage shared-memory ring with TMA (4-D tensor map over the
//    [rows, n_kv, 128] cache, 128-byte swizzle, no multicast) and mbarrier
//    transaction counts.  Each unit's first stage also carries the G query
//    rows of that kv head (1-D bulk copy).
//  * Four consumer warps each take 16 rows of every stage.  All G <= 8 query
//    heads of the kv head share each loaded K/V tile: S^T = K Q^T and
//    O^T += V^T P^T are m16n8k16 tensor-core MMAs with rows (tokens) on M and
//    query heads on N, fp32 accumulation.  Online softmax in the log2 domain
//    with shuffle max reductions; P is handed from the score accumulators to
//    the PV operand with movmatrix (no shared-memory round trip), as an fp16
//    head + fp16 remainder pair (two MMAs) so P keeps ~22 bits.
//  * End of unit: the four warps merge their (m, l, acc) in shared memory.
//    A unit that covers its whole sequence writes O (or the shard partial);
//    otherwise it writes a partial to the workspace and takes a ticket, and
//    the CTA holding the last ticket of that (b, kv head) merges all chunks in
//    chunk order (deterministic) and writes the result.  No CTA ever waits
//    for another.
//  * Optional append mode fuses kernels/kv_append.wgsl: the unit that owns
//    the new row writes it (generic stores + proxy fence) before its TMA
//    loads read it.
//
// Every mbarrier wait is bounded (time and iteration limits); on expiry the
// kernel records NWD_DEVERR_PIPE_TIMEOUT in the workspace and leaves after
// its own copies in flight have landed.
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>

#include "nwd_common.h"

namespace {

using nwd::WsHeader;

constexpr int HD = 128;                  // head_dim supported by the tiles
constexpr int NCW = 4;                   // consumer warps
constexpr int TOK = 16 * NCW;            // rows per stage
constexpr int NST = 5;                   // pipeline stages
constexpr int GMAX = 8;                  // query heads per kv head (mma N)
constexpr int NTHR = (NCW + 1) * 32;     // + producer warp
constexpr int KV_BYTES = TOK * HD * 2;   // one K (or V) stage: 16 KiB
constexpr int Q_BYTES = GMAX * HD * 2;   // query rows of one kv head
constexpr int MAXB = 4096;               // sequences per launch

constexpr uint32_t F_FIRST = 1u, F_LAST = 2u;

struct StageHdr {
  int32_t unit, b, hkv, t0, ntok, flags, nch, c;
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
  uint32_t max_units;
  int32_t single_len;
  uint32_t batch, n_heads, n_kv, group;
  float scale_log2;
  uint32_t append;   // seq_len holds the row to write; attend row + 1 rows
  uint32_t partial;  // write (m, l, o) partials instead of O
  uint32_t units_target, units_cap, min_chunk, max_chunk;
};

// ---- shared memory layout (offsets from a 1024-aligned base) ----
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + NST * KV_BYTES;
constexpr int OFF_Q = OFF_V + NST * KV_BYTES;
constexpr int OFF_MRG = OFF_Q + NST * Q_BYTES;
constexpr int MRG_FLOATS = NCW * GMAX * (HD + 2);
constexpr int OFF_PFX = OFF_MRG + MRG_FLOATS * 4;
constexpr int OFF_HDR = OFF_PFX + ((MAXB + 1) * 4 + 15) / 16 * 16;
constexpr int OFF_BAR = OFF_HDR + NST * (int)sizeof(StageHdr);
constexpr int OFF_MISC = OFF_BAR + 2 * NST * 8 + 8;  // + consumer-sync barrier
constexpr int SMEM_USED = OFF_MISC + 64;
constexpr int SMEM_BYTES = SMEM_USED + 1024;  // slack for manual 1024-byte alignment

struct Misc {
  int32_t abort;
  int32_t last;
  uint32_t chunk;
  uint32_t total_units;
  uint32_t warp_sum[NTHR / 32];
  uint64_t total_rows;
};
static_assert(sizeof(Misc) <= 64, "misc block");

constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s
constexpr uint32_t WAIT_LIMIT_ITERS = 1u << 26;

// ---------------- PTX wrappers ----------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait.  Returns false if the CTA is aborting (another thread gave
// up) or this wait ran past its limits (then it raises the abort itself).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int32_t* abort,
                                          uint32_t* dev_err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31) == 0) {
      if (*abort) return false;
      if (i >= WAIT_LIMIT_ITERS || globaltimer() - t0 > WAIT_LIMIT_NS) {
        *abort = 1;
        atomicOr(dev_err, NWD_DEVERR_PIPE_TIMEOUT);
        return false;
      }
    }
  }
}
// Warp-uniform bounded wait: every lane waits (so every lane acquires the
// barrier's completion), then the warp agrees; if any lane gave up, all do.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int32_t* abort,
                                          uint32_t* dev_err) {
  const bool ok = mbar_wait(bar, parity, abort, dev_err);
  return __all_sync(0xffffffffu, ok);
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
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

// Byte offset of 16-byte chunk `chunk16` of 128-byte row R inside a stage
// written by TMA with 128-byte swizzle (stage base 1024-aligned).
__device__ __forceinline__ uint32_t swz(uint32_t R, uint32_t chunk16) {
  return R * 128u + ((chunk16 ^ (R & 7u)) << 4);
}

// ---------------- work plan ----------------
__device__ __forceinline__ uint32_t seq_rows(const Params& p, uint32_t b) {
  if (!p.seq_len) return p.single_len > 0 ? (uint32_t)p.single_len : 0u;
  const int32_t v = p.seq_len[b];
  if (p.append) return v >= 0 ? (uint32_t)v + 1u : 0u;
  return v > 0 ? (uint32_t)v : 0u;
}
__device__ __forceinline__ int64_t seq_off(const Params& p, uint32_t b) {
  return p.row_offset ? p.row_offset[b] : 0;
}
__device__ __forceinline__ uint32_t cdiv(uint64_t a, uint64_t b) { return (uint32_t)((a + b - 1) / b); }

// Chunk length C (multiple of TOK): about units_target units overall, at
// least min_chunk rows, at most max_chunk rows unless that would exceed
// units_cap units.  Identical in every CTA.
__device__ uint32_t choose_chunk(const Params& p, uint64_t total_rows) {
  const uint64_t work = total_rows * p.n_kv;
  uint64_t c = (work + p.units_target - 1) / p.units_target;
  c = (c + TOK - 1) / TOK * TOK;
  if (c < p.min_chunk) c = p.min_chunk;
  if (c > p.max_chunk) c = p.max_chunk;
  uint64_t cu = (work + p.units_cap - 1) / p.units_cap;
  cu = (cu + TOK - 1) / TOK * TOK;
  if (c < cu) c = cu;
  if (c > 0x40000000ull) c = 0x40000000ull;
  return (uint32_t)c;
}

// Block-wide exclusive scan of per-thread values; returns this thread's
// offset, writes the grand total to *total (all threads see it after return).
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

__device__ __forceinline__ uint32_t find_seq(const uint32_t* pfx, uint32_t batch, uint32_t u) {
  // largest b with pfx[b] <= u
  uint32_t lo = 0, hi = batch;  // pfx[batch] = total > u
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (pfx[mid] <= u) lo = mid; else hi = mid;
  }
  return lo;
}

// ---------------- kernel ----------------
__global__ void __launch_bounds__(NTHR, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                  const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  uint32_t* pfx = reinterpret_cast<uint32_t*>(smem + OFF_PFX);
  StageHdr* hdr = reinterpret_cast<StageHdr*>(smem + OFF_HDR);
  Misc* misc = reinterpret_cast<Misc*>(smem + OFF_MISC);
  volatile int32_t* abort_flag = &misc->abort;
  const uint32_t bar_full = sbase + OFF_BAR;            // + 8*s
  const uint32_t bar_empty = sbase + OFF_BAR + 8 * NST; // + 8*s
  const uint32_t bar_csync = sbase + OFF_BAR + 16 * NST;
  WsHeader* wsh = reinterpret_cast<WsHeader*>(p.ws);
  uint32_t* tickets = reinterpret_cast<uint32_t*>(p.ws + p.tickets_off);
  float* ws_ml = reinterpret_cast<float*>(p.ws + p.ml_off);
  float* ws_o = reinterpret_cast<float*>(p.ws + p.o_off);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t B = p.seq_len ? p.batch : 1u;
  const uint32_t G = p.group;

  // ---- plan: total rows -> chunk -> per-sequence unit prefix ----
  if (tid == 0) {
    misc->abort = 0;
    misc->last = 0;
    misc->total_rows = 0;
#pragma unroll
    for (int s = 0; s < NST; s++) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, NCW);
    }
    mbar_init(bar_csync, NCW * 32);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint32_t seg = (B + NTHR - 1) / NTHR;
  const uint32_t beg = min(B, tid * seg), end = min(B, beg + seg);
  uint64_t rows_local = 0;
  for (uint32_t b = beg; b < end; b++) rows_local += seq_rows(p, b);
  if (rows_local)
    atomicAdd(reinterpret_cast<unsigned long long*>(&misc->total_rows),
              (unsigned long long)rows_local);
  __syncthreads();
  const uint64_t total_rows = misc->total_rows;
  const uint32_t C = choose_chunk(p, total_rows);
  uint32_t units_local = 0;
  for (uint32_t b = beg; b < end; b++) {
    const uint32_t L = seq_rows(p, b);
    units_local += p.n_kv * max(1u, cdiv(L, C));
  }
  uint32_t total_units;
  uint32_t run = block_scan(units_local, misc, &total_units);
  for (uint32_t b = beg; b < end; b++) {
    pfx[b] = run;
    run += p.n_kv * max(1u, cdiv(seq_rows(p, b), C));
  }
  if (tid == 0) pfx[B] = total_units;
  if (total_units > p.max_units) {
    if (tid == 0 && blockIdx.x == 0) atomicOr(&wsh->error, NWD_DEVERR_ROW_RANGE);
    return;  // uniform across the block; nothing launched yet
  }
  __syncthreads();

  if (warp == NCW) {
    // ======================= producer warp =======================
    const uint64_t policy = evict_first_policy();
    int stage = 0;
    uint32_t phase = 0;
    uint32_t n_issued = 0;  // stages armed so far (stage s armed ceil((n-s)/NST) times)
    bool aborted = false;
    while (!aborted) {
      uint32_t u = 0;
      if (lane == 0) u = atomicAdd(&wsh->next_unit, 1u);
      u = __shfl_sync(0xffffffffu, u, 0);
      if (u >= total_units) break;
      const uint32_t b = find_seq(pfx, B, u);
      const uint32_t L = seq_rows(p, b);
      const uint32_t nch = (pfx[b + 1] - pfx[b]) / p.n_kv;
      const uint32_t r = u - pfx[b];
      const uint32_t hkv = r / nch, c = r % nch;
      const int64_t off = seq_off(p, b);
      const uint32_t t_begin = c * C;
      const uint32_t t_end = min(L, t_begin + C);
      if (lane == 0 && c == 0 && (off < 0 || (uint64_t)off + L > p.pool_rows))
        atomicOr(&wsh->error, NWD_DEVERR_ROW_RANGE);
      if (p.append && c == nch - 1 && L > 0) {
        // fused kv_append: this unit owns row L-1 of kv head hkv
        const int64_t row = off + (int64_t)L - 1;
        if (row >= 0 && (uint64_t)row < p.pool_rows) {
          const size_t dst = ((size_t)row * p.n_kv + hkv) * HD;
          const size_t src = ((size_t)b * p.n_kv + hkv) * HD;
          const int half = lane >> 4, j = lane & 15;  // lanes 0-15: K, 16-31: V
          const uint4* s = reinterpret_cast<const uint4*>((half ? p.v_new : p.k_new) + src) + j;
          uint4* d = reinterpret_cast<uint4*>((half ? p.v_pool : p.k_pool) + dst) + j;
          *d = __ldg(s);
          asm volatile("fence.proxy.async;" ::: "memory");
        } else if (lane == 0) {
          atomicOr(&wsh->error, NWD_DEVERR_ROW_RANGE);
        }
        __syncwarp();
      }
      const uint32_t nstages = t_end > t_begin ? cdiv(t_end - t_begin, TOK) : 1u;
      for (uint32_t s = 0; s < nstages; s++) {
        if (!warp_wait(bar_empty + 8 * stage, phase ^ 1u, abort_flag, &wsh->error)) {
          aborted = true;
          break;
        }
        if (lane == 0) {
          StageHdr h;
          h.unit = (int32_t)u;
          h.b = (int32_t)b;
          h.hkv = (int32_t)hkv;
          h.t0 = (int32_t)(t_begin + s * TOK);
          h.ntok = (int32_t)(t_end > t_begin ? min((uint32_t)TOK, t_end - (t_begin + s * TOK)) : 0u);
          h.flags = (s == 0 ? F_FIRST : 0u) | (s + 1 == nstages ? F_LAST : 0u);
          h.nch = (int32_t)nch;
          h.c = (int32_t)c;
          hdr[stage] = h;
          const uint32_t fb = bar_full + 8 * stage;
          if (h.ntok > 0) {
            const uint32_t qbytes = (s == 0) ? G * HD * 2 : 0u;
            mbar_arrive_tx(fb, 2 * KV_BYTES + qbytes);
            const int row = (int)(off + (int64_t)h.t0);
            tma_load_4d(sbase + OFF_K + stage * KV_BYTES, &tmk, fb, 0, 0, (int)hkv, row, policy);
            tma_load_4d(sbase + OFF_V + stage * KV_BYTES, &tmv, fb, 0, 0, (int)hkv, row, policy);
            if (qbytes)
              bulk_load(sbase + OFF_Q + stage * Q_BYTES,
                        p.q + ((size_t)b * p.n_heads + (size_t)hkv * G) * HD, qbytes, fb);
          } else {
            mbar_arrive(fb);
          }
        }
        __syncwarp();
        n_issued++;
        if (++stage == NST) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!aborted) {
      // terminator stage
      if (warp_wait(bar_empty + 8 * stage, phase ^ 1u, abort_flag, &wsh->error)) {
        if (lane == 0) {
          hdr[stage].unit = -1;
          mbar_arrive(bar_full + 8 * stage);
        }
        __syncwarp();
      } else {
        aborted = true;
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
    if (lane == 0) {
      __threadfence();
      if (atomicAdd(&wsh->done_ctas, 1u) == gridDim.x - 1) {
        // every CTA has drawn its last unit: reset the queue for the next call
        wsh->next_unit = 0;
        wsh->done_ctas = 0;
        __threadfence();
      }
    }
    return;
  }

  // ======================= consumer warps =======================
  const uint32_t g0 = 2u * (lane & 3);      // this lane's two heads (C/B fragment cols)
  const uint32_t rowq = lane >> 2;          // fragment row
  // ldmatrix lane roles
  const uint32_t li = lane >> 3, lr = lane & 7;
  const uint32_t tokK = warp * 16 + (li & 1) * 8 + lr;  // K: matrices (rows 0-7/8-15) x (k lo/hi)
  const uint32_t tokV = warp * 16 + (li >> 1) * 8 + lr; // V^T: (d lo/hi) x (tokens lo/hi)

  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float acc[8][4];
  uint32_t qf[8][2];
  int stage = 0;
  uint32_t phase = 0, cph = 0;
  float* mrg = reinterpret_cast<float*>(smem + OFF_MRG);
  float* mrg_m = mrg;                       // [NCW][GMAX]
  float* mrg_l = mrg + NCW * GMAX;          // [NCW][GMAX]
  float* mrg_acc = mrg + 2 * NCW * GMAX;    // [NCW][GMAX][HD]

  while (true) {
    if (!warp_wait(bar_full + 8 * stage, phase, abort_flag, &wsh->error)) break;
    const StageHdr h = hdr[stage];
    if (h.unit < 0) break;
    if (h.flags & F_FIRST) {
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; mt++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[mt][j] = 0.f;
      if (h.ntok > 0) {
        const uint8_t* qs = smem + OFF_Q + stage * Q_BYTES + rowq * (HD * 2) + g0 * 2;
        const bool live = rowq < G;
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
          qf[ks][0] = live ? *reinterpret_cast<const uint32_t*>(qs + ks * 32) : 0u;
          qf[ks][1] = live ? *reinterpret_cast<const uint32_t*>(qs + ks * 32 + 16) : 0u;
        }
      }
    }
    const int valid = min(16, h.ntok - warp * 16);
    if (valid > 0) {
      const uint32_t kb = sbase + OFF_K + stage * KV_BYTES;
      const uint32_t vb = sbase + OFF_V + stage * KV_BYTES;
      // ---- S^T[16 tokens][8 heads] = K Q^T ----
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 8; ks++) {
        const uint32_t R = 2u * tokK + (uint32_t)(ks >> 2);
        const uint32_t ch = (uint32_t)(ks & 3) * 2u + (li >> 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kb + swz(R, ch), a0, a1, a2, a3);
        mma16816((ks & 1) ? s1 : s0, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
      }
      float sc[4];
#pragma unroll
      for (int j = 0; j < 4; j++) sc[j] = (s0[j] + s1[j]) * p.scale_log2;
      if ((int)rowq >= valid) sc[0] = sc[1] = -INFINITY;
      if ((int)rowq + 8 >= valid) sc[2] = sc[3] = -INFINITY;
      // ---- online softmax (log2 domain), per head column ----
      float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float base0 = mn0 == -INFINITY ? 0.f : mn0;
      const float base1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = ex2(m0 - base0), al1 = ex2(m1 - base1);
      const float p0 = ex2(sc[0] - base0), p1 = ex2(sc[1] - base1);
      const float p2 = ex2(sc[2] - base0), p3 = ex2(sc[3] - base1);
      l0 = l0 * al0 + (p0 + p2);
      l1 = l1 * al1 + (p1 + p3);
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < 8; mt++) {
        acc[mt][0] *= al0;
        acc[mt][1] *= al1;
        acc[mt][2] *= al0;
        acc[mt][3] *= al1;
      }
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
      // rows past `valid` may hold stale or foreign data: zero them in V^T
      uint32_t mlo = 0xffffffffu, mhi = 0xffffffffu;
      if (valid < 16) {
        const int te = (int)g0;  // tokens te, te+1 (regs 0,1) and te+8, te+9 (regs 2,3)
        mlo = (te < valid ? 0x0000ffffu : 0u) | (te + 1 < valid ? 0xffff0000u : 0u);
        mhi = (te + 8 < valid ? 0x0000ffffu : 0u) | (te + 9 < valid ? 0xffff0000u : 0u);
      }
      // ---- O^T[128 dims][8 heads] += V^T P^T ----
#pragma unroll
      for (int mt = 0; mt < 8; mt++) {
        const uint32_t R = 2u * tokV + (uint32_t)(mt >> 2);
        const uint32_t ch = (uint32_t)(mt & 3) * 2u + (li & 1);
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vb + swz(R, ch), a0, a1, a2, a3);
        a0 &= mlo;
        a1 &= mlo;
        a2 &= mhi;
        a3 &= mhi;
        mma16816(acc[mt], a0, a1, a2, a3, pb0, pb1);
        mma16816(acc[mt], a0, a1, a2, a3, pl0, pl1);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * stage);
    if (++stage == NST) {
      stage = 0;
      phase ^= 1u;
    }
    if (!(h.flags & F_LAST)) continue;

    // ======== end of unit: merge the four warps, then emit ========
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
    const uint32_t ct = warp * 32 + lane;
    const uint32_t g = ct >> 4, d0 = (ct & 15) * 8;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NCW; w++) M = fmaxf(M, mrg_m[w * GMAX + g]);
    float Ls = 0.f, o8[8];
#pragma unroll
    for (int j = 0; j < 8; j++) o8[j] = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; w++) {
      const float mw = mrg_m[w * GMAX + g];
      const float f = mw == -INFINITY ? 0.f : ex2(mw - M);
      Ls += f * mrg_l[w * GMAX + g];
      const float* a = mrg_acc + ((size_t)w * GMAX + g) * HD + d0;
#pragma unroll
      for (int j = 0; j < 8; j++) o8[j] += f * a[j];
    }
    if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;  // scratch free again

    const uint32_t b = (uint32_t)h.b, hkv = (uint32_t)h.hkv, nch = (uint32_t)h.nch;
    bool emit = (nch == 1);
    if (!emit) {
      const uint32_t u = (uint32_t)h.unit;
      if (g < G) {
        const size_t slot = (size_t)u * G + g;
        *reinterpret_cast<float2*>(ws_ml + slot * 2) = make_float2(M, Ls);
        float4* dst = reinterpret_cast<float4*>(ws_o + slot * HD + d0);
        dst[0] = make_float4(o8[0], o8[1], o8[2], o8[3]);
        dst[1] = make_float4(o8[4], o8[5], o8[6], o8[7]);
      }
      __threadfence();
      if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;
      if (ct == 0) {
        const uint32_t t = atomicAdd(&tickets[b * p.n_kv + hkv], 1u);
        misc->last = (t == nch - 1) ? 1 : 0;
      }
      if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;
      emit = misc->last != 0;
      if (emit) {
        __threadfence();
        const uint32_t u0 = u - (uint32_t)h.c;
        if (g < G) {
          // one online pass over the chunks in chunk order, 8 chunks' loads in
          // flight per thread (the merge is L2-latency bound, not bandwidth bound)
          M = -INFINITY;
          Ls = 0.f;
#pragma unroll
          for (int j = 0; j < 8; j++) o8[j] = 0.f;
          for (uint32_t cc = 0; cc < nch; cc += 8) {
            float2 ml[8];
            float4 x0[8], x1[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
              if (cc + j < nch) {
                const size_t slot = (size_t)(u0 + cc + j) * G + g;
                ml[j] = __ldcg(reinterpret_cast<const float2*>(ws_ml + slot * 2));
                const float4* src = reinterpret_cast<const float4*>(ws_o + slot * HD + d0);
                x0[j] = __ldcg(src);
                x1[j] = __ldcg(src + 1);
              } else {
                ml[j] = make_float2(-INFINITY, 0.f);
                x0[j] = x1[j] = make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
              if (ml[j].x == -INFINITY) continue;  // empty chunk
              const float Mn = fmaxf(M, ml[j].x);
              const float a = ex2(M - Mn);  // 0 while M is -inf
              const float f = ex2(ml[j].x - Mn);
              Ls = Ls * a + f * ml[j].y;
              o8[0] = o8[0] * a + f * x0[j].x; o8[1] = o8[1] * a + f * x0[j].y;
              o8[2] = o8[2] * a + f * x0[j].z; o8[3] = o8[3] * a + f * x0[j].w;
              o8[4] = o8[4] * a + f * x1[j].x; o8[5] = o8[5] * a + f * x1[j].y;
              o8[6] = o8[6] * a + f * x1[j].z; o8[7] = o8[7] * a + f * x1[j].w;
              M = Mn;
            }
          }
        }
        if (ct == 0) tickets[b * p.n_kv + hkv] = 0u;
      }
      // misc->last is reused by the next unit
      if (!consumer_sync(bar_csync, cph, abort_flag, &wsh->error)) break;
    }
    if (emit && g < G) {
      const size_t row = (size_t)b * p.n_heads + (size_t)hkv * G + g;
      if (p.partial) {
        *reinterpret_cast<float2*>(p.part_ml + row * 2) = make_float2(M, Ls);
        float4* dst = reinterpret_cast<float4*>(p.part_o + row * HD + d0);
        dst[0] = make_float4(o8[0], o8[1], o8[2], o8[3]);
        dst[1] = make_float4(o8[4], o8[5], o8[6], o8[7]);
      } else {
        const float inv = Ls > 0.f ? 1.f / Ls : 0.f;
        uint4 v;
        v.x = pack_half2(o8[0] * inv, o8[1] * inv);
        v.y = pack_half2(o8[2] * inv, o8[3] * inv);
        v.z = pack_half2(o8[4] * inv, o8[5] * inv);
        v.w = pack_half2(o8[6] * inv, o8[7] * inv);
        *reinterpret_cast<uint4*>(p.o + row * HD + d0) = v;
      }
    }
  }
}

// ---------------- host side ----------------
// Chunk policy: about `waves` units per CTA (one persistent CTA per SM), a
// chunk at least min_chunk rows and at most max_chunk rows (longer chunks mean
// fewer partials to merge; the queue balances ragged batches), and never more
// than cap_per_sm units per SM.  Defaults from a sweep on B200 (config-3
// ragged batch and config-2 single sequences).
struct Tuning {
  uint32_t waves = 1;
  uint32_t cap_per_sm = 64;
  uint32_t min_chunk = 256;
  uint32_t max_chunk = 4096;
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
    x.waves = env_u32("NWD_DECODE_WAVES", x.waves);
    x.cap_per_sm = env_u32("NWD_DECODE_UNITS_CAP_PER_SM", x.cap_per_sm);
    x.min_chunk = (env_u32("NWD_DECODE_MIN_CHUNK", x.min_chunk) + TOK - 1) / TOK * TOK;
    x.max_chunk = (env_u32("NWD_DECODE_MAX_CHUNK", x.max_chunk) + TOK - 1) / TOK * TOK;
    if (x.max_chunk < x.min_chunk) x.max_chunk = x.min_chunk;
    return x;
  }();
  return t;
}

bool g_smem_set[64] = {false};

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

int launch(const Call& c) {
  using namespace nwd;
  int st = check_shape(c.n_heads, c.n_kv, c.hd, c.who);
  if (st) return st;
  if (!c.q || !c.k_pool || !c.v_pool || (!c.partial && !c.o) ||
      (c.partial && (!c.part_o || !c.part_ml)) || (c.append && (!c.k_new || !c.v_new)))
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
  const uint32_t grid_max = (uint32_t)di.sm_count;
  const uint32_t units_cap = grid_max * tu.cap_per_sm;
  const uint32_t G = c.n_heads / c.n_kv;
  const WsLayout lay = ws_layout(c.batch, c.n_kv, G, c.hd, units_cap);
  if (!c.ws) return fail(NWD_ERR_WORKSPACE, "%s: workspace is NULL", c.who);
  if (c.ws_bytes < lay.total)
    return fail(NWD_ERR_WORKSPACE, "%s: workspace of %zu bytes < %zu required", c.who, c.ws_bytes,
                lay.total);
  if ((uintptr_t)c.ws & 255u)
    return fail(NWD_ERR_WORKSPACE, "%s: workspace must be 256-byte aligned", c.who);
  if (c.batch == 0) return ok();

  if (!g_smem_set[di.device]) {
    cudaError_t e =
        cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_kernel)");
    g_smem_set[di.device] = true;
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
  p.max_units = lay.max_units;
  p.batch = c.batch;
  p.n_heads = c.n_heads;
  p.n_kv = c.n_kv;
  p.group = G;
  const float scale = c.scale != 0.f ? c.scale : 1.0f / sqrtf((float)c.hd);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.append = c.append ? 1u : 0u;
  p.partial = c.partial ? 1u : 0u;
  p.units_target = grid_max * tu.waves;
  p.units_cap = units_cap;
  p.min_chunk = tu.min_chunk;
  p.max_chunk = tu.max_chunk;

  // grid: one CTA per SM, fewer when the plan cannot have that many units
  uint32_t grid = grid_max;
  if (!c.seq_len) {
    const uint32_t L = c.single_len > 0 ? (uint32_t)c.single_len : 0u;
    // upper bound on units: with C >= min_chunk
    const uint64_t ub = (uint64_t)c.n_kv * (L / tu.min_chunk + 1);
    if (ub < grid) grid = (uint32_t)ub;
  } else {
    const uint64_t ub = lay.max_units;
    if (ub < grid) grid = (uint32_t)ub;
  }
  if (grid == 0) grid = 1;
  decode_kernel<<<grid, NTHR, SMEM_BYTES, (cudaStream_t)c.stream>>>(tmk, tmv, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, c.who);
  return ok();
}

}  // namespace

using namespace nwd;

extern "C" {

int nwd_attn_decode_workspace_size(uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                                   uint32_t head_dim, size_t* bytes) {
  if (!bytes) return fail(NWD_ERR_INVALID, "nwd_attn_decode_workspace_size: bytes is NULL");
  int st = check_shape(n_heads, n_kv_heads, head_dim, "nwd_attn_decode_workspace_size");
  if (st) return st;
  DeviceInfo di;
  st = current_device_info(&di);
  if (st) return st;
  const uint32_t units_cap = (uint32_t)di.sm_count * tuning().cap_per_sm;
  *bytes = ws_layout(batch ? batch : 1u, n_kv_heads, n_heads / n_kv_heads, head_dim, units_cap).total;
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
