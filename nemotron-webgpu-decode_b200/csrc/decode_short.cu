// Decode attention for one short sequence (at most SHORT_ROWS cached rows):
// the engine's own case (kernels/sparse_attn.wgsl:32-113 dispatched once per
// token by engine/runtime.js:389-391, caches of maxSeq = 256 rows), where the
// work is at most a few MB and the general split-KV kernel's machinery (plan,
// TMA pipeline, split partials, merge tickets) is mostly latency.
//
// Up to CTA_ROWS rows a kv head is one CTA, launched without a cluster;
// beyond, a thread-block cluster of C CTAs (C up to 8, about 128 rows each by
// default).  8 warps per CTA.  A CTA copies its share of the head's K and V rows
// into shared memory with cp.async (16-byte pieces, XOR-swizzled per row so
// the matrix loads below hit distinct banks), then each warp takes every
// eighth group of 16 of those keys:
//   S = q K^T on mma.sync m16n8k16 (f16 in, f32 accumulate): A = q, the
//   group's query heads in rows 0-7 (the group is at most 8), B = K rows
//   loaded with ldmatrix; two 8-key tiles per group.
//   Online softmax per head row in log2 units; P = 2^(s - m) as an fp16 head
//   and an fp16 remainder (one fp16 rounding of P would exceed the parity
//   tolerance on outputs near zero).  The MMA's A operand takes the heads in
//   rows 0-7 and the remainders in rows 8-15, so one P V MMA per 8 output
//   columns carries both; B = V rows through ldmatrix.trans.
// The eight warps' (max, sum, output) meet in shared memory, then the C CTAs'
// through distributed shared memory (each CTA reads the others' partials
// after a cluster barrier), in a fixed order.
// With kv_append fused (runtime.js:389-391 as one call) the new row comes
// from k_new / v_new and is also written to the cache.
#include <cuda_fp16.h>

#include "nwd_common.h"

namespace {

constexpr int SHD = 128;        // head_dim
constexpr int SWARPS = 8;
constexpr int STHREADS = SWARPS * 32;
constexpr int SGMAX = 8;        // query heads per kv head (rows 0-7 of the MMA)
constexpr uint32_t CTA_ROWS = 256;    // K and V rows one CTA holds in shared memory
constexpr uint32_t MAX_CLUSTER = 8;   // portable cluster size
constexpr uint32_t SHORT_ROWS = CTA_ROWS * MAX_CLUSTER;

__device__ __forceinline__ uint32_t s_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// byte offset of 16-byte chunk c (0-15) of row r in a [rows][256 B] tile; the
// chunk index is XOR-swizzled by the row within each 128-byte half
__device__ __forceinline__ uint32_t sw_off(uint32_t r, uint32_t c) {
  return r * 256u + ((c & 8u) | ((c ^ r) & 7u)) * 16u;
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2u(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// shared memory of a CTA holding n rows: K, V, the warps' partials, the CTA's
size_t short_smem_bytes(uint32_t n) {
  const size_t rows = (n + 15) / 16 * 16;
  return 2 * rows * 256 + (size_t)(SWARPS + 1) * SGMAX * (SHD + 2) * 4;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// a float in CTA `rank`'s shared memory at the address `local` has in this CTA
__device__ __forceinline__ float ld_cluster(const float* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(s_u32(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// CLUSTER = false: one CTA per kv head (C = 1), launched without a cluster
template <bool CLUSTER>
__global__ void __launch_bounds__(STHREADS, 1)
    decode_short_kernel(const __half* __restrict__ q, const __half* __restrict__ k_new,
                        const __half* __restrict__ v_new, __half* kc, __half* vc,
                        __half* __restrict__ o, uint32_t L, uint32_t n_kv, uint32_t G,
                        float scale_log2, uint32_t append, uint32_t C) {
  extern __shared__ __align__(128) uint8_t sm[];
  // cluster of C CTAs = kv head hkv; this CTA holds rows [r_lo, r_lo + n)
  // (L <= 2048 and C <= 8: the products fit 32 bits)
  const uint32_t hkv = CLUSTER ? blockIdx.x / C : blockIdx.x;
  const uint32_t rank = CLUSTER ? blockIdx.x % C : 0u;
  const uint32_t r_lo = CLUSTER ? L * rank / C : 0u;
  const uint32_t n = CLUSTER ? L * (rank + 1) / C - r_lo : L;
  // the same layout in every CTA of the cluster (the merge reads the others'
  // partials at this CTA's own offsets): room for ceil(L / C) rows
  const uint32_t rows = ((CLUSTER ? (L + C - 1) / C : L) + 15) / 16 * 16;
  uint8_t* ks = sm;
  uint8_t* vs = sm + (size_t)rows * 256;
  float* mrg_o = reinterpret_cast<float*>(vs + (size_t)rows * 256);  // [warp][head][128]
  float* cta_o = mrg_o + SWARPS * SGMAX * SHD;                        // [head][128]
  float* mrg_ml = cta_o + SGMAX * SHD;                                // [warp][head][2]
  float* cta_ml = mrg_ml + SWARPS * SGMAX * 2;                        // [head][2]
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t g = lane >> 2, t = lane & 3;

  // the previous kernel in the stream (e.g. the q/k/v projections) must be
  // done before any row is read; until then, start this CTA's K and V rows
  // on their way into L2 (L2 is the point of coherence, so a row the previous
  // kernel still writes is updated there before it is read after the wait)
  nwd::pdl_trigger();
  for (uint32_t i = tid; i < 4 * n; i += STHREADS) {
    // four 128-byte lines per row: K lo/hi, V lo/hi
    const size_t at = ((size_t)(r_lo + (i >> 2)) * n_kv + hkv) * SHD + (i & 1) * 64;
    const __half* src = (i & 2) ? vc + at : kc + at;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(src) : "memory");
  }
  nwd::pdl_wait();

  // ---- the head's K and V rows into shared memory ----
  const uint32_t kb = s_u32(ks), vb = s_u32(vs);
  for (uint32_t i = tid; i < n * 16; i += STHREADS) {
    const uint32_t r = i >> 4, c = i & 15;  // local row r = cache row r_lo + r
    const bool fresh = append && r_lo + r == L - 1;
    const size_t at = ((size_t)(r_lo + r) * n_kv + hkv) * SHD + c * 8;
    const __half* ksrc = fresh ? k_new + (size_t)hkv * SHD + c * 8 : kc + at;
    const __half* vsrc = fresh ? v_new + (size_t)hkv * SHD + c * 8 : vc + at;
    cp16(kb + sw_off(r, c), ksrc);
    cp16(vb + sw_off(r, c), vsrc);
    if (fresh) {  // kv_append of the new row (kernels/kv_append.wgsl:13-18)
      reinterpret_cast<uint4*>(kc + at)[0] = __ldg(reinterpret_cast<const uint4*>(ksrc));
      reinterpret_cast<uint4*>(vc + at)[0] = __ldg(reinterpret_cast<const uint4*>(vsrc));
    }
  }
  // rows past the CTA's last one in its last group: P is 0 there, but 0 x NaN would not be
  for (uint32_t i = n * 16 + tid; i < rows * 16; i += STHREADS) {
    reinterpret_cast<uint4*>(ks + sw_off(i >> 4, i & 15))[0] = make_uint4(0u, 0u, 0u, 0u);
    reinterpret_cast<uint4*>(vs + sw_off(i >> 4, i & 15))[0] = make_uint4(0u, 0u, 0u, 0u);
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");

  // q as the A operand: head g in row g (rows 8-15 zero), 8 K-steps of 16
  uint32_t qa[8][2];
  const __half* qh = q + ((size_t)hkv * G + g) * SHD;
#pragma unroll
  for (int s = 0; s < 8; s++) {
    qa[s][0] = g < G ? *reinterpret_cast<const uint32_t*>(qh + 16 * s + 2 * t) : 0u;
    qa[s][1] = g < G ? *reinterpret_cast<const uint32_t*>(qh + 16 * s + 8 + 2 * t) : 0u;
  }
  __syncthreads();

  float acc[16][4];  // 16 tiles of 8 output columns: rows g (P head) and g + 8 (remainder)
#pragma unroll
  for (int n = 0; n < 16; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  float m = -INFINITY, l = 0.f;  // head g, log2 units; l over this lane's keys
  // ldmatrix row addresses: lane i feeds row (i & 7) of matrix (i >> 3)
  const uint32_t mi = lane >> 3, mr = lane & 7;
  for (uint32_t grp = warp; grp * 16 < n; grp += SWARPS) {
    const uint32_t key0 = grp * 16;
    // S for keys [key0, key0 + 8) and [key0 + 8, key0 + 16)
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 8; s++) {
      // matrices: (keys 0-7, dims 16s..+7), (keys 0-7, +8..+15), (keys 8-15, ...), (keys 8-15, ...)
      uint32_t b[4];
      ldsm_x4(kb + sw_off(key0 + mr + (mi >> 1) * 8, 2 * s + (mi & 1)), b);
      mma16816(s0, qa[s][0], 0u, qa[s][1], 0u, b[0], b[1]);
      mma16816(s1, qa[s][0], 0u, qa[s][1], 0u, b[2], b[3]);
    }
    // this lane: head g, keys key0 + 2t + {0, 1} (s0) and key0 + 8 + 2t + {0, 1} (s1)
    float v[4] = {s0[0] * scale_log2, s0[1] * scale_log2, s1[0] * scale_log2, s1[1] * scale_log2};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint32_t key = key0 + (j >> 1) * 8 + 2 * t + (j & 1);
      if (key >= n) v[j] = -INFINITY;
    }
    float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (mx > m) {  // key0 < n, so mx is finite
      const float alpha = ex2(m - mx);  // 0 while m is -inf
#pragma unroll
      for (int n = 0; n < 16; n++) {
        acc[n][0] *= alpha;
        acc[n][1] *= alpha;
        acc[n][2] *= alpha;
        acc[n][3] *= alpha;
      }
      l *= alpha;
      m = mx;
    }
    float p[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      p[j] = ex2(v[j] - m);
      l += p[j];
    }
    const __half2 h0 = __floats2half2_rn(p[0], p[1]), h1 = __floats2half2_rn(p[2], p[3]);
    const __half2 r0 = __floats2half2_rn(p[0] - __low2float(h0), p[1] - __high2float(h0));
    const __half2 r1 = __floats2half2_rn(p[2] - __low2float(h1), p[3] - __high2float(h1));
    // A: rows g = P head, rows g + 8 = P remainder; keys 2t.. (tile 0), 8 + 2t.. (tile 1)
    const uint32_t a0 = h2u(h0), a1 = h2u(r0), a2 = h2u(h1), a3 = h2u(r1);
#pragma unroll
    for (int n = 0; n < 16; n += 2) {
      // matrices: (keys 0-7, dims 8n..), (keys 8-15, dims 8n..), (keys 0-7, dims 8n+8..), (keys 8-15, ...)
      uint32_t b[4];
      ldsm_x4_t(vb + sw_off(key0 + mr + (mi & 1) * 8, n + (mi >> 1)), b);
      mma16816(acc[n], a0, a1, a2, a3, b[0], b[1]);
      mma16816(acc[n + 1], a0, a1, a2, a3, b[2], b[3]);
    }
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);

  // ---- the warps meet: (m, l, o) per head, o = head rows + remainder rows ----
  if (g < G) {
#pragma unroll
    for (int n = 0; n < 16; n++) {
      float* row = mrg_o + ((size_t)warp * SGMAX + g) * SHD + n * 8 + 2 * t;
      row[0] = acc[n][0] + acc[n][2];
      row[1] = acc[n][1] + acc[n][3];
    }
    if (t == 0) {
      mrg_ml[(warp * SGMAX + g) * 2] = m;
      mrg_ml[(warp * SGMAX + g) * 2 + 1] = l;
    }
  }
  __syncthreads();
  // the CTA's partial: (m, l) and o relative to m, per head; without a
  // cluster it is the output
  for (uint32_t i = tid; i < G * SHD; i += STHREADS) {
    const uint32_t h = i / SHD, d = i % SHD;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < SWARPS; w++) mm = fmaxf(mm, mrg_ml[(w * SGMAX + h) * 2]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < SWARPS; w++) {
      const float mw = mrg_ml[(w * SGMAX + h) * 2];
      const float e = mw == -INFINITY ? 0.f : ex2(mw - mm);
      num += e * mrg_o[((size_t)w * SGMAX + h) * SHD + d];
      den += e * mrg_ml[(w * SGMAX + h) * 2 + 1];
    }
    if (!CLUSTER) {
      o[((size_t)hkv * G + h) * SHD + d] = __float2half_rn(num / den);
      continue;
    }
    cta_o[h * SHD + d] = num;
    if (d == 0) {
      cta_ml[h * 2] = mm;
      cta_ml[h * 2 + 1] = den;
    }
  }
  if (!CLUSTER) return;
  // ---- the cluster's CTAs meet: each writes a share of the head's outputs ----
  cluster_sync();
  for (uint32_t i = rank * STHREADS + tid; i < G * SHD; i += C * STHREADS) {
    const uint32_t h = i / SHD, d = i % SHD;
    float mm = -INFINITY;
    for (uint32_t c = 0; c < C; c++) mm = fmaxf(mm, ld_cluster(cta_ml + h * 2, c));
    float num = 0.f, den = 0.f;
    for (uint32_t c = 0; c < C; c++) {
      const float mc = ld_cluster(cta_ml + h * 2, c);
      const float e = mc == -INFINITY ? 0.f : ex2(mc - mm);
      num += e * ld_cluster(cta_o + h * SHD + d, c);
      den += e * ld_cluster(cta_ml + h * 2 + 1, c);
    }
    o[((size_t)hkv * G + h) * SHD + d] = __float2half_rn(num / den);
  }
  // no CTA leaves while another may still read its shared memory
  cluster_sync();
}

bool g_short_smem_set[64][2] = {};

}  // namespace

namespace nwd {

uint32_t decode_short_max_rows() { return SHORT_ROWS; }

uint32_t decode_short_cluster(uint32_t L, uint32_t cta_rows) {
  if (cta_rows == 0 || cta_rows > CTA_ROWS) cta_rows = CTA_ROWS;
  uint32_t C = 1;
  if (L > CTA_ROWS) {
    C = (L + cta_rows - 1) / cta_rows;
    if (C > MAX_CLUSTER) C = MAX_CLUSTER;
  }
  return C;
}

int launch_decode_short(const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                        uint16_t* k_cache, uint16_t* v_cache, uint16_t* o, uint32_t L,
                        uint32_t n_kv, uint32_t group, float scale_log2, bool append,
                        uint32_t cta_rows, void* stream, const char* who) {
  if (L == 0 || L > SHORT_ROWS || group > (uint32_t)SGMAX)
    return fail(NWD_ERR_UNSUPPORTED, "%s: short decode path needs 1..%u rows and group <= %d", who,
                SHORT_ROWS, SGMAX);
  // one CTA per kv head while its rows fit one CTA (a cluster launch and its
  // barriers cost more than they save there), else a cluster of C CTAs of
  // about cta_rows rows each (never more than CTA_ROWS)
  const uint32_t C = decode_short_cluster(L, cta_rows);
  if ((L + C - 1) / C > CTA_ROWS) return fail(NWD_ERR_UNSUPPORTED, "%s: %u rows", who, L);
  if ((uint64_t)n_kv * C > 0x7fffffffull) return fail(NWD_ERR_UNSUPPORTED, "%s: too many kv heads", who);
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st) return st;
  const bool cl = C > 1;
  if (di.device < 64 && !g_short_smem_set[di.device][cl]) {
    cudaError_t e = cudaFuncSetAttribute(cl ? decode_short_kernel<true> : decode_short_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)short_smem_bytes(CTA_ROWS));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(decode_short_kernel)");
    g_short_smem_set[di.device][cl] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_kv * C);
  cfg.blockDim = dim3(STHREADS);
  cfg.dynamicSmemBytes = short_smem_bytes((L + C - 1) / C);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = C > 1 ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, cl ? decode_short_kernel<true> : decode_short_kernel<false>,
                                     reinterpret_cast<const __half*>(q),
                                     reinterpret_cast<const __half*>(k_new),
                                     reinterpret_cast<const __half*>(v_new),
                                     reinterpret_cast<__half*>(k_cache),
                                     reinterpret_cast<__half*>(v_cache), reinterpret_cast<__half*>(o),
                                     L, n_kv, group, scale_log2, append ? 1u : 0u, C);
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
}

}  // namespace nwd
