// The merge half of the long-context step over peer memory: every rank's
// shard partial kernel has pushed each (sequence, kv head) pair's partial
// into every rank's exchange buffer and raised the pair's flag there
// (decode.cu, partial mode with an exchange descriptor); here each rank waits
// for all ranks' flags of a pair and merges their partials in rank order
// (= row order, deterministic) into O.  The only waits are on flags written by
// the ranks' partial kernels (this rank's included), which never wait on
// anything, so no cycle of waits can form; every wait gives up after
// WAIT_LIMIT_NS and records NWD_DEVERR_PIPE_TIMEOUT.
//
// The kernel is a programmatic dependent launch of the partial kernel and
// never calls griddepcontrol.wait: it launches once every partial CTA has
// started (so all of them are resident), its small CTAs sit beside them
// polling the flags, and a pair is merged as soon as its last flag lands, not
// after the partial kernel has drained.  Its ordering comes from the flags:
// this rank's own flags of step e are raised only after this rank's partial
// kernel waited for the previous step's merge, so O is never written out of
// order, and a source rank rewrites a slot (two steps later) only after every
// rank's merge of that slot has finished.
#include <cuda_fp16.h>

#include "nwd_common.h"
#include "ptx.cuh"

namespace {

using namespace nwd;

constexpr int XHD = 128;

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One CTA per (sequence, kv head) pair, G * 32 threads: thread (g, lane) owns
// head g's output columns 4 * lane .. 4 * lane + 3.
__global__ void __launch_bounds__(256) xchg_merge_kernel(const float* __restrict__ data,
                                                         const uint32_t* __restrict__ flags,
                                                         __half* __restrict__ o, uint32_t world,
                                                         uint32_t epoch, uint32_t R, uint32_t P,
                                                         uint32_t n_heads, uint32_t G,
                                                         uint32_t* dev_err) {
  __shared__ int ok;
  const uint32_t pair = blockIdx.x, par = epoch & 1u;
  // the next step's partial kernel may take SMs as this step's partial CTAs
  // leave; it reads nothing before its own griddepcontrol.wait, which returns
  // once this kernel has completed
  nwd::pdl_trigger();
  if (threadIdx.x == 0) {
    int good = 1;
    const uint64_t t0 = ptx::globaltimer();
    for (uint32_t src = 0; src < world && good; src++) {
      const uint32_t* f = flags + (size_t)(par * world + src) * P + pair;
      while (ld_acquire_sys(f) != epoch) {
        __nanosleep(256);  // light polling beside the partial kernel's warps
        if (ptx::globaltimer() - t0 > ptx::WAIT_LIMIT_NS) {
          atomicOr(dev_err, NWD_DEVERR_PIPE_TIMEOUT);
          good = 0;
          break;
        }
      }
    }
    ok = good;
  }
  __syncthreads();  // the flags' acquire (thread 0) orders every thread's loads below
  if (!ok) return;
  const uint32_t g = threadIdx.x >> 5, d = (threadIdx.x & 31u) * 4u;
  if (g >= G) return;
  const uint32_t b = pair / (n_heads / G), hkv = pair % (n_heads / G);
  const uint32_t row = b * n_heads + hkv * G + g;
  float M = -INFINITY;
  for (uint32_t src = 0; src < world; src++) {
    const float* r = data + ((size_t)(par * world + src) * R + row) * XCH_ROW;
    M = fmaxf(M, __ldcg(r + XHD));
  }
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (uint32_t src = 0; src < world; src++) {
    const float* r = data + ((size_t)(par * world + src) * R + row) * XCH_ROW;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(r + XHD));
    if (!(ml.y > 0.f)) continue;  // an empty shard contributes nothing
    const float w = ex2f(ml.x - M);
    const float4 x = __ldcg(reinterpret_cast<const float4*>(r + d));
    L += w * ml.y;
    acc.x += w * x.x;
    acc.y += w * x.y;
    acc.z += w * x.z;
    acc.w += w * x.w;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  __half2 lo = __floats2half2_rn(acc.x * inv, acc.y * inv);
  __half2 hi = __floats2half2_rn(acc.z * inv, acc.w * inv);
  uint2 v;
  v.x = *reinterpret_cast<uint32_t*>(&lo);
  v.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(o + (size_t)row * XHD + d) = v;
}

}  // namespace

namespace nwd {

int launch_xchg_merge(const float* own_data, const uint32_t* own_flags, uint16_t* o,
                      uint32_t world, uint32_t epoch, uint32_t batch, uint32_t n_heads,
                      uint32_t n_kv, uint32_t* dev_err, void* stream) {
  const char* who = "nwd_mgpu_decode_step (merge)";
  if (!own_data || !own_flags || !o || !dev_err) return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  if (n_kv == 0 || n_heads % n_kv || n_heads / n_kv > 8 || world == 0 || epoch == 0)
    return fail(NWD_ERR_INVALID, "%s: bad shape", who);
  const uint32_t G = n_heads / n_kv, P = batch * n_kv, R = batch * n_heads;
  if (P == 0) return ok();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P);
  cfg.blockDim = dim3(G * 32);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, xchg_merge_kernel, own_data, own_flags,
                                     reinterpret_cast<__half*>(o), world, epoch, R, P, n_heads,
                                     G, dev_err);
  if (e != cudaSuccess) return cuda_fail(e, who);
  return ok();
}

}  // namespace nwd
