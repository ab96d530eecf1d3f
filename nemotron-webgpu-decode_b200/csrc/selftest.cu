// Failure-detection self-test: one of the library's bounded device waits is
// made to run out, so a host can check end to end that a stalled pipeline
// ends in a status (the workspace's error word) rather than a hung stream.
// The wait is the same warp-uniform mbarrier wait every kernel here uses; the
// barrier expects one arrival that nothing makes.  No fault, no trap: the
// kernel returns once the wait gives up (WAIT_LIMIT_NS, 2 s).
#include "nwd_common.h"
#include "ptx.cuh"

namespace {

using namespace nwd::ptx;

__global__ void wait_timeout_kernel(nwd::WsHeader* wsh) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int32_t abort_flag;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // phase 0 never completes: the wait must give up, raise the abort flag and
  // record NWD_DEVERR_PIPE_TIMEOUT (if it ever succeeded, it reports a range
  // error instead, so the host sees the wrong bit)
  if (warp_wait(b, 0, &abort_flag, &wsh->error) && threadIdx.x == 0)
    atomicOr(&wsh->error, NWD_DEVERR_ROW_RANGE);
}

}  // namespace

using namespace nwd;

extern "C" {

int nwd_selftest_wait_timeout(void* workspace, size_t ws_bytes, void* stream) {
  if (!workspace) return fail(NWD_ERR_WORKSPACE, "nwd_selftest_wait_timeout: workspace is NULL");
  if (ws_bytes < sizeof(WsHeader))
    return fail(NWD_ERR_WORKSPACE, "nwd_selftest_wait_timeout: workspace of %zu bytes", ws_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(NWD_ERR_WORKSPACE, "nwd_selftest_wait_timeout: workspace not 256-byte aligned");
  wait_timeout_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(reinterpret_cast<WsHeader*>(workspace));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "nwd_selftest_wait_timeout");
  return ok();
}

}  // extern "C"
