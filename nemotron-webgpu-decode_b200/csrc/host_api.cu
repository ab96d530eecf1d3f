// Device memory, copies and streams for hosts that have no CUDA runtime of
// their own: the Node.js addon, or a C/C++ engine that links only this
// library.  They stand where the reference's WebGPU helpers stand
// (kernels/gpu.js:75-99 createBuffer / createEmptyStorage / createUniform,
// :141 dispatchAndRead): the engine creates its buffers once, hands them to
// the attention entry points, and reads results back.
#include "nwd_common.h"

using namespace nwd;

extern "C" {

int nwd_set_device(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  return ok();
}

int nwd_device_count(int* count) {
  if (!count) return fail(NWD_ERR_INVALID, "nwd_device_count: count is NULL");
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    return cuda_fail(e, "cudaGetDeviceCount");
  }
  return ok();
}

int nwd_alloc(size_t bytes, void** ptr) {
  if (!ptr) return fail(NWD_ERR_INVALID, "nwd_alloc: ptr is NULL");
  *ptr = nullptr;
  if (bytes == 0) return ok();
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  e = cudaMemset(*ptr, 0, bytes);  // like createEmptyStorage: zero-filled
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_fail(e, "cudaMemset");
  }
  return ok();
}

int nwd_free(void* ptr) {
  if (!ptr) return ok();
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree");
  return ok();
}

int nwd_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return ok();
  if (!dst || !src) return fail(NWD_ERR_INVALID, "nwd_memcpy_h2d: null pointer");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync (host to device)");
  return ok();
}

int nwd_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return ok();
  if (!dst || !src) return fail(NWD_ERR_INVALID, "nwd_memcpy_d2h: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync (device to host)");
  return ok();
}

int nwd_stream_create(void** stream) {
  if (!stream) return fail(NWD_ERR_INVALID, "nwd_stream_create: stream is NULL");
  cudaStream_t s = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreateWithFlags");
  *stream = s;
  return ok();
}

int nwd_stream_destroy(void* stream) {
  if (!stream) return ok();
  cudaError_t e = cudaStreamDestroy((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamDestroy");
  return ok();
}

int nwd_stream_synchronize(void* stream) {
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  return ok();
}

}  // extern "C"
