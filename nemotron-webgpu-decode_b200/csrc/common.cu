// Host-side plumbing: error strings, device facts, TMA descriptor encoding,
// workspace layout and the workspace init/check entry points.
#include <cudaTypedefs.h>  // PFN_cuTensorMapEncodeTiled

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "nwd_common.h"

namespace nwd {

namespace {
thread_local char g_last_error[512] = {0};

std::mutex g_dev_mutex;
DeviceInfo g_devs[64];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;

struct TmapEntry {
  const void* base;
  uint64_t rows;
  uint32_t n_kv, hd, box_rows, box_chunks;
  int device;
  CUtensorMap map;
};
constexpr int kTmapCache = 16;
thread_local TmapEntry g_tmaps[kTmapCache];
thread_local int g_tmap_next = 0;
}  // namespace

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(NWD_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

int ok() {
  g_last_error[0] = 0;
  return NWD_OK;
}

int current_device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(NWD_ERR_CUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mutex);
  DeviceInfo& d = g_devs[dev];
  if (d.device != dev) {
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
    d.sm_count = prop.multiProcessorCount;
    d.major = prop.major;
    d.minor = prop.minor;
    d.smem_optin = prop.sharedMemPerBlockOptin;
    d.device = dev;
  }
  if (d.major != 10) {
    return fail(NWD_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)",
                dev, d.major, d.minor);
  }
  *out = d;
  return NWD_OK;
}

int kv_tensor_map(CUtensorMap* out, const void* base, uint64_t rows, uint32_t n_kv, uint32_t hd,
                  uint32_t box_rows, uint32_t box_chunks) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (box_chunks == 0) box_chunks = hd / 64;
  for (int i = 0; i < kTmapCache; i++) {
    TmapEntry& t = g_tmaps[i];
    if (t.base == base && t.rows == rows && t.n_kv == n_kv && t.hd == hd &&
        t.box_rows == box_rows && t.box_chunks == box_chunks && t.device == dev) {
      *out = t.map;
      return NWD_OK;
    }
  }
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    g_encode_err = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                    cudaEnableDefault, &q);
    if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) {
    return fail(NWD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable (%s)",
                cudaGetErrorString(g_encode_err));
  }
  if (hd % 64 != 0) return fail(NWD_ERR_UNSUPPORTED, "head_dim %u is not a multiple of 64", hd);
  if (rows == 0 || rows > (1ull << 31))
    return fail(NWD_ERR_INVALID, "cache rows %llu outside [1, 2^31]", (unsigned long long)rows);
  cuuint64_t dims[4] = {64, hd / 64, n_kv, rows};
  cuuint64_t strides[3] = {128, (cuuint64_t)hd * 2, (cuuint64_t)n_kv * hd * 2};
  cuuint32_t box[4] = {64, box_chunks, 1, box_rows};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap map;
  CUresult r = g_encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(NWD_ERR_INVALID,
                "cuTensorMapEncodeTiled failed (%d) for base %p rows %llu n_kv %u hd %u", (int)r,
                base, (unsigned long long)rows, n_kv, hd);
  }
  TmapEntry& t = g_tmaps[g_tmap_next];
  g_tmap_next = (g_tmap_next + 1) % kTmapCache;
  t.base = base;
  t.rows = rows;
  t.n_kv = n_kv;
  t.hd = hd;
  t.box_rows = box_rows;
  t.box_chunks = box_chunks;
  t.device = dev;
  t.map = map;
  *out = map;
  return NWD_OK;
}

static size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

WsLayout ws_layout(uint32_t batch, uint32_t n_kv, uint32_t group, uint32_t hd, uint32_t slots) {
  WsLayout L;
  L.max_units = slots;
  L.tickets_off = sizeof(WsHeader);
  size_t off = round_up(L.tickets_off + sizeof(uint32_t) * (size_t)batch * n_kv, 256);
  L.ml_off = off;
  off = round_up(off + sizeof(float) * 2 * (size_t)L.max_units * group, 256);
  L.o_off = off;
  off = round_up(off + sizeof(float) * (size_t)L.max_units * group * hd, 256);
  L.total = off;
  return L;
}

}  // namespace nwd

using namespace nwd;

extern "C" {

const char* nwd_last_error(void) { return g_last_error; }

const char* nwd_version(void) { return "nwd 0.1.0 (sm_100a)"; }

const char* nwd_status_name(int status) {
  switch (status) {
    case NWD_OK: return "NWD_OK";
    case NWD_ERR_INVALID: return "NWD_ERR_INVALID";
    case NWD_ERR_RANGE: return "NWD_ERR_RANGE";
    case NWD_ERR_UNSUPPORTED: return "NWD_ERR_UNSUPPORTED";
    case NWD_ERR_WORKSPACE: return "NWD_ERR_WORKSPACE";
    case NWD_ERR_CUDA: return "NWD_ERR_CUDA";
    case NWD_ERR_NCCL: return "NWD_ERR_NCCL";
    case NWD_ERR_TIMEOUT: return "NWD_ERR_TIMEOUT";
    case NWD_ERR_DEVICE: return "NWD_ERR_DEVICE";
    default: return "NWD_ERR_UNKNOWN";
  }
}

int nwd_workspace_init(void* workspace, size_t ws_bytes, void* stream) {
  if (!workspace) return fail(NWD_ERR_WORKSPACE, "workspace is NULL");
  if (ws_bytes < sizeof(WsHeader))
    return fail(NWD_ERR_WORKSPACE, "workspace of %zu bytes is smaller than its header", ws_bytes);
  cudaError_t e = cudaMemsetAsync(workspace, 0, ws_bytes, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  return ok();
}

int nwd_workspace_check(void* workspace, size_t ws_bytes, uint32_t* device_error, void* stream) {
  if (!workspace || ws_bytes < sizeof(WsHeader))
    return fail(NWD_ERR_WORKSPACE, "workspace is NULL or smaller than its header");
  if (!device_error) return fail(NWD_ERR_INVALID, "device_error is NULL");
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "reading the workspace error word");
  if (v) {
    e = cudaMemsetAsync(workspace, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess) return cuda_fail(e, "clearing the workspace error word");
  }
  *device_error = v;
  return ok();
}

}  // extern "C"
