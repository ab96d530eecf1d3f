// Long-context decode with each sequence's KV rows sharded across GPUs: the
// shard partial on every rank, one NCCL all-gather of the packed partials over
// NVLink, and the log-sum-exp merge in rank order, all on the caller's stream.
//
// The reference has no multi-device code (its attention is one WGSL dispatch,
// engine/runtime.js:391); this extends its single-sequence attention to rows
// held by several GPUs.  The exchange is the step's only collective.
//
// NCCL is loaded with dlopen on the first nwd_mgpu_* call (NWD_NCCL_LIBRARY,
// else "libnccl.so.2": the copy a host process has already loaded, or the
// system's), so single-GPU users never load it.  Communicators are
// non-blocking: every wait on NCCL (init, enqueue, step completion, finalize)
// polls ncclCommGetAsyncError under a host-side deadline and, when the
// deadline passes or NCCL reports an error, calls ncclCommAbort (which ends
// the collective's kernels) and returns NWD_ERR_TIMEOUT / NWD_ERR_NCCL.
#include <dlfcn.h>
#include <nccl.h>  // types and constants only; the functions come from dlopen

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>

#include "nwd_common.h"

struct nwd_mgpu {
  ncclComm_t comm = nullptr;
  int world = 0, rank = 0, device = 0;
  uint32_t step_deadline_ms = 0;
  bool aborted = false;
  bool timing = false;
  bool have_times = false;
  cudaEvent_t ev_done = nullptr;  // completion of the last step (no timing)
  cudaEvent_t ev_t0 = nullptr, ev_t1 = nullptr, ev_t2 = nullptr;  // timing events
};

namespace {

using namespace nwd;

struct NcclApi {
  void* lib = nullptr;
  int version = 0;
  ncclResult_t (*GetVersion)(int*) = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  const char* (*GetLastError)(ncclComm_t) = nullptr;
};

NcclApi g_nccl;
std::once_flag g_nccl_once;
char g_nccl_err[256] = {0};

template <typename F>
bool sym(void* lib, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(lib, name));
  return *out != nullptr;
}

int nccl_api(const NcclApi** out) {
  std::call_once(g_nccl_once, [] {
    const char* env = getenv("NWD_NCCL_LIBRARY");
    const char* name = (env && *env) ? env : "libnccl.so.2";
    void* lib = dlopen(name, RTLD_NOW | RTLD_LOCAL);
    if (!lib) {
      snprintf(g_nccl_err, sizeof(g_nccl_err), "dlopen(%s): %s", name, dlerror());
      return;
    }
    NcclApi a;
    a.lib = lib;
    bool ok = sym(lib, "ncclGetVersion", &a.GetVersion) &&
              sym(lib, "ncclGetUniqueId", &a.GetUniqueId) &&
              sym(lib, "ncclCommInitRankConfig", &a.CommInitRankConfig) &&
              sym(lib, "ncclCommGetAsyncError", &a.CommGetAsyncError) &&
              sym(lib, "ncclCommAbort", &a.CommAbort) &&
              sym(lib, "ncclCommFinalize", &a.CommFinalize) &&
              sym(lib, "ncclCommDestroy", &a.CommDestroy) &&
              sym(lib, "ncclAllGather", &a.AllGather) &&
              sym(lib, "ncclGetErrorString", &a.GetErrorString) &&
              sym(lib, "ncclGetLastError", &a.GetLastError);
    if (!ok) {
      snprintf(g_nccl_err, sizeof(g_nccl_err), "%s lacks an NCCL entry point (needs >= 2.14)", name);
      return;
    }
    a.GetVersion(&a.version);
    g_nccl = a;
  });
  if (!g_nccl.lib) return fail(NWD_ERR_NCCL, "NCCL is unavailable: %s", g_nccl_err);
  *out = &g_nccl;
  return NWD_OK;
}

using Clock = std::chrono::steady_clock;

double ms_since(Clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

// Polls at a few microseconds first (a step's completion is usually close),
// then every 50 us.
void poll_pause(uint32_t i) {
  if (i < 64) {
    std::this_thread::sleep_for(std::chrono::microseconds(2));
  } else {
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// Aborts the communicator (ends its kernels in flight) and marks the handle
// unusable for steps.
void abort_comm(nwd_mgpu* m, const NcclApi* api) {
  if (m->comm && !m->aborted) api->CommAbort(m->comm);
  m->aborted = true;
}

// Waits until the communicator has no operation being set up (non-blocking
// init / enqueue / finalize), within `deadline_ms`.
int wait_ready(nwd_mgpu* m, const NcclApi* api, uint32_t deadline_ms, const char* what) {
  const Clock::time_point t0 = Clock::now();
  for (uint32_t i = 0;; i++) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = api->CommGetAsyncError(m->comm, &st);
    if (r != ncclSuccess) st = r;
    if (st == ncclSuccess) return NWD_OK;
    if (st != ncclInProgress) {
      const char* detail = api->GetLastError(m->comm);
      int rc = fail(NWD_ERR_NCCL, "rank %d: %s: %s (%s)", m->rank, what, api->GetErrorString(st),
                    detail ? detail : "");
      abort_comm(m, api);
      return rc;
    }
    if (ms_since(t0) > deadline_ms) {
      abort_comm(m, api);
      return fail(NWD_ERR_TIMEOUT, "rank %d: %s did not finish within %u ms; communicator aborted",
                  m->rank, what, deadline_ms);
    }
    poll_pause(i);
  }
}

struct MgpuLayout {
  size_t decode_bytes;  // the shard partial's workspace
  size_t send_off;      // this rank's packed partials when the all-gather is not in place
  size_t gather_off;    // [world][rows * (hd + 2)] f32
  size_t total;
  size_t count;  // floats per rank
  bool in_place;
};

size_t round256(size_t x) { return (x + 255) / 256 * 256; }

int mgpu_layout(int world, uint32_t batch, uint32_t n_heads, uint32_t n_kv, uint32_t hd,
                MgpuLayout* out) {
  size_t dec = 0;
  int st = nwd_attn_decode_workspace_size(batch, n_heads, n_kv, hd, &dec);
  if (st) return st;
  MgpuLayout L;
  L.count = (size_t)batch * n_heads * (hd + 2);
  // in place when every rank's slot starts on a 16-byte boundary (the partial
  // kernel's part_o alignment)
  L.in_place = (L.count * sizeof(float)) % 16 == 0;
  L.decode_bytes = round256(dec);
  L.send_off = L.decode_bytes;
  L.gather_off = L.send_off + (L.in_place ? 0 : round256(L.count * sizeof(float)));
  L.total = L.gather_off + round256((size_t)world * L.count * sizeof(float));
  *out = L;
  return NWD_OK;
}

int check_handle(nwd_mgpu* m, const char* who) {
  if (!m) return fail(NWD_ERR_INVALID, "%s: handle is NULL", who);
  if (m->aborted)
    return fail(NWD_ERR_NCCL, "%s: rank %d's communicator was aborted after an earlier error", who,
                m->rank);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev != m->device)
    return fail(NWD_ERR_INVALID, "%s: current device %d, communicator device %d", who, dev,
                m->device);
  return NWD_OK;
}

}  // namespace

extern "C" {

int nwd_mgpu_unique_id(uint8_t* id) {
  if (!id) return fail(NWD_ERR_INVALID, "nwd_mgpu_unique_id: id is NULL");
  const NcclApi* api = nullptr;
  int st = nccl_api(&api);
  if (st) return st;
  ncclUniqueId uid;
  ncclResult_t r = api->GetUniqueId(&uid);
  if (r != ncclSuccess)
    return fail(NWD_ERR_NCCL, "ncclGetUniqueId: %s", api->GetErrorString(r));
  static_assert(sizeof(uid) == NWD_MGPU_ID_BYTES, "NCCL unique id size");
  memcpy(id, &uid, sizeof(uid));
  return ok();
}

int nwd_mgpu_init(const uint8_t* id, int world, int rank, int device, uint32_t init_deadline_ms,
                  uint32_t step_deadline_ms, nwd_mgpu** out) {
  const char* who = "nwd_mgpu_init";
  if (!id || !out) return fail(NWD_ERR_INVALID, "%s: null pointer", who);
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return fail(NWD_ERR_INVALID, "%s: rank %d outside world %d", who, rank, world);
  if (init_deadline_ms == 0 || step_deadline_ms == 0)
    return fail(NWD_ERR_INVALID, "%s: deadlines must be > 0 ms", who);
  const NcclApi* api = nullptr;
  int st = nccl_api(&api);
  if (st) return st;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  DeviceInfo di;
  st = current_device_info(&di);
  if (st) return st;
  nwd_mgpu* m = new (std::nothrow) nwd_mgpu();
  if (!m) return fail(NWD_ERR_INVALID, "%s: out of host memory", who);
  m->world = world;
  m->rank = rank;
  m->device = device;
  m->step_deadline_ms = step_deadline_ms;
  e = cudaEventCreateWithFlags(&m->ev_done, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreate(&m->ev_t0);
  if (e == cudaSuccess) e = cudaEventCreate(&m->ev_t1);
  if (e == cudaSuccess) e = cudaEventCreate(&m->ev_t2);
  if (e != cudaSuccess) {
    st = cuda_fail(e, "cudaEventCreate");
    nwd_mgpu_abort(m);
    return st;
  }
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = api->CommInitRankConfig(&m->comm, world, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    st = fail(NWD_ERR_NCCL, "rank %d: ncclCommInitRankConfig: %s", rank, api->GetErrorString(r));
    if (m->comm) abort_comm(m, api);
    m->comm = nullptr;
    nwd_mgpu_abort(m);
    return st;
  }
  st = wait_ready(m, api, init_deadline_ms, "communicator set-up");
  if (st) {
    const std::string keep = nwd_last_error();
    nwd_mgpu_abort(m);
    return fail(st, "%s", keep.c_str());
  }
  *out = m;
  return ok();
}

int nwd_mgpu_workspace_size(int world, uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                            uint32_t head_dim, size_t* bytes) {
  if (!bytes) return fail(NWD_ERR_INVALID, "nwd_mgpu_workspace_size: bytes is NULL");
  if (world < 1) return fail(NWD_ERR_INVALID, "nwd_mgpu_workspace_size: world %d", world);
  MgpuLayout L;
  int st = mgpu_layout(world, batch, n_heads, n_kv_heads, head_dim, &L);
  if (st) return st;
  *bytes = L.total;
  return ok();
}

int nwd_mgpu_set_timing(nwd_mgpu* m, int on) {
  if (!m) return fail(NWD_ERR_INVALID, "nwd_mgpu_set_timing: handle is NULL");
  m->timing = on != 0;
  m->have_times = false;
  return ok();
}

int nwd_mgpu_decode_step(nwd_mgpu* m, const uint16_t* q, const uint16_t* k_pool,
                         const uint16_t* v_pool, uint64_t pool_rows, const int64_t* row_offset,
                         const int32_t* seq_len, uint16_t* o, uint32_t batch, uint32_t n_heads,
                         uint32_t n_kv_heads, uint32_t head_dim, float scale, void* workspace,
                         size_t ws_bytes, void* stream) {
  const char* who = "nwd_mgpu_decode_step";
  int st = check_handle(m, who);
  if (st) return st;
  if (!workspace || ((uintptr_t)workspace & 255u))
    return fail(NWD_ERR_WORKSPACE, "%s: workspace NULL or not 256-byte aligned", who);
  MgpuLayout L;
  st = mgpu_layout(m->world, batch, n_heads, n_kv_heads, head_dim, &L);
  if (st) return st;
  if (ws_bytes < L.total)
    return fail(NWD_ERR_WORKSPACE, "%s: workspace of %zu bytes < %zu required", who, ws_bytes,
                L.total);
  if (!o) return fail(NWD_ERR_INVALID, "%s: o is NULL", who);
  const NcclApi* api = nullptr;
  st = nccl_api(&api);
  if (st) return st;
  // an error NCCL reported since the last step ends this one before any launch
  ncclResult_t async = ncclSuccess;
  api->CommGetAsyncError(m->comm, &async);
  if (async != ncclSuccess && async != ncclInProgress) {
    st = fail(NWD_ERR_NCCL, "rank %d: communicator error before the step: %s", m->rank,
              api->GetErrorString(async));
    abort_comm(m, api);
    return st;
  }
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* gather = reinterpret_cast<float*>(ws + L.gather_off);
  float* mine = L.in_place ? gather + (size_t)m->rank * L.count
                           : reinterpret_cast<float*>(ws + L.send_off);
  const size_t n_o = (size_t)batch * n_heads * head_dim;
  cudaError_t e;
  if (m->timing && (e = cudaEventRecord(m->ev_t0, s)) != cudaSuccess)
    return cuda_fail(e, "cudaEventRecord");
  // 1. this rank's partial (m, l, o) of every (sequence, head) over its rows
  st = nwd_attn_decode_partial(q, k_pool, v_pool, pool_rows, row_offset, seq_len, mine,
                               mine + n_o, batch, n_heads, n_kv_heads, head_dim, scale, workspace,
                               L.decode_bytes, stream);
  if (st) return st;
  if (m->timing && (e = cudaEventRecord(m->ev_t1, s)) != cudaSuccess)
    return cuda_fail(e, "cudaEventRecord");
  // 2. every rank's packed partials, rank order
  ncclResult_t r = api->AllGather(mine, gather, L.count, ncclFloat32, m->comm, s);
  if (r != ncclSuccess && r != ncclInProgress) {
    st = fail(NWD_ERR_NCCL, "rank %d: ncclAllGather: %s", m->rank, api->GetErrorString(r));
    abort_comm(m, api);
    return st;
  }
  if (r == ncclInProgress) {
    st = wait_ready(m, api, m->step_deadline_ms, "enqueueing the all-gather");
    if (st) return st;
  }
  // 3. the merge in rank order (= row order): every rank holds O
  st = nwd_attn_merge_packed(gather, o, (uint32_t)m->world, batch, n_heads, head_dim, stream);
  if (st) return st;
  if (m->timing && (e = cudaEventRecord(m->ev_t2, s)) != cudaSuccess)
    return cuda_fail(e, "cudaEventRecord");
  e = cudaEventRecord(m->ev_done, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  m->have_times = m->timing;
  return ok();
}

int nwd_mgpu_sync(nwd_mgpu* m) {
  const char* who = "nwd_mgpu_sync";
  if (!m) return fail(NWD_ERR_INVALID, "%s: handle is NULL", who);
  const NcclApi* api = nullptr;
  int st = nccl_api(&api);
  if (st) return st;
  if (m->aborted) return fail(NWD_ERR_NCCL, "%s: rank %d's communicator was aborted", who, m->rank);
  cudaEvent_t ev = m->ev_done;
  const Clock::time_point t0 = Clock::now();
  for (uint32_t i = 0;; i++) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return ok();
    if (e != cudaErrorNotReady) return cuda_fail(e, "waiting for the sharded step");
    ncclResult_t async = ncclSuccess;
    api->CommGetAsyncError(m->comm, &async);
    const bool nccl_err = async != ncclSuccess && async != ncclInProgress;
    const bool late = ms_since(t0) > m->step_deadline_ms;
    if (nccl_err || late) {
      abort_comm(m, api);
      // the abort ends the collective's kernels; let the stream drain (bounded)
      // so nothing of the step is still in flight when this returns
      const Clock::time_point t1 = Clock::now();
      bool drained = false;
      for (uint32_t j = 0; ms_since(t1) < 5000.0; j++) {
        if (cudaEventQuery(ev) != cudaErrorNotReady) {
          drained = true;
          break;
        }
        poll_pause(j);
      }
      if (nccl_err)
        return fail(NWD_ERR_NCCL, "rank %d: the all-gather failed: %s; communicator aborted%s",
                    m->rank, api->GetErrorString(async),
                    drained ? "" : " (the stream had not drained 5 s later)");
      return fail(NWD_ERR_TIMEOUT,
                  "rank %d: the sharded step did not complete within %u ms (a peer missing?); "
                  "communicator aborted%s",
                  m->rank, m->step_deadline_ms,
                  drained ? "" : " (the stream had not drained 5 s later)");
    }
    poll_pause(i);
  }
}

int nwd_mgpu_step_times(nwd_mgpu* m, float* partial_ms, float* exchange_ms) {
  if (!m || !partial_ms || !exchange_ms)
    return fail(NWD_ERR_INVALID, "nwd_mgpu_step_times: null pointer");
  if (!m->have_times)
    return fail(NWD_ERR_INVALID, "nwd_mgpu_step_times: no timed step (nwd_mgpu_set_timing)");
  cudaError_t e = cudaEventElapsedTime(partial_ms, m->ev_t0, m->ev_t1);
  if (e == cudaSuccess) e = cudaEventElapsedTime(exchange_ms, m->ev_t1, m->ev_t2);
  if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime (call nwd_mgpu_sync first)");
  return ok();
}

int nwd_mgpu_destroy(nwd_mgpu* m) {
  if (!m) return ok();
  int st = NWD_OK;
  std::string msg;
  const NcclApi* api = nullptr;
  if (m->comm && !m->aborted && nccl_api(&api) == NWD_OK) {
    ncclResult_t r = api->CommFinalize(m->comm);
    if (r == ncclSuccess || r == ncclInProgress) {
      st = wait_ready(m, api, m->step_deadline_ms, "ncclCommFinalize");
      if (st) msg = nwd_last_error();
    } else {
      st = fail(NWD_ERR_NCCL, "ncclCommFinalize: %s", api->GetErrorString(r));
      msg = nwd_last_error();
      abort_comm(m, api);
    }
    if (!m->aborted) api->CommDestroy(m->comm);
  }
  m->comm = nullptr;
  if (m->ev_done) cudaEventDestroy(m->ev_done);
  if (m->ev_t0) cudaEventDestroy(m->ev_t0);
  if (m->ev_t1) cudaEventDestroy(m->ev_t1);
  if (m->ev_t2) cudaEventDestroy(m->ev_t2);
  delete m;
  if (st) return fail(st, "%s", msg.c_str());
  return ok();
}

int nwd_mgpu_abort(nwd_mgpu* m) {
  if (!m) return ok();
  const NcclApi* api = nullptr;
  if (m->comm && nccl_api(&api) == NWD_OK) abort_comm(m, api);
  m->comm = nullptr;
  m->aborted = true;
  return nwd_mgpu_destroy(m);
}

int nwd_mgpu_nccl_version(int* version) {
  if (!version) return fail(NWD_ERR_INVALID, "nwd_mgpu_nccl_version: version is NULL");
  const NcclApi* api = nullptr;
  int st = nccl_api(&api);
  if (st) return st;
  *version = api->version;
  return ok();
}

}  // extern "C"
