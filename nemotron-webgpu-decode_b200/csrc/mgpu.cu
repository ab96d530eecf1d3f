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
//
// The exchange itself runs over peer memory when every rank can map every
// other rank's memory (NVLink / NVSwitch): each rank allocates one exchange
// buffer with the driver's virtual-memory API (a POSIX file descriptor per
// allocation, passed to the other ranks over Unix-domain sockets, so a
// rank's mapping of a peer's buffer keeps that memory alive whatever the peer
// does), the shard partial kernel writes each pair's partial straight into
// every rank's buffer and raises the pair's flag there, and a merge kernel on
// each rank waits (bounded) for all ranks' flags and merges (xchg.cu).  That
// replaces the all-gather and its separate merge; NCCL then serves only the
// set-up's votes.  If any rank cannot set it up, all ranks keep the NCCL
// path (NWD_MGPU_P2P=0 forces it).
#include <cudaTypedefs.h>  // PFN_cuMem*
#include <dlfcn.h>
#include <fcntl.h>
#include <nccl.h>  // types and constants only; the functions come from dlopen
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <thread>

#include "nwd_common.h"

// Peer-memory exchange state of one communicator (see the file comment).
struct P2pState {
  int state = 0;  // 0 not set up yet, 1 active, -1 off (the NCCL path)
  uint32_t R = 0, P = 0;
  size_t bytes = 0;       // mapped size of every rank's buffer
  size_t data_bytes = 0;  // the partials; the flags follow
  CUmemGenericAllocationHandle h[nwd::XCH_MAX_RANKS] = {};
  CUdeviceptr va[nwd::XCH_MAX_RANKS] = {};
  bool held[nwd::XCH_MAX_RANKS] = {};    // handle created / imported
  bool mapped[nwd::XCH_MAX_RANKS] = {};  // address reserved and mapped
  uint32_t epoch = 0;
};

struct nwd_mgpu {
  ncclComm_t comm = nullptr;
  int world = 0, rank = 0, device = 0;
  uint32_t step_deadline_ms = 0;
  bool aborted = false;
  bool timing = false;
  bool have_times = false;
  cudaEvent_t ev_done = nullptr;  // completion of the last step (no timing)
  cudaEvent_t ev_t0 = nullptr, ev_t1 = nullptr, ev_t2 = nullptr;  // timing events
  uint8_t id[NWD_MGPU_ID_BYTES] = {};
  P2pState p2p;
  void* last_ws = nullptr;  // the last step's workspace (its error word)
  bool last_p2p = false;
  cudaStream_t aux = nullptr;  // reads of that error word, independent of the caller's streams
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

// ---------------- peer-memory exchange: set-up and teardown ----------------

struct VmmApi {
  PFN_cuMemGetAllocationGranularity_v10020 granularity = nullptr;
  PFN_cuMemCreate_v10020 create = nullptr;
  PFN_cuMemRelease_v10020 release = nullptr;
  PFN_cuMemExportToShareableHandle_v10020 export_fd = nullptr;
  PFN_cuMemImportFromShareableHandle_v10020 import_fd = nullptr;
  PFN_cuMemAddressReserve_v10020 reserve = nullptr;
  PFN_cuMemAddressFree_v10020 free_va = nullptr;
  PFN_cuMemMap_v10020 map = nullptr;
  PFN_cuMemUnmap_v10020 unmap = nullptr;
  PFN_cuMemSetAccess_v10020 access = nullptr;
  bool ok = false;
};
VmmApi g_vmm;
std::once_flag g_vmm_once;

const VmmApi* vmm_api() {
  std::call_once(g_vmm_once, [] {
    auto get = [](const char* name, void** fn) {
      cudaDriverEntryPointQueryResult q;
      return cudaGetDriverEntryPointByVersion(name, fn, 12000, cudaEnableDefault, &q) ==
                 cudaSuccess &&
             q == cudaDriverEntryPointSuccess && *fn;
    };
    VmmApi a;
    a.ok = get("cuMemGetAllocationGranularity", (void**)&a.granularity) &&
           get("cuMemCreate", (void**)&a.create) && get("cuMemRelease", (void**)&a.release) &&
           get("cuMemExportToShareableHandle", (void**)&a.export_fd) &&
           get("cuMemImportFromShareableHandle", (void**)&a.import_fd) &&
           get("cuMemAddressReserve", (void**)&a.reserve) &&
           get("cuMemAddressFree", (void**)&a.free_va) && get("cuMemMap", (void**)&a.map) &&
           get("cuMemUnmap", (void**)&a.unmap) && get("cuMemSetAccess", (void**)&a.access);
    g_vmm = a;
  });
  return g_vmm.ok ? &g_vmm : nullptr;
}

// Unmaps and releases every buffer of the exchange (own and imported).
void p2p_teardown(nwd_mgpu* m) {
  const VmmApi* v = vmm_api();
  P2pState& x = m->p2p;
  for (int r = 0; r < nwd::XCH_MAX_RANKS && v; r++) {
    if (x.mapped[r]) {
      v->unmap(x.va[r], x.bytes);
      v->free_va(x.va[r], x.bytes);
    }
    if (x.held[r]) v->release(x.h[r]);
    x.mapped[r] = x.held[r] = false;
    x.va[r] = 0;
  }
  x.bytes = x.data_bytes = 0;
  x.R = x.P = 0;
}

// Waits for `ev` within the step deadline (the communicator is aborted if it
// runs out, as in nwd_mgpu_sync).
int wait_event(nwd_mgpu* m, const NcclApi* api, cudaEvent_t ev, const char* what) {
  const Clock::time_point t0 = Clock::now();
  for (uint32_t i = 0;; i++) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return NWD_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, what);
    if (ms_since(t0) > m->step_deadline_ms) {
      abort_comm(m, api);
      return fail(NWD_ERR_TIMEOUT, "rank %d: %s did not finish within %u ms; communicator aborted",
                  m->rank, what, m->step_deadline_ms);
    }
    poll_pause(i);
  }
}

// Every rank's `mine` (0 or 1) through one all-gather on the caller's stream
// (dev: >= 4 * world bytes of device scratch); *all = every rank said 1.
int comm_vote(nwd_mgpu* m, const NcclApi* api, int mine, bool* all, void* dev, void* stream) {
  cudaStream_t s = (cudaStream_t)stream;
  int32_t* d = static_cast<int32_t*>(dev);
  cudaError_t e = cudaMemcpyAsync(d + m->rank, &mine, 4, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "exchange set-up vote");
  ncclResult_t r = api->AllGather(d + m->rank, d, 1, ncclInt32, m->comm, s);
  if (r != ncclSuccess && r != ncclInProgress) {
    abort_comm(m, api);
    return fail(NWD_ERR_NCCL, "rank %d: set-up vote: %s", m->rank, api->GetErrorString(r));
  }
  int st = wait_ready(m, api, m->step_deadline_ms, "the set-up vote");
  if (st) return st;
  int32_t votes[nwd::XCH_MAX_RANKS];
  e = cudaMemcpyAsync(votes, d, 4 * m->world, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaEventRecord(m->ev_done, s);
  if (e != cudaSuccess) return cuda_fail(e, "exchange set-up vote");
  st = wait_event(m, api, m->ev_done, "the set-up vote");
  if (st) return st;
  bool a = true;
  for (int i = 0; i < m->world; i++) a = a && votes[i] == 1;
  *all = a;
  return NWD_OK;
}

// Abstract Unix-socket address of rank r's listener for this communicator.
socklen_t p2p_addr(const nwd_mgpu* m, int r, sockaddr_un* a) {
  memset(a, 0, sizeof(*a));
  a->sun_family = AF_UNIX;
  uint64_t h = 1469598103934665603ull;  // FNV-1a over the whole communicator id
  for (int i = 0; i < NWD_MGPU_ID_BYTES; i++) h = (h ^ m->id[i]) * 1099511628211ull;
  char name[96];
  const int n = snprintf(name, sizeof(name), "nwd-xchg-%016llx-%d", (unsigned long long)h, r);
  memcpy(a->sun_path + 1, name, (size_t)n);  // sun_path[0] = 0: the abstract namespace
  return (socklen_t)(offsetof(sockaddr_un, sun_path) + 1 + n);
}

bool send_fd(int sock, int fd, int32_t rank) {
  msghdr msg = {};
  iovec iov = {&rank, sizeof(rank)};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  alignas(cmsghdr) char ctl[CMSG_SPACE(sizeof(int))] = {};
  msg.msg_control = ctl;
  msg.msg_controllen = sizeof(ctl);
  cmsghdr* c = CMSG_FIRSTHDR(&msg);
  c->cmsg_level = SOL_SOCKET;
  c->cmsg_type = SCM_RIGHTS;
  c->cmsg_len = CMSG_LEN(sizeof(int));
  memcpy(CMSG_DATA(c), &fd, sizeof(int));
  return sendmsg(sock, &msg, MSG_NOSIGNAL) == (ssize_t)sizeof(rank);
}

bool recv_fd(int sock, int* fd, int32_t* rank) {
  msghdr msg = {};
  iovec iov = {rank, sizeof(*rank)};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  alignas(cmsghdr) char ctl[CMSG_SPACE(sizeof(int))] = {};
  msg.msg_control = ctl;
  msg.msg_controllen = sizeof(ctl);
  if (recvmsg(sock, &msg, MSG_CMSG_CLOEXEC) != (ssize_t)sizeof(*rank)) return false;
  cmsghdr* c = CMSG_FIRSTHDR(&msg);
  if (!c || c->cmsg_level != SOL_SOCKET || c->cmsg_type != SCM_RIGHTS) return false;
  memcpy(fd, CMSG_DATA(c), sizeof(int));
  return true;
}

// Collective: every rank allocates and zeroes its exchange buffer for (R, P),
// the ranks swap the buffers' file descriptors and map each other's buffers.
// On any failure every rank ends with the exchange off (state -1) and the
// NCCL path; only a failed vote (NCCL) is an error.
int p2p_setup(nwd_mgpu* m, const NcclApi* api, uint32_t R, uint32_t P, void* vote_dev,
              void* stream) {
  P2pState& x = m->p2p;
  p2p_teardown(m);
  x.state = -1;
  const char* env = getenv("NWD_MGPU_P2P");
  const bool wanted = !(env && env[0] == '0') && m->world <= nwd::XCH_MAX_RANKS;
  const VmmApi* v = wanted ? vmm_api() : nullptr;
  int okv = v ? 1 : 0;
  int fd = -1, lsock = -1;
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = m->device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  // 1. this rank's buffer, zeroed (its flags must read 0 before any peer writes)
  if (okv) {
    CUmemAllocationProp prop = {};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = m->device;
    size_t gran = 0;
    x.data_bytes = nwd::xchg_data_floats((uint32_t)m->world, R) * 4;
    const size_t need = nwd::xchg_bytes((uint32_t)m->world, R, P);
    okv = v->granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM) == CUDA_SUCCESS && gran;
    if (okv) {
      x.bytes = (need + gran - 1) / gran * gran;
      okv = v->create(&x.h[m->rank], x.bytes, &prop, 0) == CUDA_SUCCESS;
      x.held[m->rank] = okv;
    }
    if (okv) okv = v->reserve(&x.va[m->rank], x.bytes, gran, 0, 0) == CUDA_SUCCESS;
    if (okv) {
      okv = v->map(x.va[m->rank], x.bytes, 0, x.h[m->rank], 0) == CUDA_SUCCESS;
      if (!okv) v->free_va(x.va[m->rank], x.bytes);
      x.mapped[m->rank] = okv;
    }
    if (okv) okv = v->access(x.va[m->rank], x.bytes, &acc, 1) == CUDA_SUCCESS;
    if (okv)
      okv = cudaMemsetAsync((void*)x.va[m->rank], 0, x.bytes, (cudaStream_t)stream) == cudaSuccess;
    if (okv)
      okv = v->export_fd(&fd, x.h[m->rank], CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) ==
            CUDA_SUCCESS;
  }
  // 2. a listener for the peers' descriptors
  if (okv && m->world > 1) {
    sockaddr_un a;
    const socklen_t len = p2p_addr(m, m->rank, &a);
    lsock = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    okv = lsock >= 0 && bind(lsock, (sockaddr*)&a, len) == 0 && listen(lsock, 64) == 0;
  }
  bool all = false;
  int st = comm_vote(m, api, okv, &all, vote_dev, stream);  // also: every rank listens
  if (st || !all) goto done;
  okv = 1;
  if (m->world > 1) {
    // 3. this rank's descriptor to every peer, then every peer's to this rank
    const Clock::time_point t0 = Clock::now();
    for (int r = 0; r < m->world && okv; r++) {
      if (r == m->rank) continue;
      sockaddr_un a;
      const socklen_t len = p2p_addr(m, r, &a);
      int c = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
      okv = c >= 0 && connect(c, (sockaddr*)&a, len) == 0 && send_fd(c, fd, m->rank);
      if (c >= 0) close(c);
    }
    int got = 0, fds[nwd::XCH_MAX_RANKS];
    for (int r = 0; r < nwd::XCH_MAX_RANKS; r++) fds[r] = -1;
    while (okv && got < m->world - 1) {
      pollfd pf = {lsock, POLLIN, 0};
      const double left = m->step_deadline_ms - ms_since(t0);
      if (left <= 0 || poll(&pf, 1, (int)left + 1) <= 0) {
        okv = 0;
        break;
      }
      int c = accept4(lsock, nullptr, nullptr, SOCK_CLOEXEC);
      int32_t src = -1;
      int pfd = -1;
      okv = c >= 0 && recv_fd(c, &pfd, &src) && src >= 0 && src < m->world && src != m->rank &&
            fds[src] < 0;
      if (c >= 0) close(c);
      if (okv) {
        fds[src] = pfd;
        got++;
      } else if (pfd >= 0) {
        close(pfd);
      }
    }
    // 4. map every peer's buffer for this device
    for (int r = 0; r < m->world; r++) {
      if (r == m->rank || fds[r] < 0) continue;
      if (okv) {
        okv = v->import_fd(&x.h[r], (void*)(uintptr_t)fds[r],
                           CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) == CUDA_SUCCESS;
        x.held[r] = okv;
        if (okv) okv = v->reserve(&x.va[r], x.bytes, 0, 0, 0) == CUDA_SUCCESS;
        if (okv) {
          okv = v->map(x.va[r], x.bytes, 0, x.h[r], 0) == CUDA_SUCCESS;
          if (!okv) v->free_va(x.va[r], x.bytes);
          x.mapped[r] = okv;
        }
        if (okv) okv = v->access(x.va[r], x.bytes, &acc, 1) == CUDA_SUCCESS;
      }
      close(fds[r]);  // the imported handle keeps the allocation
    }
  }
  st = comm_vote(m, api, okv, &all, vote_dev, stream);
  if (!st && all) {
    x.state = 1;
    x.R = R;
    x.P = P;
    x.epoch = 0;
  }
done:
  if (fd >= 0) close(fd);
  if (lsock >= 0) close(lsock);
  if (x.state != 1) {
    p2p_teardown(m);
    x.state = -1;
  }
  return st;
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
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m->aux, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    st = cuda_fail(e, "cudaEventCreate");
    nwd_mgpu_abort(m);
    return st;
  }
  memcpy(m->id, id, NWD_MGPU_ID_BYTES);
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
  // the peer-memory exchange: set up (collectively) on the first step of a
  // shape; every rank takes the same branch, since the set-up's votes agree
  const uint32_t R = batch * n_heads, P = batch * n_kv_heads;
  if (head_dim == 128 && (m->p2p.state == 0 || (m->p2p.state == 1 && (m->p2p.R != R ||
                                                                       m->p2p.P != P)))) {
    st = p2p_setup(m, api, R, P, gather, stream);
    if (st) return st;
  }
  m->last_ws = workspace;
  m->last_p2p = m->p2p.state == 1;
  if (m->last_p2p) {
    P2pState& x = m->p2p;
    nwd::XchgDesc d = {};
    d.world = (uint32_t)m->world;
    d.rank = (uint32_t)m->rank;
    d.epoch = ++x.epoch;
    if (d.epoch == 0) d.epoch = x.epoch = 1;  // after 2^32 steps: 0 never marks a step
    d.R = R;
    d.P = P;
    for (int r = 0; r < m->world; r++) {
      d.data[r] = reinterpret_cast<float*>(x.va[r]);
      d.flags[r] = reinterpret_cast<uint32_t*>(x.va[r] + x.data_bytes);
    }
    if (m->timing && (e = cudaEventRecord(m->ev_t0, s)) != cudaSuccess)
      return cuda_fail(e, "cudaEventRecord");
    // 1. this rank's partials, pushed into every rank's exchange buffer
    st = nwd::decode_partial_xchg(q, k_pool, v_pool, pool_rows, row_offset, seq_len, batch,
                                  n_heads, n_kv_heads, head_dim, scale, workspace,
                                  L.decode_bytes, stream, d);
    if (st) return st;
    if (m->timing && (e = cudaEventRecord(m->ev_t1, s)) != cudaSuccess)
      return cuda_fail(e, "cudaEventRecord");
    // 2. wait for every rank's partials of each pair and merge them in rank order
    st = nwd::launch_xchg_merge(d.data[m->rank], d.flags[m->rank], o, d.world, d.epoch, batch,
                                n_heads, n_kv_heads, static_cast<uint32_t*>(workspace), stream);
    if (st) return st;
    if (m->timing && (e = cudaEventRecord(m->ev_t2, s)) != cudaSuccess)
      return cuda_fail(e, "cudaEventRecord");
    e = cudaEventRecord(m->ev_done, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    m->have_times = m->timing;
    return ok();
  }
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
    if (e == cudaSuccess) {
      if (m->last_p2p && m->last_ws) {
        // a merge that gave up waiting for a peer's partials leaves its mark in
        // the workspace's error word (NWD_DEVERR_PIPE_TIMEOUT)
        uint32_t err = 0;
        e = cudaMemcpyAsync(&err, m->last_ws, sizeof(err), cudaMemcpyDeviceToHost, m->aux);
        if (e == cudaSuccess) e = cudaStreamSynchronize(m->aux);
        if (e == cudaSuccess && err) e = cudaMemsetAsync(m->last_ws, 0, sizeof(err), m->aux);
        if (e == cudaSuccess && err) e = cudaStreamSynchronize(m->aux);
        if (e != cudaSuccess) return cuda_fail(e, "reading the workspace error word");
        if (err & NWD_DEVERR_PIPE_TIMEOUT) {
          abort_comm(m, api);
          return fail(NWD_ERR_TIMEOUT,
                      "rank %d: a peer's partials did not arrive within the device wait limit "
                      "(a peer missing?); communicator aborted",
                      m->rank);
        }
        if (err) return fail(NWD_ERR_DEVICE, "rank %d: device error %u in the sharded step",
                             m->rank, err);
      }
      return ok();
    }
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
  // every rank's buffers mapped here (the peers' allocations stay alive until
  // their last mapping goes); the device must be idle on this handle's work
  if (m->p2p.state == 1 || m->p2p.bytes) {
    if (m->last_p2p) cudaEventSynchronize(m->ev_done);
    p2p_teardown(m);
  }
  if (m->aux) cudaStreamDestroy(m->aux);
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

int nwd_mgpu_exchange_mode(nwd_mgpu* m, int* mode) {
  if (!m || !mode) return fail(NWD_ERR_INVALID, "nwd_mgpu_exchange_mode: null pointer");
  *mode = m->p2p.state;  // 1 peer memory, -1 NCCL all-gather, 0 no step yet
  return ok();
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
