// Internal host/device helpers shared by the library's translation units.
#pragma once

#include <cuda.h>  // CUtensorMap and enums only; the driver is reached via cudaGetDriverEntryPoint
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "nwd.h"

namespace nwd {

// ---- error reporting (thread-local last error) ----
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int cuda_fail(cudaError_t e, const char* what);
int ok();  // clears the last error, returns NWD_OK

// ---- per-device facts ----
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int major = 0, minor = 0;
  size_t smem_optin = 0;
};
int current_device_info(DeviceInfo* out);

// ---- TMA descriptors ----
// Encodes (or returns a cached copy of) the 4-D tensor map the decode kernel
// uses for a token-major cache [rows, n_kv, hd] of fp16:
//   dims {64, hd/64, n_kv, rows}, box {64, box_chunks, 1, box_rows}, 128-byte
//   swizzle (box_chunks = hd/64 loads whole rows; 1 loads one 64-wide column
//   chunk, the layout the tcgen05 operand descriptors expect).
int kv_tensor_map(CUtensorMap* out, const void* base, uint64_t rows, uint32_t n_kv, uint32_t hd,
                  uint32_t box_rows, uint32_t box_chunks = 0);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- decode of one short sequence (decode_short.cu) ----
// A cluster of CTAs per kv head, each holding about cta_rows of its K and V
// rows in shared memory (0 = the most a CTA holds): for 1..max rows and at
// most 8 query heads per kv head, head_dim 128.  With append, row L - 1 comes
// from k_new / v_new and is written to the caches.
uint32_t decode_short_max_rows();
// CTAs per kv head the short kernel uses for L rows (1: no cluster).
uint32_t decode_short_cluster(uint32_t L, uint32_t cta_rows);
int launch_decode_short(const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                        uint16_t* k_cache, uint16_t* v_cache, uint16_t* o, uint32_t L,
                        uint32_t n_kv, uint32_t group, float scale_log2, bool append,
                        uint32_t cta_rows, void* stream, const char* who);

// ---- programmatic dependent launch ----
// A kernel launched with launch_pdl() may start while the kernel before it in
// the stream is still running.  Such a kernel calls pdl_trigger() at entry (so
// the kernel after it may start early in turn) and pdl_wait() in every CTA, on
// every path, before it reads or writes memory that another kernel writes or
// reads: pdl_wait() returns once the previous kernel has completed and its
// writes are visible.  Before it, only constant inputs (weights) are read;
// other memory may only be prefetched into L2 (which brings nothing into the
// SM and, L2 being the point of coherence, never yields a stale value).
// Because every CTA waits, a kernel completes only after the one before it,
// so ordering stays transitive along the stream.
#ifdef __CUDACC__
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}
#endif

// ---- the long-context exchange over peer memory (mgpu.cu, xchg.cu) ----
// Every rank owns one exchange buffer in its own GPU memory, mapped by every
// rank: [2 parities][world source ranks][R rows][XCH_ROW floats] of partials
// (o[128], then m, l; R = batch * n_heads, row = b * n_heads + h), then
// [2 parities][world][P pairs] u32 flags (P = batch * n_kv, pair = b * n_kv +
// hkv).  Step `epoch` (from 1) uses parity epoch & 1: source rank r writes its
// partials of a pair into every rank's slot [parity][r] and then, at system
// scope with release, the pair's flag there to `epoch`; each rank's merge
// waits until all world flags of a pair read `epoch`.
constexpr int XCH_MAX_RANKS = 8;
constexpr uint32_t XCH_ROW = 132;  // floats per (b, h) row: o[128], m, l, pad (16-byte rows)
struct XchgDesc {
  float* data[XCH_MAX_RANKS];      // destination rank r's buffer, as mapped in this process
  uint32_t* flags[XCH_MAX_RANKS];  // destination rank r's flag block
  uint32_t world, rank, epoch, R, P;
};
inline size_t xchg_data_floats(uint32_t world, uint32_t R) { return (size_t)2 * world * R * XCH_ROW; }
inline size_t xchg_bytes(uint32_t world, uint32_t R, uint32_t P) {
  return xchg_data_floats(world, R) * 4 + (size_t)2 * world * P * 4;
}
// The shard partial of every (sequence, kv head) pair pushed to every rank
// (decode.cu), and the waiting merge of the pairs' partials into O (xchg.cu).
int decode_partial_xchg(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                        uint64_t pool_rows, const int64_t* row_offset, const int32_t* seq_len,
                        uint32_t batch, uint32_t n_heads, uint32_t n_kv, uint32_t head_dim,
                        float scale, void* workspace, size_t ws_bytes, void* stream,
                        const XchgDesc& x);
int launch_xchg_merge(const float* own_data, const uint32_t* own_flags, uint16_t* o,
                      uint32_t world, uint32_t epoch, uint32_t batch, uint32_t n_heads,
                      uint32_t n_kv, uint32_t* dev_err, void* stream);

// ---- workspace layout shared by the decode kernels ----
// [0, 256)            header: error word, scheduler counters
// [256, +tickets)     uint32 per (sequence, kv head) merge tickets
// then                float2 (m, l) per (unit, head) and float[hd] per (unit, head)
struct WsHeader {
  uint32_t error;  // NWD_DEVERR_* bits
  uint32_t pad[63];
};
static_assert(sizeof(WsHeader) == 256, "header is 256 bytes");

struct WsLayout {
  size_t tickets_off, ml_off, o_off, total;
  uint32_t max_units;  // partial slots
};
// Layout for `batch` sequences, kv heads n_kv, group g, with `slots` partial
// slots (decode.cu: two per CTA).
WsLayout ws_layout(uint32_t batch, uint32_t n_kv, uint32_t group, uint32_t hd, uint32_t slots);

}  // namespace nwd
