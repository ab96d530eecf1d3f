// N-API addon over the nwd C ABI: the binding engine/runtime.js would load in
// place of the WGSL pipelines of its attention layers (engine/runtime.js:101-102,
// :331-333, :389-391).  Built only where Node's headers exist (node-gyp /
// cmake-js with node_api.h); this repository's build does not compile it.
//
// JS surface (mirrors the WGSL Params of the two replaced kernels):
//   nwd.kvAppend(src, cache, {seq, n_kv, hd, cap})
//       kernels/kv_append.wgsl Params {seq, n_kv, hd} (+ cap, the row capacity)
//   nwd.attention(q, kCache, vCache, o, {n_heads, n_kv_heads, head_dim, seq, cap})
//       kernels/sparse_attn.wgsl Params {n_heads, n_kv_heads, head_dim, seq}
//   nwd.kvAppendAttention(q, kNew, vNew, kCache, vCache, o, {..., seq, cap})
//       the engine step of runtime.js:389-391 in one launch
//   nwd.q4Gemv(a, {b, scales, zp}, y, {K, N, n_blocks, epilogue, a_f16})
//       kernels/matmul_nbits_sg.wgsl Params {K, N, n_blocks, epilogue}
//       (runtime.js:212-218); the weight object is the engine's q4 buffers;
//       a_f16 = 1 for an fp16 activation vector (the attention output)
//   nwd.q4QkvAppend(hNorm, wq, wk, wv, qOut, kCache, vCache,
//                   {seq, cap, K, n_heads, n_kv_heads, head_dim})
//       the q/k/v GEMVs and both kv_append dispatches of runtime.js:385-390
//   nwd.alloc(bytes) / nwd.upload(buf, typedArray) / nwd.download(buf, typedArray)
//       device buffers through the library's own helpers (nwd_alloc,
//       nwd_memcpy_*), in place of kernels/gpu.js:75-99 / :141; the addon
//       needs no CUDA runtime of its own
//   nwd.mgpuUniqueId() -> Buffer(128)
//   nwd.mgpuInit(id, {world, rank, device, init_deadline_ms, step_deadline_ms})
//   nwd.mgpuDecodeStep(comm, q, kPool, vPool, rowOffset, seqLen, o,
//                      {batch, n_heads, n_kv_heads, head_dim, pool_rows})
//   nwd.mgpuSync(comm) / nwd.mgpuDestroy(comm)
//       the long-context step sharded across GPUs (nwd_mgpu_*): one process
//       per GPU; rank 0's id reaches the other processes by any channel
// Buffers are napi_external wrappers of device pointers, freed when the
// wrapper is garbage-collected.  A non-zero status
// throws Error(nwd_last_error()), as runtime.js throws on errors (:448, :484).
#include <node_api.h>

#include <cstdint>
#include <string>

#include "nwd.h"

namespace {

struct DevBuf {
  void* ptr;
  size_t bytes;
};

napi_value throw_status(napi_env env, int status) {
  std::string msg = std::string(nwd_status_name(status)) + ": " + nwd_last_error();
  napi_throw_error(env, nullptr, msg.c_str());
  return nullptr;
}

void finalize_buf(napi_env, void* data, void*) {
  auto* b = static_cast<DevBuf*>(data);
  if (b->ptr) nwd_free(b->ptr);
  delete b;
}

DevBuf* get_buf(napi_env env, napi_value v) {
  void* data = nullptr;
  if (napi_get_value_external(env, v, &data) != napi_ok) {
    napi_throw_type_error(env, nullptr, "expected a device buffer from nwd.alloc");
    return nullptr;
  }
  return static_cast<DevBuf*>(data);
}

uint32_t get_u32(napi_env env, napi_value obj, const char* key, uint32_t dflt = 0,
                 bool required = true) {
  bool has = false;
  napi_has_named_property(env, obj, key, &has);
  if (!has) {
    if (required) napi_throw_type_error(env, nullptr, (std::string("missing ") + key).c_str());
    return dflt;
  }
  napi_value v;
  napi_get_named_property(env, obj, key, &v);
  uint32_t out = dflt;
  napi_get_value_uint32(env, v, &out);
  return out;
}

// Per-engine scratch: one workspace per attention shape, zeroed once.
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
  uint32_t nh = 0, nkv = 0, hd = 0;
};
Workspace g_ws;

int ensure_ws(uint32_t nh, uint32_t nkv, uint32_t hd) {
  if (g_ws.ptr && g_ws.nh == nh && g_ws.nkv == nkv && g_ws.hd == hd) return NWD_OK;
  size_t bytes = 0;
  int st = nwd_attn_decode_workspace_size(1, nh, nkv, hd, &bytes);
  if (st) return st;
  if (g_ws.ptr) nwd_free(g_ws.ptr);
  g_ws = Workspace{};
  st = nwd_alloc(bytes, &g_ws.ptr);  // zero-filled: ready for its first use
  if (st) return st;
  g_ws.bytes = bytes;
  g_ws.nh = nh;
  g_ws.nkv = nkv;
  g_ws.hd = hd;
  return NWD_OK;
}

napi_value Alloc(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  int64_t bytes = 0;
  napi_get_value_int64(env, argv[0], &bytes);
  auto* b = new DevBuf{nullptr, (size_t)bytes};
  int st = nwd_alloc(b->bytes, &b->ptr);
  if (st) {
    delete b;
    return throw_status(env, st);
  }
  napi_value out;
  napi_create_external(env, b, finalize_buf, nullptr, &out);
  return out;
}

napi_value Copy(napi_env env, napi_callback_info info, bool upload) {
  size_t argc = 2;
  napi_value argv[2];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  DevBuf* b = get_buf(env, argv[0]);
  if (!b) return nullptr;
  napi_typedarray_type type;
  size_t length;
  void* data;
  napi_value ab;
  size_t offset;
  napi_get_typedarray_info(env, argv[1], &type, &length, &data, &ab, &offset);
  size_t elem = (type == napi_uint16_array || type == napi_int16_array) ? 2
                : (type == napi_uint8_array || type == napi_int8_array)   ? 1
                                                                           : 4;
  size_t bytes = length * elem;
  if (bytes > b->bytes) {
    napi_throw_range_error(env, nullptr, "typed array larger than the device buffer");
    return nullptr;
  }
  // pageable JS memory: the upload returns once the data is staged, the
  // download once it has landed (legacy default stream, ordered after the
  // engine's launches)
  int st = upload ? nwd_memcpy_h2d(b->ptr, data, bytes, nullptr)
                  : nwd_memcpy_d2h(data, b->ptr, bytes, nullptr);
  return st ? throw_status(env, st) : nullptr;
}
napi_value Upload(napi_env env, napi_callback_info info) { return Copy(env, info, true); }
napi_value Download(napi_env env, napi_callback_info info) { return Copy(env, info, false); }

napi_value KvAppend(napi_env env, napi_callback_info info) {
  size_t argc = 3;
  napi_value argv[3];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  DevBuf* src = get_buf(env, argv[0]);
  DevBuf* cache = get_buf(env, argv[1]);
  if (!src || !cache) return nullptr;
  uint32_t seq = get_u32(env, argv[2], "seq"), n_kv = get_u32(env, argv[2], "n_kv"),
           hd = get_u32(env, argv[2], "hd");
  uint32_t cap = get_u32(env, argv[2], "cap", (uint32_t)(cache->bytes / (2ull * n_kv * hd)), false);
  int st = nwd_kv_append((const uint16_t*)src->ptr, (uint16_t*)cache->ptr, seq, n_kv, hd, cap,
                         nullptr);
  return st ? throw_status(env, st) : nullptr;
}

napi_value Attention(napi_env env, napi_callback_info info) {
  size_t argc = 5;
  napi_value argv[5];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  DevBuf *q = get_buf(env, argv[0]), *k = get_buf(env, argv[1]), *v = get_buf(env, argv[2]),
         *o = get_buf(env, argv[3]);
  if (!q || !k || !v || !o) return nullptr;
  uint32_t nh = get_u32(env, argv[4], "n_heads"), nkv = get_u32(env, argv[4], "n_kv_heads"),
           hd = get_u32(env, argv[4], "head_dim"), seq = get_u32(env, argv[4], "seq");
  uint32_t cap = get_u32(env, argv[4], "cap", (uint32_t)(k->bytes / (2ull * nkv * hd)), false);
  int st = ensure_ws(nh, nkv, hd);
  if (!st)
    st = nwd_attn_decode((const uint16_t*)q->ptr, (const uint16_t*)k->ptr,
                         (const uint16_t*)v->ptr, (uint16_t*)o->ptr, nh, nkv, hd, seq, cap, 0.0f,
                         g_ws.ptr, g_ws.bytes, nullptr);
  return st ? throw_status(env, st) : nullptr;
}

napi_value KvAppendAttention(napi_env env, napi_callback_info info) {
  size_t argc = 7;
  napi_value argv[7];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  DevBuf *q = get_buf(env, argv[0]), *kn = get_buf(env, argv[1]), *vn = get_buf(env, argv[2]),
         *kc = get_buf(env, argv[3]), *vc = get_buf(env, argv[4]), *o = get_buf(env, argv[5]);
  if (!q || !kn || !vn || !kc || !vc || !o) return nullptr;
  uint32_t nh = get_u32(env, argv[6], "n_heads"), nkv = get_u32(env, argv[6], "n_kv_heads"),
           hd = get_u32(env, argv[6], "head_dim"), seq = get_u32(env, argv[6], "seq");
  uint32_t cap = get_u32(env, argv[6], "cap", (uint32_t)(kc->bytes / (2ull * nkv * hd)), false);
  int st = ensure_ws(nh, nkv, hd);
  if (!st)
    st = nwd_kv_append_attn_decode((const uint16_t*)q->ptr, (const uint16_t*)kn->ptr,
                                   (const uint16_t*)vn->ptr, (uint16_t*)kc->ptr,
                                   (uint16_t*)vc->ptr, (uint16_t*)o->ptr, nh, nkv, hd, seq, cap,
                                   0.0f, g_ws.ptr, g_ws.bytes, nullptr);
  return st ? throw_status(env, st) : nullptr;
}

// {b, scales, zp} -> the three device buffers of one q4 matrix
bool get_q4(napi_env env, napi_value obj, DevBuf** b, DevBuf** s, DevBuf** z) {
  napi_value v;
  const char* keys[3] = {"b", "scales", "zp"};
  DevBuf** outs[3] = {b, s, z};
  for (int i = 0; i < 3; i++) {
    if (napi_get_named_property(env, obj, keys[i], &v) != napi_ok) {
      napi_throw_type_error(env, nullptr, "expected a q4 weight object {b, scales, zp}");
      return false;
    }
    *outs[i] = get_buf(env, v);
    if (!*outs[i]) return false;
  }
  return true;
}

napi_value Q4Gemv(napi_env env, napi_callback_info info) {
  size_t argc = 4;
  napi_value argv[4];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  DevBuf *a = get_buf(env, argv[0]), *y = get_buf(env, argv[2]);
  DevBuf *b = nullptr, *s = nullptr, *z = nullptr;
  if (!a || !y || !get_q4(env, argv[1], &b, &s, &z)) return nullptr;
  const uint32_t K = get_u32(env, argv[3], "K"), N = get_u32(env, argv[3], "N"),
                 nb = get_u32(env, argv[3], "n_blocks"),
                 ep = get_u32(env, argv[3], "epilogue", 0, false),
                 f16 = get_u32(env, argv[3], "a_f16", 0, false);
  int st = f16 ? nwd_q4_gemv_f16a((const uint16_t*)a->ptr, (const uint32_t*)b->ptr,
                                  (const float*)s->ptr, (const uint32_t*)z->ptr, (float*)y->ptr, K,
                                  N, nb, ep, nullptr)
               : nwd_q4_gemv((const float*)a->ptr, (const uint32_t*)b->ptr, (const float*)s->ptr,
                             (const uint32_t*)z->ptr, (float*)y->ptr, K, N, nb, ep, nullptr);
  return st ? throw_status(env, st) : nullptr;
}

napi_value Q4QkvAppend(napi_env env, napi_callback_info info) {
  size_t argc = 8;
  napi_value argv[8];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  DevBuf *h = get_buf(env, argv[0]), *q = get_buf(env, argv[4]), *kc = get_buf(env, argv[5]),
         *vc = get_buf(env, argv[6]);
  DevBuf *bq = nullptr, *sq = nullptr, *zq = nullptr, *bk = nullptr, *sk = nullptr,
         *zk = nullptr, *bv = nullptr, *sv = nullptr, *zv = nullptr;
  if (!h || !q || !kc || !vc || !get_q4(env, argv[1], &bq, &sq, &zq) ||
      !get_q4(env, argv[2], &bk, &sk, &zk) || !get_q4(env, argv[3], &bv, &sv, &zv))
    return nullptr;
  const uint32_t nh = get_u32(env, argv[7], "n_heads"), nkv = get_u32(env, argv[7], "n_kv_heads"),
                 hd = get_u32(env, argv[7], "head_dim"), seq = get_u32(env, argv[7], "seq"),
                 K = get_u32(env, argv[7], "K");
  const uint32_t cap =
      get_u32(env, argv[7], "cap", (uint32_t)(kc->bytes / (2ull * nkv * hd)), false);
  int st = nwd_q4_qkv_append(
      (const float*)h->ptr, (const uint32_t*)bq->ptr, (const float*)sq->ptr,
      (const uint32_t*)zq->ptr, (const uint32_t*)bk->ptr, (const float*)sk->ptr,
      (const uint32_t*)zk->ptr, (const uint32_t*)bv->ptr, (const float*)sv->ptr,
      (const uint32_t*)zv->ptr, (uint16_t*)q->ptr, (uint16_t*)kc->ptr, (uint16_t*)vc->ptr, seq,
      cap, K, nh, nkv, hd, nullptr);
  return st ? throw_status(env, st) : nullptr;
}

// ---- long contexts sharded across GPUs (nwd_mgpu_*) ----
struct Comm {
  nwd_mgpu* m = nullptr;
  DevBuf ws{nullptr, 0};
  uint32_t batch = 0, nh = 0, nkv = 0, hd = 0;
  int world = 0;
};

void finalize_comm(napi_env, void* data, void*) {
  auto* c = static_cast<Comm*>(data);
  if (c->m) nwd_mgpu_destroy(c->m);
  if (c->ws.ptr) nwd_free(c->ws.ptr);
  delete c;
}

napi_value MgpuUniqueId(napi_env env, napi_callback_info) {
  uint8_t id[NWD_MGPU_ID_BYTES];
  int st = nwd_mgpu_unique_id(id);
  if (st) return throw_status(env, st);
  napi_value out;
  void* data = nullptr;
  napi_create_buffer_copy(env, sizeof(id), id, &data, &out);
  return out;
}

napi_value MgpuInit(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  void* id = nullptr;
  size_t len = 0;
  if (napi_get_buffer_info(env, argv[0], &id, &len) != napi_ok || len != NWD_MGPU_ID_BYTES) {
    napi_throw_type_error(env, nullptr, "expected the 128-byte id from mgpuUniqueId");
    return nullptr;
  }
  auto* c = new Comm;
  c->world = (int)get_u32(env, argv[1], "world");
  const int rank = (int)get_u32(env, argv[1], "rank");
  const int device = (int)get_u32(env, argv[1], "device", (uint32_t)rank, false);
  const uint32_t init_ms = get_u32(env, argv[1], "init_deadline_ms", 120000, false);
  const uint32_t step_ms = get_u32(env, argv[1], "step_deadline_ms", 60000, false);
  int st = nwd_mgpu_init(static_cast<const uint8_t*>(id), c->world, rank, device, init_ms, step_ms,
                         &c->m);
  if (st) {
    delete c;
    return throw_status(env, st);
  }
  napi_value out;
  napi_create_external(env, c, finalize_comm, nullptr, &out);
  return out;
}

Comm* get_comm(napi_env env, napi_value v) {
  void* data = nullptr;
  if (napi_get_value_external(env, v, &data) != napi_ok || !data) {
    napi_throw_type_error(env, nullptr, "expected a communicator from mgpuInit");
    return nullptr;
  }
  return static_cast<Comm*>(data);
}

napi_value MgpuDecodeStep(napi_env env, napi_callback_info info) {
  size_t argc = 8;
  napi_value argv[8];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  Comm* c = get_comm(env, argv[0]);
  DevBuf *q = get_buf(env, argv[1]), *k = get_buf(env, argv[2]), *v = get_buf(env, argv[3]),
         *ro = get_buf(env, argv[4]), *sl = get_buf(env, argv[5]), *o = get_buf(env, argv[6]);
  if (!c || !q || !k || !v || !ro || !sl || !o) return nullptr;
  const uint32_t batch = get_u32(env, argv[7], "batch"), nh = get_u32(env, argv[7], "n_heads"),
                 nkv = get_u32(env, argv[7], "n_kv_heads"), hd = get_u32(env, argv[7], "head_dim");
  const uint64_t rows = get_u32(env, argv[7], "pool_rows", (uint32_t)(k->bytes / (2ull * nkv * hd)),
                                false);
  if (!c->ws.ptr || c->batch != batch || c->nh != nh || c->nkv != nkv || c->hd != hd) {
    size_t bytes = 0;
    int st = nwd_mgpu_workspace_size(c->world, batch, nh, nkv, hd, &bytes);
    if (!st && c->ws.ptr) st = nwd_free(c->ws.ptr);
    c->ws = DevBuf{nullptr, 0};
    if (!st) st = nwd_alloc(bytes, &c->ws.ptr);  // zero-filled
    if (st) return throw_status(env, st);
    c->ws.bytes = bytes;
    c->batch = batch;
    c->nh = nh;
    c->nkv = nkv;
    c->hd = hd;
  }
  int st = nwd_mgpu_decode_step(c->m, (const uint16_t*)q->ptr, (const uint16_t*)k->ptr,
                                (const uint16_t*)v->ptr, rows, (const int64_t*)ro->ptr,
                                (const int32_t*)sl->ptr, (uint16_t*)o->ptr, batch, nh, nkv, hd,
                                0.0f, c->ws.ptr, c->ws.bytes, nullptr);
  return st ? throw_status(env, st) : nullptr;
}

napi_value MgpuSync(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  Comm* c = get_comm(env, argv[0]);
  if (!c) return nullptr;
  int st = nwd_mgpu_sync(c->m);
  return st ? throw_status(env, st) : nullptr;
}

napi_value MgpuDestroy(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr);
  Comm* c = get_comm(env, argv[0]);
  if (!c) return nullptr;
  int st = nwd_mgpu_destroy(c->m);
  c->m = nullptr;  // the finalizer frees the rest
  return st ? throw_status(env, st) : nullptr;
}

napi_value Init(napi_env env, napi_value exports) {
  napi_property_descriptor props[] = {
      {"alloc", nullptr, Alloc, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"upload", nullptr, Upload, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"download", nullptr, Download, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"kvAppend", nullptr, KvAppend, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"attention", nullptr, Attention, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"kvAppendAttention", nullptr, KvAppendAttention, nullptr, nullptr, nullptr, napi_default,
       nullptr},
      {"q4Gemv", nullptr, Q4Gemv, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"q4QkvAppend", nullptr, Q4QkvAppend, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"mgpuUniqueId", nullptr, MgpuUniqueId, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"mgpuInit", nullptr, MgpuInit, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"mgpuDecodeStep", nullptr, MgpuDecodeStep, nullptr, nullptr, nullptr, napi_default,
       nullptr},
      {"mgpuSync", nullptr, MgpuSync, nullptr, nullptr, nullptr, napi_default, nullptr},
      {"mgpuDestroy", nullptr, MgpuDestroy, nullptr, nullptr, nullptr, napi_default, nullptr},
  };
  napi_define_properties(env, exports, sizeof(props) / sizeof(props[0]), props);
  return exports;
}

}  // namespace

NAPI_MODULE(NODE_GYP_MODULE_NAME, Init)
