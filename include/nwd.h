/*
 * nwd.h — C ABI of the B200 (sm_100a) decode-attention engine.
 *
 * This library replaces the two WGSL dispatch sites of the Nemotron WebGPU
 * decode engine's attention layers:
 *   - kernels/kv_append.wgsl   (KV-cache row write, dispatched at engine/runtime.js:389-390)
 *   - kernels/sparse_attn.wgsl (GQA decode attention, dispatched at engine/runtime.js:391)
 * and extends them to ragged batches, long contexts and multi-GPU shards.
 *
 * Conventions
 *   - Every entry point returns an int status: NWD_OK (0) or one of NWD_ERR_*.
 *     On error nothing is launched and nwd_last_error() returns a message
 *     (thread-local, valid until the next call on the same thread).  This
 *     mirrors the reference's throw-on-error style (engine/runtime.js:448,
 *     kernels/gpu.js:127-131): a JS shim turns a non-zero status into
 *     `throw new Error(nwd_last_error())`.
 *   - Tensors are device pointers.  fp16 data are passed as `uint16_t*`
 *     (IEEE binary16 bit patterns).  Buffers are owned by the caller; the
 *     library never allocates or frees caller memory.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Calls are stream-ordered and asynchronous.
 *   - KV caches are token-major, exactly as the reference lays them out
 *     (kernels/sparse_attn.wgsl:49,107; kernels/kv_append.wgsl:17):
 *     element (t, h, i) of a cache lives at ((t * n_kv + h) * hd + i).
 *   - Softmax scale: pass 0.0f for the reference's inverseSqrt(head_dim)
 *     (kernels/sparse_attn.wgsl:42).
 *   - The attention kernels support head_dim == 128 and a GQA group
 *     n_heads / n_kv_heads in 1..8 (the engine uses 40/8 = 5,
 *     engine/config.js:10-12).  Other shapes return NWD_ERR_UNSUPPORTED.
 */
#ifndef NWD_H
#define NWD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NWD_OK 0
#define NWD_ERR_INVALID 1     /* null pointer, zero shape, n_heads % n_kv_heads != 0 */
#define NWD_ERR_RANGE 2       /* seq >= cache capacity (engine/runtime.js:448) */
#define NWD_ERR_UNSUPPORTED 3 /* shape outside the kernels' supported set */
#define NWD_ERR_WORKSPACE 4   /* workspace missing, too small or misaligned */
#define NWD_ERR_CUDA 5        /* CUDA runtime / driver error */
#define NWD_ERR_NCCL 6        /* NCCL missing or a collective failed */
#define NWD_ERR_TIMEOUT 7     /* a bounded device- or host-side wait gave up */
#define NWD_ERR_DEVICE 8      /* a kernel recorded an error in its workspace */

/* Last error message of the calling thread ("" if none). */
const char* nwd_last_error(void);
/* Library version string. */
const char* nwd_version(void);
/* Name of a status code. */
const char* nwd_status_name(int status);

/* ------------------------------------------------------------------ */
/* KV-cache append                                                     */
/* ------------------------------------------------------------------ */

/* kernels/kv_append.wgsl:1-18 — cache[seq * n_kv * hd + i] = src[i] for
 * i < n_kv * hd.  Argument order follows the WGSL Params {seq, n_kv, hd}.
 * `cap` is the cache capacity in rows (engine/config.js:24 maxSeq); seq >= cap
 * returns NWD_ERR_RANGE without launching (engine/runtime.js:448). Bit-exact. */
int nwd_kv_append(const uint16_t* src, uint16_t* cache, uint32_t seq, uint32_t n_kv,
                  uint32_t hd, uint32_t cap, void* stream);

/* The engine's two kv_append dispatches (K then V, engine/runtime.js:389-390)
 * as one launch. */
int nwd_kv_append_kv(const uint16_t* k_src, const uint16_t* v_src, uint16_t* k_cache,
                     uint16_t* v_cache, uint32_t seq, uint32_t n_kv, uint32_t hd, uint32_t cap,
                     void* stream);

/* Ragged batch of the same write: sequence b writes its row pos[b] of a
 * region that starts at pool row row_offset[b].
 *   k_src, v_src : [batch, n_kv, hd]
 *   k_pool, v_pool: [pool_rows, n_kv, hd]
 *   row_offset   : device int64[batch];  pos: device int32[batch]
 * Rows with row_offset[b] + pos[b] outside [0, pool_rows) are skipped and
 * counted in the optional device word `*err_count` (may be NULL). */
int nwd_kv_append_batched(const uint16_t* k_src, const uint16_t* v_src, uint16_t* k_pool,
                          uint16_t* v_pool, uint64_t pool_rows, const int64_t* row_offset,
                          const int32_t* pos, uint32_t batch, uint32_t n_kv, uint32_t hd,
                          uint32_t* err_count, void* stream);

/* ------------------------------------------------------------------ */
/* Decode attention (split-KV flash-decode)                            */
/* ------------------------------------------------------------------ */

/* Bytes of workspace the decode calls below need for `batch` sequences on
 * the current device.  The workspace must be zero-filled once before its
 * first use (nwd_workspace_init or cudaMemset); every call leaves it ready
 * for the next.  Its layout follows the call's (batch, n_heads, n_kv_heads,
 * head_dim): use one workspace per shape, or zero it again before using it
 * for another.  Calls that share one workspace must not overlap on the GPU.
 * The base pointer must be 256-byte aligned.  If nwd_workspace_check reports
 * a device error, zero the workspace before reusing it. */
int nwd_attn_decode_workspace_size(uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                                   uint32_t head_dim, size_t* bytes);

/* Zero-fills a workspace on `stream`. */
int nwd_workspace_init(void* workspace, size_t ws_bytes, void* stream);

/* Reads (synchronously, on `stream`) and clears the device-side error word
 * of a workspace: 0 = no error, else a NWD_DEVERR_* code. */
int nwd_workspace_check(void* workspace, size_t ws_bytes, uint32_t* device_error,
                        void* stream);

#define NWD_DEVERR_PIPE_TIMEOUT 1u  /* an mbarrier wait hit its iteration limit */
#define NWD_DEVERR_ROW_RANGE 2u     /* a row index fell outside the pool */

/* Failure-detection self-test: launches one CTA whose bounded mbarrier wait
 * (the one every kernel here uses) is made to run out; after about 2 s the
 * kernel returns and the workspace's error word holds
 * NWD_DEVERR_PIPE_TIMEOUT (read it with nwd_workspace_check).  The stream and
 * the context stay usable.  No counterpart in the reference (its waits are
 * WebGPU barriers; failures surface through error scopes, runtime.js:474-487). */
int nwd_selftest_wait_timeout(void* workspace, size_t ws_bytes, void* stream);

/* Softmax `scale` below: finite and >= 0; 0 selects the reference's
 * inverseSqrt(head_dim). */

/* kernels/sparse_attn.wgsl:32-113 — for each query head h:
 *   O[h,:] = softmax(scale * Q[h,:] . K[t, h/group, :]^T, t < seq) . V[t, h/group, :]
 * The first four scalars are the WGSL Params {n_heads, n_kv_heads, head_dim,
 * seq} (kernels/sparse_attn.wgsl:12-17); `seq` is the number of cached rows
 * attended (the engine passes this.seq + 1, engine/runtime.js:452).
 *   q: [n_heads, head_dim]   k_cache, v_cache: [cap, n_kv_heads, head_dim]
 *   o: [n_heads, head_dim]   fp16 in, fp32 accumulation, fp16 out.
 * seq == 0 writes zeros (the WGSL's acc stays 0). */
int nwd_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                    uint16_t* o, uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                    uint32_t seq, uint32_t cap, float scale, void* workspace, size_t ws_bytes,
                    void* stream);

/* Same computation as nwd_attn_decode, for callers that cannot allocate
 * device memory: a host that only receives buffers it did not create (a
 * JavaScript engine handing over existing GPU buffers through an addon, an
 * embedder with a fixed memory budget) has no way to provide the workspace.
 * This entry point takes none.  It allocates nothing; its scratch is a
 * fixed array built into the library (about 1.3 MB, which every GPU that
 * loads the library keeps until the process exits), sized for one sequence
 * with up to 64 kv heads on up to 160 SMs; larger shapes return
 * NWD_ERR_UNSUPPORTED.  The first call on a device looks up the scratch's
 * device address; make that first call before any stream capture.  All calls
 * share the one scratch: calls that may overlap on the GPU (different
 * streams, or different host threads) race and must be serialised by the
 * caller.  A call that uses the scratch (more than 2048 rows) clears its
 * merge tickets on `stream` before its launch; the scratch's device error
 * word is kept across calls until nwd_noalloc_check reads it.  No
 * counterpart in the reference. */
int nwd_attn_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                            uint16_t* o, uint32_t n_heads, uint32_t n_kv_heads,
                            uint32_t head_dim, uint32_t seq, uint32_t cap, float scale,
                            void* stream);

/* Reads (synchronously, on `stream`) and clears the device error word of the
 * built-in scratch of nwd_attn_decode_noalloc on the current device: 0 = no
 * error since the last check, else NWD_DEVERR_* bits (a bounded wait that
 * gave up, a row outside the cache).  The counterpart of nwd_workspace_check
 * for callers without a workspace; allocates nothing. */
int nwd_noalloc_check(uint32_t* device_error, void* stream);

/* How a decode call of this shape runs on the current device, without
 * launching anything: batch 1 plans nwd_attn_decode of `seq` rows (and the
 * fused step attending `seq` rows), batch > 1 the batched entry points
 * (`seq` is ignored).  kernel: 0 = the split-KV kernel, 1 = the short
 * single-sequence kernel; grid: CTAs; split: pieces per kv head of a single
 * sequence (0 = the batch's flattened split); cluster: CTAs per thread-block
 * cluster whose pieces merge over distributed shared memory (0 = none);
 * groups: consumer warp groups of the split-KV kernel.  No counterpart in the
 * reference (its attention is one fixed dispatch, engine/runtime.js:391). */
int nwd_attn_decode_plan(uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                         uint32_t head_dim, uint32_t seq, int* kernel, int* grid, int* split,
                         int* cluster, int* groups);

/* One engine attention step (engine/runtime.js:389-391 with the uniforms of
 * :451-452): writes k_new/v_new ([n_kv_heads, head_dim]) into row `seq` of the
 * caches, then attends over rows 0..seq (seq + 1 rows), in one launch. */
int nwd_kv_append_attn_decode(const uint16_t* q, const uint16_t* k_new, const uint16_t* v_new,
                              uint16_t* k_cache, uint16_t* v_cache, uint16_t* o,
                              uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                              uint32_t seq, uint32_t cap, float scale, void* workspace,
                              size_t ws_bytes, void* stream);

/* Ragged batch of independent sequences sharing one KV pool.
 *   q, o        : [batch, n_heads, head_dim]
 *   k_pool, v_pool: [pool_rows, n_kv_heads, head_dim]
 *   row_offset  : device int64[batch] — first pool row of sequence b
 *   seq_len     : device int32[batch] — rows attended for sequence b
 * batch <= 4096 per call. */
int nwd_attn_decode_batched(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                            uint64_t pool_rows, const int64_t* row_offset,
                            const int32_t* seq_len, uint16_t* o, uint32_t batch,
                            uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                            float scale, void* workspace, size_t ws_bytes, void* stream);

/* Batched engine step: sequence b writes k_new/v_new[b] into its row pos[b],
 * then attends over pos[b] + 1 rows.  One launch. */
int nwd_kv_append_attn_decode_batched(const uint16_t* q, const uint16_t* k_new,
                                      const uint16_t* v_new, uint16_t* k_pool, uint16_t* v_pool,
                                      uint64_t pool_rows, const int64_t* row_offset,
                                      const int32_t* pos, uint16_t* o, uint32_t batch,
                                      uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim,
                                      float scale, void* workspace, size_t ws_bytes,
                                      void* stream);

/* Partial attention over a shard of each sequence's rows, for merging across
 * shards (GPUs).  Same inputs as nwd_attn_decode_batched; instead of O it
 * writes, per (b, h), a triple (m, l, o) with
 *   l * 2^m = sum_t 2^(s_t*log2(e))          o[i] * 2^m = sum_t 2^(s_t*log2(e)) * V[t,i]
 *   part_ml[(b*n_heads+h)*2 + 0] = m,  part_ml[(b*n_heads+h)*2 + 1] = l,
 *   part_o [(b*n_heads+h)*head_dim + i] = o[i],
 * where s_t = scale * q.k_t and m (log2 units) is a reference maximum within
 * 8 of max_t s_t*log2(e) (m <= the true maximum, so every term is <= 2^8).
 * An empty shard writes m = -inf, l = 0, o = 0. */
int nwd_attn_decode_partial(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                            uint64_t pool_rows, const int64_t* row_offset,
                            const int32_t* seq_len, float* part_o, float* part_ml,
                            uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                            uint32_t head_dim, float scale, void* workspace, size_t ws_bytes,
                            void* stream);

/* Log-sum-exp merge of `shards` partials laid out [shards][batch*n_heads][...]
 * (as nwd_attn_decode_partial writes them) into o [batch, n_heads, head_dim]
 * fp16: o = sum_r o_r 2^(m_r - M) / sum_r l_r 2^(m_r - M), M = max_r m_r.
 * Shards are merged in index order. */
int nwd_attn_merge(const float* part_o, const float* part_ml, uint16_t* o, uint32_t shards,
                   uint32_t batch, uint32_t n_heads, uint32_t head_dim, void* stream);

/* The same merge over packed partials: shard s occupies
 * packed[s * R * (head_dim + 2) ...], R = batch * n_heads, holding its o
 * ([R][head_dim], as part_o) followed by its (m, l) pairs ([R][2], as
 * part_ml).  A rank that points nwd_attn_decode_partial's part_o / part_ml at
 * the two halves of one buffer can exchange its partials with a single
 * all-gather and merge the gathered [shards][...] buffer here.  At most 4096
 * shards.  No counterpart in the reference (it has no multi-device code). */
int nwd_attn_merge_packed(const float* packed, uint16_t* o, uint32_t shards, uint32_t batch,
                          uint32_t n_heads, uint32_t head_dim, void* stream);

/* ------------------------------------------------------------------ */
/* Long contexts sharded across GPUs (NCCL over NVLink)                */
/* ------------------------------------------------------------------ */

/* One process (or thread) per GPU.  Each sequence's cached rows are split into
 * contiguous shards, one per rank; a step computes every rank's shard partial
 * (nwd_attn_decode_partial), all-gathers the packed partials with NCCL and
 * merges them in rank order (nwd_attn_merge_packed), so every rank ends with
 * the full O.  The reference has no multi-device code: this extends its
 * single-sequence attention (kernels/sparse_attn.wgsl:32-113, dispatched at
 * engine/runtime.js:391) to rows held by several GPUs.
 *
 * When every rank can map every other rank's memory (NVLink / NVSwitch) the
 * exchange runs over peer memory: the shard partial kernel writes each pair's
 * partial into every rank's exchange buffer (allocated by the library with the
 * driver's virtual-memory API, its file descriptor passed to the peers over a
 * Unix-domain socket) and a merge kernel on each rank waits, bounded, for all
 * ranks' flags; otherwise (or with NWD_MGPU_P2P=0) by NCCL all-gather.
 * NCCL is loaded at run time on the first nwd_mgpu_* call (NWD_NCCL_LIBRARY,
 * else libnccl.so.2 as the process finds it).  Communicators are
 * non-blocking: every wait (set-up, enqueue, step completion, finalize) runs
 * under a host-side deadline; when it passes, or NCCL reports an error, the
 * communicator is aborted (ncclCommAbort ends its kernels), the call returns
 * NWD_ERR_TIMEOUT or NWD_ERR_NCCL and the handle only accepts
 * nwd_mgpu_destroy / nwd_mgpu_abort.  This is how a rank learns that a peer
 * left: its next step's wait runs out instead of hanging (the reference's
 * counterpart is WebGPU device loss, engine/runtime.js:474-487, :700-715). */

#define NWD_MGPU_ID_BYTES 128
typedef struct nwd_mgpu nwd_mgpu;

/* A new communicator id (on one rank; every rank passes the same bytes to
 * nwd_mgpu_init). */
int nwd_mgpu_unique_id(uint8_t* id /* [NWD_MGPU_ID_BYTES] */);

/* Joins the communicator as `rank` of `world` on `device` (made current).
 * init_deadline_ms bounds the set-up (all ranks must join within it);
 * step_deadline_ms bounds every later wait. */
int nwd_mgpu_init(const uint8_t* id, int world, int rank, int device, uint32_t init_deadline_ms,
                  uint32_t step_deadline_ms, nwd_mgpu** out);

/* Workspace bytes for nwd_mgpu_decode_step on the current device: the shard
 * partial's workspace plus the gathered partials ([world][batch * n_heads *
 * (head_dim + 2)] f32).  Zero it once (nwd_workspace_init); 256-byte aligned. */
int nwd_mgpu_workspace_size(int world, uint32_t batch, uint32_t n_heads, uint32_t n_kv_heads,
                            uint32_t head_dim, size_t* bytes);

/* One sharded step, asynchronous on `stream`: this rank's rows of sequence b
 * are pool rows [row_offset[b], row_offset[b] + seq_len[b]) (device arrays,
 * as nwd_attn_decode_partial); q [batch, n_heads, head_dim] must be the same
 * on every rank; every rank receives o [batch, n_heads, head_dim] fp16.  All
 * ranks must make the same calls in the same order.  Returns once the step is
 * enqueued (or the enqueue's wait ran out); nwd_mgpu_sync waits for it. */
int nwd_mgpu_decode_step(nwd_mgpu* m, const uint16_t* q, const uint16_t* k_pool,
                         const uint16_t* v_pool, uint64_t pool_rows, const int64_t* row_offset,
                         const int32_t* seq_len, uint16_t* o, uint32_t batch, uint32_t n_heads,
                         uint32_t n_kv_heads, uint32_t head_dim, float scale, void* workspace,
                         size_t ws_bytes, void* stream);

/* Waits (polling, within step_deadline_ms) for the last step enqueued on this
 * handle.  On a deadline or an NCCL error it aborts the communicator, lets
 * the stream drain and returns NWD_ERR_TIMEOUT / NWD_ERR_NCCL. */
int nwd_mgpu_sync(nwd_mgpu* m);

/* Per-step device timing (CUDA events around the shard partial and around
 * the all-gather + merge), off by default. */
int nwd_mgpu_set_timing(nwd_mgpu* m, int on);
int nwd_mgpu_step_times(nwd_mgpu* m, float* partial_ms, float* exchange_ms);

/* Finalizes (within step_deadline_ms; aborts if that runs out) and frees. */
int nwd_mgpu_destroy(nwd_mgpu* m);
/* Aborts without waiting for peers (a rank leaving) and frees. */
int nwd_mgpu_abort(nwd_mgpu* m);
/* The loaded NCCL's version code (e.g. 22809). */
int nwd_mgpu_nccl_version(int* version);
/* How the steps exchange partials: 1 = over peer memory (the partial kernel
 * writes each pair's partial into every rank's exchange buffer, a merge
 * kernel waits for all ranks' flags), -1 = NCCL all-gather + merge (some rank
 * could not map every other rank's memory, or NWD_MGPU_P2P=0), 0 = not
 * decided yet (no step made).  Decided collectively on the first step of a
 * shape. */
int nwd_mgpu_exchange_mode(nwd_mgpu* m, int* mode);

/* ------------------------------------------------------------------ */
/* Device memory and streams for hosts without a CUDA runtime          */
/* ------------------------------------------------------------------ */

/* The addon's (or a C engine's) buffer and queue helpers, in place of the
 * reference's WebGPU helpers (kernels/gpu.js:75-99 createBuffer /
 * createEmptyStorage / createUniform, :141 dispatchAndRead). */
int nwd_set_device(int device);
int nwd_device_count(int* count);
/* Zero-filled device memory (256-byte aligned, as every workspace needs). */
int nwd_alloc(size_t bytes, void** ptr);
int nwd_free(void* ptr);
/* Asynchronous on `stream`; a pinned `src` must stay unchanged until the
 * stream has passed the copy, a pageable one may be reused on return. */
int nwd_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
/* Returns once `dst` holds the data (the stream is synchronised). */
int nwd_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int nwd_stream_create(void** stream);
int nwd_stream_destroy(void* stream);
int nwd_stream_synchronize(void* stream);

/* ------------------------------------------------------------------ */
/* The q4 projections either side of the path                          */
/* ------------------------------------------------------------------ */

/* kernels/matmul_nbits_sg.wgsl (the engine's decode GEMV, picked by
 * engine/runtime.js:221-233, params uniform runtime.js:212-218): Y[N] f32 from
 * A[K] f32 and 4-bit weights in the MatMulNBits layout the engine loads:
 * b = [N][n_blocks][4] u32 (32 values per block, element j of a word in bits
 * [4j, 4j+4), 16-byte aligned), scales = [N][n_blocks] f32, zp = 4-bit zero
 * points packed 8 per u32, nibble n*n_blocks + blk.  Element value
 * (q - zero) * scale; K must be 32 * n_blocks (at most 14080).  epilogue:
 * 0 = store, 1 = relu2 (matmul_nbits_sg.wgsl:76-79, the MLP up projection),
 * 2 = Y[n] += result (the residual add of kernels/add.wgsl fused, as
 * runtime.js:392-393 applies it after o_proj). */
int nwd_q4_gemv(const float* a, const uint32_t* b, const float* scales, const uint32_t* zp,
                float* y, uint32_t K, uint32_t N, uint32_t n_blocks, uint32_t epilogue,
                void* stream);

/* The same GEMV with A in fp16, for o_proj fed by the fp16 attention output
 * (the reference's attention output buffer is f32: runtime.js:334). */
int nwd_q4_gemv_f16a(const uint16_t* a, const uint32_t* b, const float* scales,
                     const uint32_t* zp, float* y, uint32_t K, uint32_t N, uint32_t n_blocks,
                     uint32_t epilogue, void* stream);

/* An attention layer's three projections in one launch, with the token's
 * k / v written straight into the caches: runtime.js:389-391's q, k and v
 * GEMVs (:321-329) followed by kv_append of k and of v.  h = the normalised
 * hidden state [K] f32; q_out [n_heads * head_dim] fp16; the k and v results
 * go to cache row `seq` ([cap][n_kv_heads][head_dim] fp16).  seq >= cap fails
 * with "seq N exceeds maxSeq M" (runtime.js:448) before any launch. */
int nwd_q4_qkv_append(const float* h, const uint32_t* bq, const float* sq, const uint32_t* zq,
                      const uint32_t* bk, const float* sk, const uint32_t* zk, const uint32_t* bv,
                      const float* sv, const uint32_t* zv, uint16_t* q_out, uint16_t* k_cache,
                      uint16_t* v_cache, uint32_t seq, uint32_t cap, uint32_t K,
                      uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, void* stream);

/* L2 prefetch of up to 16 device buffers (ptrs[i], bytes[i]; host arrays),
 * e.g. the next projection's q4 weights, issued on a side stream while a
 * latency-bound kernel leaves HBM idle.  A hint only: it moves no data into
 * any SM, orders nothing and never changes a result.  No counterpart in the
 * reference (runtime.js:385-394 runs the layer's dispatches back to back). */
int nwd_prefetch_l2(const void* const* ptrs, const uint64_t* bytes, uint32_t n, void* stream);

/* ------------------------------------------------------------------ */
/* Prompt chunks (causal prefill)                                      */
/* ------------------------------------------------------------------ */

/* The kv_append path for a prompt chunk: kernels/kv_append.wgsl:13-18 for
 * n_rows consecutive rows per sequence.  Sequence b's rows
 * [b, 0..n_rows) of k_src / v_src ([batch, n_rows, n_kv, hd]) go to pool rows
 * row_offset[b] + start_pos + i.  Rows outside the pool are skipped and
 * flagged (NWD_DEVERR_ROW_RANGE) in the workspace's error word when a
 * workspace is given (may be NULL).  Bit-exact. */
int nwd_kv_append_rows(const uint16_t* k_src, const uint16_t* v_src, uint16_t* k_pool,
                       uint16_t* v_pool, uint64_t pool_rows, const int64_t* row_offset,
                       uint32_t start_pos, uint32_t n_rows, uint32_t batch, uint32_t n_kv,
                       uint32_t hd, void* workspace, size_t ws_bytes, void* stream);

/* Causal attention for a prompt chunk of n_q tokens per sequence on the
 * tcgen05 tensor cores (TMEM accumulators).  The reference feeds a prompt one
 * decode step per token (engine/runtime.js:640-643), so token i of a chunk
 * whose K/V rows sit at start_pos .. start_pos+n_q-1 attends rows
 * 0 .. start_pos+i: kernels/sparse_attn.wgsl once per token, computed here as
 * one dense contraction.
 *   q, o          : [batch, n_q, n_heads, head_dim]
 *   k_pool, v_pool: [pool_rows, n_kv_heads, head_dim]; sequence b's rows start
 *                   at pool row row_offset[b] (device int64[batch]) and must
 *                   already hold the chunk's rows (nwd_kv_append_rows)
 * head_dim 128; any GQA group.  workspace: >= 256 bytes, zeroed, 256-byte
 * aligned (a decode workspace serves); its first word receives device errors. */
int nwd_attn_prefill(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                     uint64_t pool_rows, const int64_t* row_offset, uint16_t* o, uint32_t batch,
                     uint32_t n_q, uint32_t start_pos, uint32_t n_heads, uint32_t n_kv_heads,
                     uint32_t head_dim, float scale, void* workspace, size_t ws_bytes,
                     void* stream);

/* ------------------------------------------------------------------ */
/* Synthetic inputs                                                    */
/* ------------------------------------------------------------------ */

/* Fills dst[0..n) with the deterministic fp16 N(0,1) stream element
 * offset+i of `seed` (Irwin-Hall sum of 12 16-bit uniforms from splitmix64,
 * integer-exact, bit-identical to the CPU oracle's generator). */
int nwd_fill_normal_f16(uint16_t* dst, uint64_t n, uint64_t seed, uint64_t offset,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NWD_H */
