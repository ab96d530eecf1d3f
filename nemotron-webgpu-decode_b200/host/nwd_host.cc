// nwd_host: a C++ engine host that drives the decode-attention path through
// the C ABI (include/nwd.h) alone: no Python, no PyTorch, no CUDA runtime of
// its own (libnwd.so carries it).  It stands where engine/runtime.js stands
// when its attention dispatch sites call the library instead of WGSL, so it
// shows the boundary works for a host that is not this package's Python.
//
//   nwd_host trace --out O.bin [--expect E.bin] [--fused 0|1] [--device D]
//       The engine's attention-layer sequence for config 1 (engine/config.js:
//       Hq 40, Hkv 8, head_dim 128, maxSeq 256), ordered as
//       DecodeEngine.submitStep orders it (engine/runtime.js:447-467): the
//       seq < maxSeq guard (:448), kv_append of K and V at row seq and the
//       attention over seq + 1 rows (:389-391 with the uniforms of :451-452),
//       then seq += 1 (:467); 24 prompt tokens and 127 new ones as generate
//       runs them (:640-646), i.e. 151 steps.  The step's q / k / v come from
//       the library's deterministic generator on the device (where the
//       engine's projections would write them).  Writes the 151 outputs
//       (fp16 [151][40][128]) to O.bin; with --expect (f32, same shape) it
//       reports the largest errors against it.  Then it keeps stepping until
//       the guard fires at seq 256 and records the error message, resets the
//       caches as reset() does (:630-631) and checks that step 0 again gives
//       the first run's output bit for bit.  One JSON line on stdout.
//
//   nwd_host mgpu --world N --rank R --id-file F [--device D] [--batch B]
//                 [--rows L] [--heads 32] [--kv-heads 8] [--steps S]
//                 [--leave-after K] [--init-deadline-ms T] [--step-deadline-ms T]
//                 [--out O.bin]
//       One rank of the long-context decode sharded across GPUs
//       (nwd_mgpu_*): rank R holds rows [L*R/N, L*(R+1)/N) of each of B
//       sequences, generated as the bench's config 5 generates them (seeds
//       5000 / 5001 at the global row's element offset; q seed 5002).  Rank 0
//       creates the communicator id and publishes it in F (written to F.tmp,
//       then renamed); the others wait for F.  Rank 0 writes the final O
//       (fp16 [B][heads][128]) to O.bin.  With --leave-after K the last rank
//       leaves after K completed steps (nothing of it in flight: it aborts its
//       communicator locally and exits); every other rank's next step must
//       then end with an error status within its step deadline, after which
//       the rank runs a single-GPU decode to show its context still works.
//       One JSON line per rank on stdout.
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <chrono>
#include <cmath>
#include <string>
#include <thread>
#include <vector>

#include "nwd.h"

namespace {

struct Args {
  std::vector<std::string> v;
  std::string get(const char* key, const char* def) const {
    for (size_t i = 0; i + 1 < v.size(); i++)
      if (v[i] == key) return v[i + 1];
    return def ? def : "";
  }
  long num(const char* key, long def) const {
    std::string s = get(key, nullptr);
    return s.empty() ? def : strtol(s.c_str(), nullptr, 10);
  }
};

std::string json_str(const std::string& s) {
  std::string o = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\') {
      o += '\\';
      o += c;
    } else if ((unsigned char)c < 0x20) {
      o += ' ';
    } else {
      o += c;
    }
  }
  return o + "\"";
}

// Ends the program with a JSON error line when a call fails unexpectedly.
void need(int st, const char* what) {
  if (st != NWD_OK) {
    printf("{\"ok\": false, \"failed\": %s, \"status\": %s, \"message\": %s}\n",
           json_str(what).c_str(), json_str(nwd_status_name(st)).c_str(),
           json_str(nwd_last_error()).c_str());
    fflush(stdout);
    exit(2);
  }
}

float h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      exp = 127 - 15 + 1;
      while (!(man & 0x400)) {
        man <<= 1;
        exp--;
      }
      bits = sign | (exp << 23) | ((man & 0x3ff) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

bool write_file(const std::string& path, const void* p, size_t n) {
  FILE* f = fopen(path.c_str(), "wb");
  if (!f) return false;
  const bool ok = fwrite(p, 1, n, f) == n;
  return fclose(f) == 0 && ok;
}

bool read_file(const std::string& path, void* p, size_t n) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  const bool ok = fread(p, 1, n, f) == n;
  fclose(f);
  return ok;
}

// ------------------------------------------------------------------ trace

int run_trace(const Args& a) {
  const uint32_t HQ = 40, HKV = 8, HD = 128, MAXSEQ = 256;  // engine/config.js:10-12,24
  const uint32_t PROMPT = 24, NEW = 128;
  const uint32_t STEPS = PROMPT + NEW - 1;  // generate(): prompt steps + (newTokens - 1)
  const bool fused = a.num("--fused", 1) != 0;
  const std::string out_path = a.get("--out", "");
  const std::string expect_path = a.get("--expect", "");
  need(nwd_set_device((int)a.num("--device", 0)), "nwd_set_device");
  void* stream = nullptr;
  need(nwd_stream_create(&stream), "nwd_stream_create");

  // the engine's buffers (runtime.js:120-123, :170-173): q, k, v, attnO and one
  // attention layer's caches, created once
  const size_t row = (size_t)HKV * HD, qn = (size_t)HQ * HD;
  void *q, *k, *v, *o, *kc, *vc, *ws;
  need(nwd_alloc(qn * 2, &q), "nwd_alloc");
  need(nwd_alloc(row * 2, &k), "nwd_alloc");
  need(nwd_alloc(row * 2, &v), "nwd_alloc");
  need(nwd_alloc(qn * 2, &o), "nwd_alloc");
  need(nwd_alloc(MAXSEQ * row * 2, &kc), "nwd_alloc");
  need(nwd_alloc(MAXSEQ * row * 2, &vc), "nwd_alloc");
  size_t ws_bytes = 0;
  need(nwd_attn_decode_workspace_size(1, HQ, HKV, HD, &ws_bytes), "workspace_size");
  need(nwd_alloc(ws_bytes, &ws), "nwd_alloc");  // zero-filled: ready for first use

  uint32_t seq = 0;  // DecodeEngine.seq
  std::string guard_msg;
  int guard_status = NWD_OK;
  // one submitStep: the step's q/k/v (written by the projections in the
  // engine; here by the generator), the guard, the dispatches, seq += 1
  auto submit_step = [&](uint32_t s) -> int {
    need(nwd_fill_normal_f16((uint16_t*)q, qn, 101, (uint64_t)s * qn, stream), "fill q");
    need(nwd_fill_normal_f16((uint16_t*)k, row, 102, (uint64_t)s * row, stream), "fill k");
    need(nwd_fill_normal_f16((uint16_t*)v, row, 103, (uint64_t)s * row, stream), "fill v");
    int st;
    if (fused) {
      st = nwd_kv_append_attn_decode((const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v,
                                     (uint16_t*)kc, (uint16_t*)vc, (uint16_t*)o, HQ, HKV, HD, seq,
                                     MAXSEQ, 0.0f, ws, ws_bytes, stream);
    } else {  // the reference's three dispatches, one for one
      st = nwd_kv_append((const uint16_t*)k, (uint16_t*)kc, seq, HKV, HD, MAXSEQ, stream);
      if (st == NWD_OK)
        st = nwd_kv_append((const uint16_t*)v, (uint16_t*)vc, seq, HKV, HD, MAXSEQ, stream);
      if (st == NWD_OK)
        st = nwd_attn_decode((const uint16_t*)q, (const uint16_t*)kc, (const uint16_t*)vc,
                             (uint16_t*)o, HQ, HKV, HD, seq + 1, MAXSEQ, 0.0f, ws, ws_bytes,
                             stream);
    }
    if (st == NWD_OK) seq += 1;
    return st;
  };

  std::vector<uint16_t> outs((size_t)STEPS * qn);
  for (uint32_t s = 0; s < STEPS; s++) {
    need(submit_step(s), "step");
    need(nwd_memcpy_d2h(&outs[(size_t)s * qn], o, qn * 2, stream), "read o");
  }
  uint32_t dev_err = 0;
  need(nwd_workspace_check(ws, ws_bytes, &dev_err, stream), "nwd_workspace_check");

  // errors against the expected outputs (max-abs; max-rel with a 1e-3 floor)
  double max_abs = -1.0, max_rel = -1.0;
  bool finite = true;
  if (!expect_path.empty()) {
    std::vector<float> ref((size_t)STEPS * qn);
    if (!read_file(expect_path, ref.data(), ref.size() * 4)) {
      printf("{\"ok\": false, \"failed\": \"reading --expect\"}\n");
      return 2;
    }
    max_abs = max_rel = 0.0;
    for (size_t i = 0; i < ref.size(); i++) {
      const double g = h2f(outs[i]);
      if (!std::isfinite(g)) finite = false;
      const double d = fabs(g - (double)ref[i]);
      const double r = d / std::max(fabs((double)ref[i]), 1e-3);
      if (d > max_abs) max_abs = d;
      if (r > max_rel) max_rel = r;
    }
  }
  if (!out_path.empty() && !write_file(out_path, outs.data(), outs.size() * 2)) {
    printf("{\"ok\": false, \"failed\": \"writing --out\"}\n");
    return 2;
  }

  // keep stepping until the guard of runtime.js:448 fires
  uint32_t s = STEPS;
  for (;; s++) {
    const int st = submit_step(s);
    if (st != NWD_OK) {
      guard_status = st;
      guard_msg = nwd_last_error();
      break;
    }
    if (seq > MAXSEQ) break;  // cannot happen: the guard must fire at seq == MAXSEQ
  }
  const uint32_t guard_seq = seq;
  need(nwd_stream_synchronize(stream), "sync");

  // reset() (runtime.js:615-633): seq = 0, caches wiped with zeros
  seq = 0;
  std::vector<uint8_t> zeros(MAXSEQ * row * 2, 0);
  need(nwd_memcpy_h2d(kc, zeros.data(), zeros.size(), stream), "wipe k cache");
  need(nwd_memcpy_h2d(vc, zeros.data(), zeros.size(), stream), "wipe v cache");
  need(submit_step(0), "step after reset");
  std::vector<uint16_t> again(qn);
  need(nwd_memcpy_d2h(again.data(), o, qn * 2, stream), "read o");
  const bool reset_same = memcmp(again.data(), outs.data(), qn * 2) == 0;
  // the wiped caches hold exactly the one row written after the reset
  std::vector<uint16_t> kcache(MAXSEQ * row);
  need(nwd_memcpy_d2h(kcache.data(), kc, kcache.size() * 2, stream), "read k cache");
  bool rest_zero = true;
  for (size_t i = row; i < kcache.size(); i++) rest_zero = rest_zero && kcache[i] == 0;

  need(nwd_free(q), "free");
  need(nwd_free(k), "free");
  need(nwd_free(v), "free");
  need(nwd_free(o), "free");
  need(nwd_free(kc), "free");
  need(nwd_free(vc), "free");
  need(nwd_free(ws), "free");
  need(nwd_stream_destroy(stream), "nwd_stream_destroy");
  const bool ok = dev_err == 0 && finite && guard_status == NWD_ERR_RANGE && reset_same &&
                  rest_zero && (expect_path.empty() || (max_abs <= 2e-3 && max_rel <= 1e-2));
  printf("{\"ok\": %s, \"mode\": \"trace\", \"fused\": %s, \"steps\": %u, \"max_abs\": %.6g, "
         "\"max_rel\": %.6g, \"finite\": %s, \"device_error\": %u, \"guard_status\": %s, "
         "\"guard_seq\": %u, \"guard_message\": %s, \"reset_step0_bit_exact\": %s, "
         "\"reset_rows_zero\": %s, \"version\": %s}\n",
         ok ? "true" : "false", fused ? "true" : "false", STEPS, max_abs, max_rel,
         finite ? "true" : "false", dev_err, json_str(nwd_status_name(guard_status)).c_str(),
         guard_seq, json_str(guard_msg).c_str(), reset_same ? "true" : "false",
         rest_zero ? "true" : "false", json_str(nwd_version()).c_str());
  return ok ? 0 : 1;
}

// ------------------------------------------------------------------ mgpu

using Clock = std::chrono::steady_clock;

int run_mgpu(const Args& a) {
  const int world = (int)a.num("--world", 1), rank = (int)a.num("--rank", 0);
  const int device = (int)a.num("--device", rank);
  const uint32_t B = (uint32_t)a.num("--batch", 4), HQ = (uint32_t)a.num("--heads", 32);
  const uint32_t HKV = (uint32_t)a.num("--kv-heads", 8), HD = 128;
  const uint64_t L = (uint64_t)a.num("--rows", 1 << 20);
  const int steps = (int)a.num("--steps", 3), leave_after = (int)a.num("--leave-after", -1);
  const uint32_t init_ms = (uint32_t)a.num("--init-deadline-ms", 120000);
  const uint32_t step_ms = (uint32_t)a.num("--step-deadline-ms", 60000);
  const std::string id_path = a.get("--id-file", ""), out_path = a.get("--out", "");
  if (id_path.empty() || world < 1 || rank < 0 || rank >= world) {
    printf("{\"ok\": false, \"failed\": \"arguments (--world, --rank, --id-file)\"}\n");
    return 2;
  }
  need(nwd_set_device(device), "nwd_set_device");

  // the communicator id: rank 0 creates and publishes it, the others wait
  uint8_t id[NWD_MGPU_ID_BYTES];
  if (rank == 0) {
    need(nwd_mgpu_unique_id(id), "nwd_mgpu_unique_id");
    const std::string tmp = id_path + ".tmp";
    if (!write_file(tmp, id, sizeof(id)) || rename(tmp.c_str(), id_path.c_str()) != 0) {
      printf("{\"ok\": false, \"failed\": \"publishing the id\"}\n");
      return 2;
    }
  } else {
    const Clock::time_point t0 = Clock::now();
    while (!read_file(id_path, id, sizeof(id))) {
      if (Clock::now() - t0 > std::chrono::milliseconds(init_ms)) {
        printf("{\"ok\": false, \"rank\": %d, \"failed\": \"no id file\"}\n", rank);
        return 2;
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(20));
    }
  }
  nwd_mgpu* comm = nullptr;
  need(nwd_mgpu_init(id, world, rank, device, init_ms, step_ms, &comm), "nwd_mgpu_init");
  void* stream = nullptr;
  need(nwd_stream_create(&stream), "nwd_stream_create");

  // this rank's shard of every sequence, contiguous in one pool
  const size_t row = (size_t)HKV * HD;
  std::vector<int64_t> offs(B);
  std::vector<int32_t> lens(B);
  uint64_t pool_rows = 0;
  for (uint32_t b = 0; b < B; b++) {
    const uint64_t lo = L * rank / world, hi = L * (rank + 1) / world;
    offs[b] = (int64_t)pool_rows;
    lens[b] = (int32_t)(hi - lo);
    pool_rows += hi - lo;
  }
  if (pool_rows == 0) pool_rows = 1;
  void *kp, *vp, *q, *o, *d_offs, *d_lens, *ws;
  need(nwd_alloc(pool_rows * row * 2, &kp), "nwd_alloc k pool");
  need(nwd_alloc(pool_rows * row * 2, &vp), "nwd_alloc v pool");
  need(nwd_alloc((size_t)B * HQ * HD * 2, &q), "nwd_alloc");
  need(nwd_alloc((size_t)B * HQ * HD * 2, &o), "nwd_alloc");
  need(nwd_alloc(B * 8, &d_offs), "nwd_alloc");
  need(nwd_alloc(B * 4, &d_lens), "nwd_alloc");
  size_t ws_bytes = 0;
  need(nwd_mgpu_workspace_size(world, B, HQ, HKV, HD, &ws_bytes), "nwd_mgpu_workspace_size");
  need(nwd_alloc(ws_bytes, &ws), "nwd_alloc workspace");
  need(nwd_memcpy_h2d(d_offs, offs.data(), B * 8, stream), "copy offsets");
  need(nwd_memcpy_h2d(d_lens, lens.data(), B * 4, stream), "copy lengths");
  for (uint32_t b = 0; b < B; b++) {
    const uint64_t lo = L * rank / world;
    uint16_t* kdst = (uint16_t*)kp + (size_t)offs[b] * row;
    uint16_t* vdst = (uint16_t*)vp + (size_t)offs[b] * row;
    need(nwd_fill_normal_f16(kdst, (uint64_t)lens[b] * row, 5000, (b * L + lo) * row, stream),
         "fill k");
    need(nwd_fill_normal_f16(vdst, (uint64_t)lens[b] * row, 5001, (b * L + lo) * row, stream),
         "fill v");
  }
  need(nwd_fill_normal_f16((uint16_t*)q, (uint64_t)B * HQ * HD, 5002, 0, stream), "fill q");
  need(nwd_stream_synchronize(stream), "sync");

  auto step = [&]() -> int {
    int st = nwd_mgpu_decode_step(comm, (const uint16_t*)q, (const uint16_t*)kp,
                                  (const uint16_t*)vp, pool_rows, (const int64_t*)d_offs,
                                  (const int32_t*)d_lens, (uint16_t*)o, B, HQ, HKV, HD, 0.0f, ws,
                                  ws_bytes, stream);
    if (st == NWD_OK) st = nwd_mgpu_sync(comm);
    return st;
  };

  int done = 0;
  for (; done < steps; done++) {
    if (leave_after >= 0 && done == leave_after) break;
    need(step(), "sharded step");
  }
  uint32_t dev_err = 0;
  need(nwd_workspace_check(ws, ws_bytes, &dev_err, stream), "nwd_workspace_check");

  if (leave_after >= 0 && done == leave_after) {
    if (rank == world - 1) {
      // the leaving rank: nothing of it is in flight (its last step was
      // synchronised); it drops its communicator locally and exits
      need(nwd_mgpu_abort(comm), "nwd_mgpu_abort");
      printf("{\"ok\": true, \"mode\": \"mgpu\", \"rank\": %d, \"left_after\": %d}\n", rank, done);
      fflush(stdout);
      return 0;
    }
    // the others: the next step must end with an error within the deadline
    const Clock::time_point t0 = Clock::now();
    const int st = step();
    const double el = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    const std::string msg = nwd_last_error();
    nwd_mgpu_destroy(comm);  // the failed wait aborted it: this only frees the handle
    // the context still works: a single-GPU decode over this rank's rows
    size_t ws1_bytes = 0;
    need(nwd_attn_decode_workspace_size(1, HQ, HKV, HD, &ws1_bytes), "workspace_size");
    void* ws1 = nullptr;
    need(nwd_alloc(ws1_bytes, &ws1), "nwd_alloc");
    const int st2 = nwd_attn_decode((const uint16_t*)q, (const uint16_t*)kp, (const uint16_t*)vp,
                                    (uint16_t*)o, HQ, HKV, HD, (uint32_t)lens[0],
                                    (uint32_t)pool_rows, 0.0f, ws1, ws1_bytes, stream);
    uint32_t err2 = 0;
    const int st3 = nwd_workspace_check(ws1, ws1_bytes, &err2, stream);
    const bool ok = st != NWD_OK && el < step_ms + 10000.0 && st2 == NWD_OK && st3 == NWD_OK &&
                    err2 == 0;
    printf("{\"ok\": %s, \"mode\": \"mgpu\", \"rank\": %d, \"steps_done\": %d, "
           "\"failed_step_status\": %s, \"elapsed_ms\": %.1f, \"deadline_ms\": %u, "
           "\"message\": %s, \"after\": %s}\n",
           ok ? "true" : "false", rank, done, json_str(nwd_status_name(st)).c_str(), el, step_ms,
           json_str(msg).c_str(), json_str(nwd_status_name(st2)).c_str());
    fflush(stdout);
    return ok ? 0 : 1;
  }

  std::vector<uint16_t> out((size_t)B * HQ * HD);
  need(nwd_memcpy_d2h(out.data(), o, out.size() * 2, stream), "read o");
  if (rank == 0 && !out_path.empty() && !write_file(out_path, out.data(), out.size() * 2)) {
    printf("{\"ok\": false, \"failed\": \"writing --out\"}\n");
    return 2;
  }
  int nccl_version = 0, mode = 0;
  need(nwd_mgpu_nccl_version(&nccl_version), "nwd_mgpu_nccl_version");
  need(nwd_mgpu_exchange_mode(comm, &mode), "nwd_mgpu_exchange_mode");
  need(nwd_mgpu_destroy(comm), "nwd_mgpu_destroy");
  for (void* p : {kp, vp, q, o, d_offs, d_lens, ws}) need(nwd_free(p), "nwd_free");
  need(nwd_stream_destroy(stream), "nwd_stream_destroy");
  printf("{\"ok\": %s, \"mode\": \"mgpu\", \"rank\": %d, \"world\": %d, \"steps\": %d, "
         "\"device_error\": %u, \"nccl_version\": %d, \"exchange\": \"%s\"}\n",
         dev_err == 0 ? "true" : "false", rank, world, done, dev_err, nccl_version,
         mode == 1 ? "peer" : mode == -1 ? "nccl" : "undecided");
  return dev_err == 0 ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  Args a;
  for (int i = 2; i < argc; i++) a.v.push_back(argv[i]);
  const std::string mode = argc > 1 ? argv[1] : "";
  if (mode == "trace") return run_trace(a);
  if (mode == "mgpu") return run_mgpu(a);
  fprintf(stderr, "usage: nwd_host trace|mgpu [options] (see the header of nwd_host.cc)\n");
  return 2;
}
