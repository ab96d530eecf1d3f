/*
 * nwd_oracle.c — CPU restatement of the reference decode-attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this code, and
 * only as the checker or the timed CPU baseline; the product never calls it.
 *
 * What it restates (paths inside the reference project):
 *   - kernels/kv_append.wgsl:13-18   -> oracle_kv_append
 *   - kernels/sparse_attn.wgsl:32-113 -> oracle_attn_head_f32 (operation
 *     order kept: per-key dot over d ascending then *scale; 64-lane strided
 *     thread max + shared tree max; exp(s - max) stored in place; strided
 *     thread sums + tree sum; inv_sum = 1/sum; acc += p * inv_sum * V over
 *     t ascending), generalised past the WGSL's 256-key cap
 *     (kernels/sparse_attn.wgsl:29).
 *   - engine/runtime.js:447-467 step sequencing (append row seq, attend
 *     seq + 1 rows) is exercised by the callers in tests/.
 *   - kernels/matmul_nbits_sg.wgsl:32-137 (+ kernels/add.wgsl:15-16) ->
 *     oracle_q4_gemv_f32: the q4 GEMV of the projections either side of
 *     the path (q/k/v before it, o_proj + residual after it).
 *
 * Parity status: UNPINNED.  The reference ships no tests, golden vectors or
 * CPU implementation of this path, and its WGSL needs a WebGPU device
 * (browser + graphics stack) that this machine does not have.  This file is
 * checked against hand-derivable known answers and an independent float64
 * numpy restatement (tests/golden/).
 *
 * Compile with -ffp-contract=off so every f32 multiply and add rounds as
 * the WGSL expressions do.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define WG 64u                                  /* kernels/sparse_attn.wgsl:25 */
static const float NEG_INF = -3.4028234663852886e38f; /* kernels/sparse_attn.wgsl:26 */

/* ---------------- binary16 conversions ---------------- */

float oracle_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do {
                e++;
                man <<= 1;
            } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
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

/* float -> binary16, round to nearest even (IEEE 754). */
uint16_t oracle_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) { /* inf or nan */
        return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (absx < 0x38800000u) { /* below 2^-14: subnormal half (or zero) */
        if (absx < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to 0 */
        uint32_t e = absx >> 23;               /* 102..112 */
        uint32_t m = (absx & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e;             /* 14..24 */
        uint32_t r = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = absx + 0xc8000000u; /* rebias exponent: -112 << 23 */
    uint32_t lsb = (r >> 13) & 1u;
    r += 0xfffu + lsb;
    return (uint16_t)(sign | (r >> 13));
}

void oracle_h2f_array(const uint16_t* src, float* dst, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) dst[i] = oracle_h2f(src[i]);
}

void oracle_f2h_array(const float* src, uint16_t* dst, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) dst[i] = oracle_f2h(src[i]);
}

/* ---------------- deterministic fp16 N(0,1) generator ---------------- */

static inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

/* Element i of stream `seed`: the sum S of twelve 16-bit uniforms taken from
 * three splitmix64 outputs has mean 393210 and standard deviation ~65536, so
 * (S - 393210) / 65536 is an Irwin-Hall(12) approximation of N(0,1).  The
 * integer difference and the power-of-two scale are exact in f32; the final
 * rounding to fp16 is round-to-nearest-even.  The CUDA generator does the
 * same integer steps and produces the same bits. */
uint16_t oracle_normal_f16(uint64_t seed, uint64_t i) {
    uint64_t base = splitmix64(seed) + 3ull * i;
    int64_t s = 0;
    for (int j = 0; j < 3; j++) {
        uint64_t h = splitmix64(base + (uint64_t)j);
        s += (int64_t)(h & 0xffffu) + (int64_t)((h >> 16) & 0xffffu) +
             (int64_t)((h >> 32) & 0xffffu) + (int64_t)(h >> 48);
    }
    float x = (float)(s - 393210) * (1.0f / 65536.0f);
    return oracle_f2h(x);
}

void oracle_fill_normal_f16(uint16_t* dst, uint64_t n, uint64_t seed, uint64_t offset) {
#pragma omp parallel for schedule(static) if (n > (1u << 16))
    for (int64_t i = 0; i < (int64_t)n; i++) dst[i] = oracle_normal_f16(seed, offset + (uint64_t)i);
}

/* ---------------- kv_append ---------------- */

/* kernels/kv_append.wgsl:13-18 */
void oracle_kv_append(const uint16_t* src, uint16_t* cache, uint32_t seq, uint32_t n_kv,
                      uint32_t hd) {
    uint64_t n = (uint64_t)n_kv * hd;
    for (uint64_t i = 0; i < n; i++) cache[(uint64_t)seq * n + i] = src[i];
}

/* ---------------- attention, f32 (the WGSL's arithmetic) ---------------- */

static float default_scale(uint32_t hd, float scale) {
    return scale != 0.0f ? scale : 1.0f / sqrtf((float)hd); /* sparse_attn.wgsl:42 */
}

/* One query head of kernels/sparse_attn.wgsl:32-113.
 *   q: [hd] (fp16 bits); k, v: token-major cache rows with row stride
 *   n_kv*hd starting at row 0; out: [hd] f32.  scores: scratch[seq]. */
static void attn_head_f32(const uint16_t* q, const uint16_t* k, const uint16_t* v, float* out,
                          uint32_t n_kv, uint32_t hkv, uint32_t hd, uint32_t seq, float scale,
                          float* scores) {
    float red[WG];
    /* sparse_attn.wgsl:45-58: scores */
    for (uint32_t t = 0; t < seq; t++) {
        float dot = 0.0f;
        const uint16_t* kr = k + ((uint64_t)t * n_kv + hkv) * hd;
        for (uint32_t d = 0; d < hd; d++) dot = dot + oracle_h2f(q[d]) * oracle_h2f(kr[d]);
        scores[t] = dot * scale;
    }
    /* :61-77 thread max (keys tid, tid+64, ...) then tree max */
    for (uint32_t tid = 0; tid < WG; tid++) {
        float m = NEG_INF;
        for (uint32_t t = tid; t < seq; t += WG) m = fmaxf(m, scores[t]);
        red[tid] = m;
    }
    for (uint32_t stride = WG / 2; stride > 0; stride /= 2)
        for (uint32_t tid = 0; tid < stride; tid++) red[tid] = fmaxf(red[tid], red[tid + stride]);
    float row_max = red[0];
    /* :80-98 exp, strided sums, tree sum */
    for (uint32_t tid = 0; tid < WG; tid++) {
        float s = 0.0f;
        for (uint32_t t = tid; t < seq; t += WG) {
            float p = expf(scores[t] - row_max);
            scores[t] = p;
            s = s + p;
        }
        red[tid] = s;
    }
    for (uint32_t stride = WG / 2; stride > 0; stride /= 2)
        for (uint32_t tid = 0; tid < stride; tid++) red[tid] = red[tid] + red[tid + stride];
    float inv_sum = 1.0f / red[0];
    /* :100-113 P.V, keys ascending, (p * inv_sum) * V */
    for (uint32_t d = 0; d < hd; d++) {
        float acc = 0.0f;
        for (uint32_t t = 0; t < seq; t++) {
            float vv = oracle_h2f(v[((uint64_t)t * n_kv + hkv) * hd + d]);
            acc = acc + scores[t] * inv_sum * vv;
        }
        out[d] = acc;
    }
}

/* Ragged batch: sequence b reads cache rows [row_offset[b], row_offset[b] +
 * seq_len[b]) of the pools; q/out are [batch, n_heads, hd].  With batch = 1,
 * row_offset = {0} and seq_len = {seq} this is exactly one dispatch of the
 * reference kernel.  seq_len[b] == 0 yields zeros, as the WGSL does (its
 * P.V loop never runs).  out is f32; round with oracle_f2h_array. */
void oracle_attn_batched_f32(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                             const int64_t* row_offset, const int32_t* seq_len, float* out,
                             uint32_t batch, uint32_t n_heads, uint32_t n_kv, uint32_t hd,
                             float scale) {
    scale = default_scale(hd, scale);
    uint32_t group = n_heads / n_kv; /* sparse_attn.wgsl:38 */
    int64_t total = (int64_t)batch * n_heads;
#pragma omp parallel
    {
        uint32_t cap = 0;
        float* scores = NULL;
#pragma omp for schedule(dynamic, 1)
        for (int64_t bh = 0; bh < total; bh++) {
            uint32_t b = (uint32_t)(bh / n_heads), h = (uint32_t)(bh % n_heads);
            uint32_t L = seq_len[b] > 0 ? (uint32_t)seq_len[b] : 0u;
            if (L > cap) {
                free(scores);
                cap = L;
                scores = (float*)malloc(sizeof(float) * cap);
            }
            const uint64_t row0 = (uint64_t)row_offset[b] * n_kv * hd;
            attn_head_f32(q + (uint64_t)bh * hd, k_pool + row0, v_pool + row0,
                          out + (uint64_t)bh * hd, n_kv, h / group, hd, L, scale, scores);
        }
        free(scores);
    }
}

/* Single sequence, the reference's own call: Params {n_heads, n_kv_heads,
 * head_dim, seq} over caches starting at row 0. */
void oracle_attn_f32(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                     float* out, uint32_t n_heads, uint32_t n_kv, uint32_t hd, uint32_t seq,
                     float scale) {
    int64_t off = 0;
    int32_t L = (int32_t)seq;
    oracle_attn_batched_f32(q, k_cache, v_cache, &off, &L, out, 1, n_heads, n_kv, hd, scale);
}

/* ---------------- causal prefill ---------------- */

/* The reference has no prefill: it runs the prompt one decode step per token
 * (engine/runtime.js:640-643), so token i of a chunk starting at row
 * start_pos attends rows 0 .. start_pos + i.  This is exactly that: one
 * kernels/sparse_attn.wgsl evaluation per (sequence, token, head).
 *   q, out: [batch, n_q, n_heads, hd]; pools [rows, n_kv, hd];
 *   sequence b's rows start at pool row row_offset[b]. */
void oracle_attn_prefill_f32(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                             const int64_t* row_offset, float* out, uint32_t batch, uint32_t n_q,
                             uint32_t start_pos, uint32_t n_heads, uint32_t n_kv, uint32_t hd,
                             float scale) {
    scale = default_scale(hd, scale);
    uint32_t group = n_heads / n_kv;
    int64_t total = (int64_t)batch * n_q * n_heads;
#pragma omp parallel
    {
        float* scores = (float*)malloc(sizeof(float) * (start_pos + n_q + 1));
#pragma omp for schedule(dynamic, 16)
        for (int64_t idx = 0; idx < total; idx++) {
            uint32_t h = (uint32_t)(idx % n_heads);
            uint32_t i = (uint32_t)((idx / n_heads) % n_q);
            uint32_t b = (uint32_t)(idx / ((int64_t)n_heads * n_q));
            const uint64_t row0 = (uint64_t)row_offset[b] * n_kv * hd;
            attn_head_f32(q + (uint64_t)idx * hd, k_pool + row0, v_pool + row0,
                          out + (uint64_t)idx * hd, n_kv, h / group, hd, start_pos + i + 1, scale,
                          scores);
        }
        free(scores);
    }
}

/* ---------------- attention, f64 (drift check at long L) ---------------- */

void oracle_attn_batched_f64(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                             const int64_t* row_offset, const int32_t* seq_len, double* out,
                             uint32_t batch, uint32_t n_heads, uint32_t n_kv, uint32_t hd,
                             double scale) {
    if (scale == 0.0) scale = 1.0 / sqrt((double)hd);
    uint32_t group = n_heads / n_kv;
    int64_t total = (int64_t)batch * n_heads;
#pragma omp parallel
    {
        uint32_t cap = 0;
        double* sc = NULL;
#pragma omp for schedule(dynamic, 1)
        for (int64_t bh = 0; bh < total; bh++) {
            uint32_t b = (uint32_t)(bh / n_heads), h = (uint32_t)(bh % n_heads);
            uint32_t hkv = h / group;
            uint32_t L = seq_len[b] > 0 ? (uint32_t)seq_len[b] : 0u;
            if (L > cap) {
                free(sc);
                cap = L;
                sc = (double*)malloc(sizeof(double) * cap);
            }
            const uint16_t* qh = q + (uint64_t)bh * hd;
            const uint16_t* kb = k_pool + (uint64_t)row_offset[b] * n_kv * hd;
            const uint16_t* vb = v_pool + (uint64_t)row_offset[b] * n_kv * hd;
            double* o = out + (uint64_t)bh * hd;
            double m = -INFINITY;
            for (uint32_t t = 0; t < L; t++) {
                double dot = 0.0;
                const uint16_t* kr = kb + ((uint64_t)t * n_kv + hkv) * hd;
                for (uint32_t d = 0; d < hd; d++) dot += (double)oracle_h2f(qh[d]) * oracle_h2f(kr[d]);
                sc[t] = dot * scale;
                if (sc[t] > m) m = sc[t];
            }
            double sum = 0.0;
            for (uint32_t t = 0; t < L; t++) {
                sc[t] = exp(sc[t] - m);
                sum += sc[t];
            }
            for (uint32_t d = 0; d < hd; d++) o[d] = 0.0;
            for (uint32_t t = 0; t < L; t++) {
                const uint16_t* vr = vb + ((uint64_t)t * n_kv + hkv) * hd;
                double w = sc[t] / sum;
                for (uint32_t d = 0; d < hd; d++) o[d] += w * oracle_h2f(vr[d]);
            }
        }
        free(sc);
    }
}

/* ---------------- shard partials + log-sum-exp merge ---------------- */

/* Partial of one shard in the library's convention (log2 units):
 *   m = max_t s_t*log2(e), l = sum_t 2^(s_t*log2 e - m), o = sum 2^(..)*V.
 * Computed in f64 and stored as f32. */
void oracle_attn_partial(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                         const int64_t* row_offset, const int32_t* seq_len, float* part_o,
                         float* part_ml, uint32_t batch, uint32_t n_heads, uint32_t n_kv,
                         uint32_t hd, float scale) {
    double sc_ = scale != 0.0f ? (double)scale : 1.0 / sqrt((double)hd);
    const double LOG2E = 1.4426950408889634;
    uint32_t group = n_heads / n_kv;
    int64_t total = (int64_t)batch * n_heads;
#pragma omp parallel
    {
        uint32_t cap = 0;
        double* sc = NULL;
        double* acc = (double*)malloc(sizeof(double) * hd);
#pragma omp for schedule(dynamic, 1)
        for (int64_t bh = 0; bh < total; bh++) {
            uint32_t b = (uint32_t)(bh / n_heads), h = (uint32_t)(bh % n_heads);
            uint32_t hkv = h / group;
            uint32_t L = seq_len[b] > 0 ? (uint32_t)seq_len[b] : 0u;
            if (L > cap) {
                free(sc);
                cap = L;
                sc = (double*)malloc(sizeof(double) * cap);
            }
            const uint16_t* qh = q + (uint64_t)bh * hd;
            const uint16_t* kb = k_pool + (uint64_t)row_offset[b] * n_kv * hd;
            const uint16_t* vb = v_pool + (uint64_t)row_offset[b] * n_kv * hd;
            double m = -INFINITY, l = 0.0;
            for (uint32_t t = 0; t < L; t++) {
                double dot = 0.0;
                const uint16_t* kr = kb + ((uint64_t)t * n_kv + hkv) * hd;
                for (uint32_t d = 0; d < hd; d++) dot += (double)oracle_h2f(qh[d]) * oracle_h2f(kr[d]);
                sc[t] = dot * sc_ * LOG2E;
                if (sc[t] > m) m = sc[t];
            }
            for (uint32_t d = 0; d < hd; d++) acc[d] = 0.0;
            for (uint32_t t = 0; t < L; t++) {
                double w = exp2(sc[t] - m);
                l += w;
                const uint16_t* vr = vb + ((uint64_t)t * n_kv + hkv) * hd;
                for (uint32_t d = 0; d < hd; d++) acc[d] += w * oracle_h2f(vr[d]);
            }
            part_ml[bh * 2 + 0] = L ? (float)m : -INFINITY;
            part_ml[bh * 2 + 1] = (float)l;
            for (uint32_t d = 0; d < hd; d++) part_o[(uint64_t)bh * hd + d] = (float)acc[d];
        }
        free(sc);
        free(acc);
    }
}

/* Merge `shards` partials [shards][rows][...] (rows = batch*n_heads) in
 * shard order: M = max m_r, l = sum l_r 2^(m_r - M), o = sum o_r 2^(m_r - M),
 * out = o / l (0 where l == 0). */
void oracle_attn_merge(const float* part_o, const float* part_ml, float* out, uint32_t shards,
                       uint32_t rows, uint32_t hd) {
    for (uint32_t r = 0; r < rows; r++) {
        double M = -INFINITY;
        for (uint32_t s = 0; s < shards; s++) {
            double m = part_ml[((uint64_t)s * rows + r) * 2];
            if (m > M) M = m;
        }
        double l = 0.0;
        for (uint32_t s = 0; s < shards; s++) {
            const float* ml = part_ml + ((uint64_t)s * rows + r) * 2;
            if (ml[1] > 0.0f) l += ml[1] * exp2((double)ml[0] - M);
        }
        for (uint32_t d = 0; d < hd; d++) {
            double o = 0.0;
            for (uint32_t s = 0; s < shards; s++) {
                const float* ml = part_ml + ((uint64_t)s * rows + r) * 2;
                if (ml[1] > 0.0f) o += part_o[((uint64_t)s * rows + r) * hd + d] * exp2((double)ml[0] - M);
            }
            out[(uint64_t)r * hd + d] = l > 0.0 ? (float)(o / l) : 0.0f;
        }
    }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---------------- q4 GEMV: the projections either side of the path ---------------- */

/* kernels/matmul_nbits_sg.wgsl:32-137, the GEMV the engine runs for an
 * attention layer's q/k/v projections (runtime.js:321-329) and its o_proj
 * (:330, followed by the residual add of kernels/add.wgsl, runtime.js:392-393).
 * Weights of column n: n_blocks blocks of 32 four-bit values, 16 bytes (four
 * u32 words) per block; element j of a word is bits [4j, 4j+4) (a byte holds
 * elements 2b in its low nibble and 2b+1 in its high nibble, :38-41); one f32
 * scale per block ([N][n_blocks]); one 4-bit zero point per block, packed 8 per
 * u32, nibble n*n_blocks + blk, low nibble first (:28-31).  Element value
 * (q - zero) * scale.  The reference sums a block word by word, each word as
 * dot(a0, d0) + dot(a1, d1) (:33-64, dot taken left to right here); thread t of
 * its 256 adds blocks t, t+256, ... in order (:101-128); each subgroup of 32
 * reduces by xor shuffles 1, 2, .., 16 (:66-74: a pairwise tree, lane 0 kept)
 * and the 8 subgroup sums are added in order (:129-135).  epilogue 1 = relu2
 * (:76-79); epilogue 2 = the engine's residual add, Y[n] = Y[n] + result
 * (kernels/add.wgsl:15-16). */
static float q4_word_dot(uint32_t p, float s, float z, const float* a) {
    float d[8];
    for (int j = 0; j < 8; j++) d[j] = ((float)((p >> (4 * j)) & 15u) - z) * s;
    const float d0 = ((a[0] * d[0] + a[1] * d[1]) + a[2] * d[2]) + a[3] * d[3];
    const float d1 = ((a[4] * d[4] + a[5] * d[5]) + a[6] * d[6]) + a[7] * d[7];
    return d0 + d1;
}

static float q4_zero(const uint32_t* zp, uint64_t nib) {
    return (float)((zp[nib / 8u] >> ((nib % 8u) * 4u)) & 15u);
}

void oracle_q4_gemv_f32(const float* A, const uint32_t* B, const float* scales,
                        const uint32_t* zp, float* Y, uint32_t N, uint32_t n_blocks,
                        uint32_t epilogue) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < (int64_t)N; n++) {
        float lane[256];
        for (int t = 0; t < 256; t++) lane[t] = 0.0f;
        for (uint32_t blk = 0; blk < n_blocks; blk++) {
            const uint64_t i = (uint64_t)n * n_blocks + blk;
            float acc = 0.0f;
            for (int w = 0; w < 4; w++)
                acc += q4_word_dot(B[4 * i + w], scales[i], q4_zero(zp, i), A + 32ull * blk + 8 * w);
            lane[blk % 256u] += acc;
        }
        float tot = 0.0f;
        for (int sg = 0; sg < 8; sg++) {
            float v[32];
            memcpy(v, lane + 32 * sg, sizeof v);
            for (int step = 1; step < 32; step <<= 1)
                for (int i = 0; i < 32; i += 2 * step) v[i] = v[i] + v[i + step];
            tot += v[0];
        }
        if (epilogue == 1) {
            const float r = tot > 0.0f ? tot : 0.0f;
            tot = r * r;
        } else if (epilogue == 2) {
            tot = Y[n] + tot;
        }
        Y[n] = tot;
    }
}

/* The same GEMV in float64 (any order), to size the f32 rounding. */
void oracle_q4_gemv_f64(const float* A, const uint32_t* B, const float* scales,
                        const uint32_t* zp, double* Y, uint32_t N, uint32_t n_blocks) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < (int64_t)N; n++) {
        double tot = 0.0;
        for (uint32_t blk = 0; blk < n_blocks; blk++) {
            const uint64_t i = (uint64_t)n * n_blocks + blk;
            const double s = scales[i], z = q4_zero(zp, i);
            for (int j = 0; j < 32; j++) {
                const uint32_t q = (B[4 * i + j / 8] >> (4 * (j % 8))) & 15u;
                tot += (double)A[32ull * blk + j] * (((double)q - z) * s);
            }
        }
        Y[n] = tot;
    }
}

/* Deterministic synthetic q4 weights (not part of the reference): packed words
 * are raw splitmix64 bits (uniform nibbles), zero points likewise, scales
 * 2^-9 + u * 2^-7 with u a 16-bit uniform (exact in f32). */
void oracle_fill_q4(uint32_t* B, float* scales, uint32_t* zp, uint32_t N, uint32_t n_blocks,
                    uint64_t seed) {
    const uint64_t blocks = (uint64_t)N * n_blocks;
    const uint64_t mix = splitmix64(seed);
#pragma omp parallel for schedule(static) if (blocks > 4096)
    for (int64_t i = 0; i < (int64_t)blocks; i++) {
        const uint64_t h0 = splitmix64(mix + 4ull * (uint64_t)i);
        const uint64_t h1 = splitmix64(mix + 4ull * (uint64_t)i + 1);
        const uint64_t h2 = splitmix64(mix + 4ull * (uint64_t)i + 2);
        B[4 * i + 0] = (uint32_t)h0;
        B[4 * i + 1] = (uint32_t)(h0 >> 32);
        B[4 * i + 2] = (uint32_t)h1;
        B[4 * i + 3] = (uint32_t)(h1 >> 32);
        scales[i] = 0.001953125f + (float)(h2 & 0xffffu) * (0.0078125f / 65536.0f);
    }
    const uint64_t words = (blocks + 7) / 8;
#pragma omp parallel for schedule(static) if (words > 4096)
    for (int64_t w = 0; w < (int64_t)words; w++)
        zp[w] = (uint32_t)splitmix64(mix ^ 0x5a5a5a5a5a5a5a5aull ^ (uint64_t)w);
}
