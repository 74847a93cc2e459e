// lstk_oracle.cpp - CPU restatement of the reference's attention hot path. TEST INFRASTRUCTURE ONLY.
//
// This file is the checker the CUDA path is compared against, and the timed CPU baseline in
// bench.py. Nothing in the product (localstack_b200/) links or calls it.
//
// What it restates. The reference's attention node, attn_block (src/qwen3.cpp:128-171), records
// ggml ops: rms_norm + mul (QK-RMSNorm, :112-114 and :139-140), rope_ext NEOX (:143-146),
// set_rows f32->f16 into the cache (:150-153) and flash_attn_ext with a 0/-inf mask and
// GGML_PREC_F32 (:155-167). Those ops live in ggml, a third-party dependency pulled in through the
// third_party/llama.cpp submodule pinned at 23b0202a189c44a54625aadcb37a946dd1d6278d
// (docs/llama_cpp_commit.txt:1), which is EMPTY in the reference checkout. The functions below
// restate ggml's published CPU algorithms for those ops, in this file's own code:
//   - rms_norm: sum of squares of float products accumulated in double, mean rounded to float,
//     scale = 1/sqrtf(mean + eps), y = x * scale; then mul by the weight as a separate float op.
//   - rope NEOX: per position, theta_0 = pos, theta_{i+1} = theta_i * powf(base, -2/n_dims)
//     (repeated float multiplication), cos/sin from libm cosf/sinf; pairs (i, i + n_dims/2)
//     rotated as x0*c - x1*s, x0*s + x1*c with every float operation rounded separately.
//   - set_rows f32 -> f16 with IEEE round-to-nearest-even.
//   - flash_attn_ext: online softmax over the cells [0, n_kv) in cell order, skipping -inf mask
//     entries. Two precision modes: ORC_MODE_GGML mirrors ggml's CPU kernel (Q rounded to f16
//     before the K dot, the V accumulator kept in f16, expf, S = S*ms + vs); ORC_MODE_EXACT
//     uses f32 Q and double arithmetic throughout.
//
// PARITY UNPINNED: the reference holds no golden vectors or known-answer tests for this path
// and its ggml implementation is absent, so these restatements cannot be checked against the
// reference's own outputs. Only the KV-cache bookkeeping is pinned (the reference's own
// src/kv_cache.cpp compiles here against oracle/ref_shim and is compared in tests/).
//
// Compile with -ffp-contract=off: the bit-exact parts (norm, rope, f16 rounding) must not be
// fused into FMAs.

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

typedef _Float16 f16;

inline uint16_t f32_to_f16_bits(float x) {
    f16 h = (f16) x;
    uint16_t b;
    std::memcpy(&b, &h, 2);
    return b;
}

inline float f16_bits_to_f32(uint16_t b) {
    f16 h;
    std::memcpy(&h, &b, 2);
    return (float) h;
}

inline float bf16_bits_to_f32(uint16_t b) {
    uint32_t u = (uint32_t) b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Runs fn(i) for i in [0, n) on up to n_threads threads (0 = all hardware threads).
template <class F>
void parallel_for(int64_t n, int n_threads, F fn) {
    if (n_threads <= 0) n_threads = (int) std::max(1u, std::thread::hardware_concurrency());
    n_threads = (int) std::min<int64_t>(n_threads, std::max<int64_t>(n, 1));
    if (n_threads <= 1) {
        for (int64_t i = 0; i < n; i++) fn(i);
        return;
    }
    std::atomic<int64_t> next{0};
    std::vector<std::thread> pool;
    for (int t = 0; t < n_threads; t++) {
        pool.emplace_back([&]() {
            for (;;) {
                const int64_t i = next.fetch_add(1);
                if (i >= n) break;
                fn(i);
            }
        });
    }
    for (auto &th : pool) th.join();
}

// ggml rms_norm over one row of ne0 floats followed by the weight multiply (src/qwen3.cpp:112-114).
void rms_norm_mul_row(const float *x, float *y, int64_t ne0, const float *gamma, float eps) {
    double sum = 0.0;
    for (int64_t i = 0; i < ne0; i++) sum += (double) (x[i] * x[i]);
    const float mean = (float) (sum / (double) ne0);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < ne0; i++) {
        const float v = x[i] * scale;
        y[i] = gamma ? v * gamma[i] : v;
    }
}

// ggml's per-position rope cache for the configuration attn_block uses: freq_factors null,
// ext_factor 0 (YaRN ramp inert), attn_factor 1 (src/qwen3.cpp:141-146).
void rope_cache(int64_t pos, int n_dims, float freq_base, float freq_scale, float *cs) {
    const float theta_scale = powf(freq_base, -2.0f / (float) n_dims);
    float theta = (float) pos;
    for (int i = 0; i < n_dims / 2; i++) {
        const float t = freq_scale * theta;
        cs[2 * i + 0] = cosf(t);
        cs[2 * i + 1] = sinf(t);
        theta *= theta_scale;
    }
}

// NEOX rotation of one head row in place: pairs (i, i + n_dims/2).
void rope_neox_row(float *x, int n_dims, const float *cs) {
    const int half = n_dims / 2;
    for (int i = 0; i < half; i++) {
        const float c = cs[2 * i + 0];
        const float s = cs[2 * i + 1];
        const float x0 = x[i];
        const float x1 = x[i + half];
        const float a = x0 * c;
        const float b = x1 * s;
        const float d = x0 * s;
        const float e = x1 * c;
        x[i] = a - b;
        x[i + half] = d + e;
    }
}

}  // namespace

extern "C" {

enum { ORC_MODE_GGML = 0, ORC_MODE_EXACT = 1 };
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2 };

void orc_f32_to_f16(const float *x, uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = f32_to_f16_bits(x[i]);
}

void orc_f16_to_f32(const uint16_t *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = f16_bits_to_f32(x[i]);
}

void orc_rms_norm_mul(const float *x, float *y, int64_t n_rows, int64_t ne0, const float *gamma, float eps) {
    for (int64_t r = 0; r < n_rows; r++) rms_norm_mul_row(x + r * ne0, y + r * ne0, ne0, gamma, eps);
}

void orc_rope_cache(int64_t pos, int n_dims, float freq_base, float freq_scale, float *cs) {
    rope_cache(pos, n_dims, freq_base, freq_scale, cs);
}

// x: [n_tokens][n_heads][head_dim] f32, rotated in place over the first n_dims dims.
void orc_rope_neox(float *x, int64_t n_tokens, int64_t n_heads, int64_t head_dim, const int32_t *pos, int n_dims,
                   float freq_base, float freq_scale) {
    std::vector<float> cs(n_dims);
    for (int64_t t = 0; t < n_tokens; t++) {
        rope_cache(pos[t], n_dims, freq_base, freq_scale, cs.data());
        for (int64_t h = 0; h < n_heads; h++) rope_neox_row(x + (t * n_heads + h) * head_dim, n_dims, cs.data());
    }
}

// ggml_set_rows into an f16 [n_dst_rows][row_elems] matrix: dst[idx[r]] = f16(src row r).
int orc_set_rows_f16(uint16_t *dst, int64_t row_elems, int64_t n_dst_rows, const float *src, int64_t src_row_stride,
                     int64_t n_src_rows, const int64_t *idx) {
    for (int64_t r = 0; r < n_src_rows; r++) {
        if (idx[r] < 0 || idx[r] >= n_dst_rows) return -1;
        uint16_t *d = dst + idx[r] * row_elems;
        const float *s = src + r * src_row_stride;
        for (int64_t i = 0; i < row_elems; i++) d[i] = f32_to_f16_bits(s[i]);
    }
    return 0;
}

// attn_block steps 2-4 (src/qwen3.cpp:139-153): QK-RMSNorm, NEOX RoPE on Q and K, then the K and
// V rows scattered as f16 into the cache at `cells`. Inputs are token-major [T][H][D] rows with
// per-token strides in elements; in_dtype selects f32 or bf16 (bf16 widens exactly to f32).
// A NULL q_gamma / k_gamma means the model has no QK-norm (Qwen2): those rows are only roped.
// Writes the normed+roped Q as f32 to q_out [T][n_head][D]. Returns 0, or -1 on a bad cell.
int orc_kv_append(const void *q_in, const void *k_in, const void *v_in, int in_dtype, int64_t q_stride,
                  int64_t k_stride, int64_t v_stride, int n_tokens, int n_head, int n_head_kv, int head_dim,
                  const int32_t *positions, const int64_t *cells, const float *q_gamma, const float *k_gamma, float eps,
                  float freq_base, float freq_scale, uint16_t *k_cache, uint16_t *v_cache, int64_t n_cells,
                  float *q_out) {
    auto load = [&](const void *base, int64_t off) -> float {
        if (in_dtype == ORC_BF16) return bf16_bits_to_f32(((const uint16_t *) base)[off]);
        return ((const float *) base)[off];
    };
    std::vector<float> row(head_dim), normed(head_dim), cs(head_dim);
    for (int t = 0; t < n_tokens; t++) {
        if (cells[t] < 0 || cells[t] >= n_cells) return -1;
        rope_cache(positions[t], head_dim, freq_base, freq_scale, cs.data());
        for (int h = 0; h < n_head; h++) {
            for (int i = 0; i < head_dim; i++) row[i] = load(q_in, t * q_stride + (int64_t) h * head_dim + i);
            // No weight means no QK-norm node at all (Qwen2, src/qwen3.cpp:139-140).
            if (q_gamma) rms_norm_mul_row(row.data(), normed.data(), head_dim, q_gamma, eps);
            else normed = row;
            rope_neox_row(normed.data(), head_dim, cs.data());
            std::memcpy(q_out + ((int64_t) t * n_head + h) * head_dim, normed.data(), sizeof(float) * head_dim);
        }
        const int64_t row_elems = (int64_t) n_head_kv * head_dim;
        for (int h = 0; h < n_head_kv; h++) {
            for (int i = 0; i < head_dim; i++) row[i] = load(k_in, t * k_stride + (int64_t) h * head_dim + i);
            if (k_gamma) rms_norm_mul_row(row.data(), normed.data(), head_dim, k_gamma, eps);
            else normed = row;
            rope_neox_row(normed.data(), head_dim, cs.data());
            uint16_t *kd = k_cache + cells[t] * row_elems + (int64_t) h * head_dim;
            for (int i = 0; i < head_dim; i++) kd[i] = f32_to_f16_bits(normed[i]);
            uint16_t *vd = v_cache + cells[t] * row_elems + (int64_t) h * head_dim;
            for (int i = 0; i < head_dim; i++) vd[i] = f32_to_f16_bits(load(v_in, t * v_stride + (int64_t) h * head_dim + i));
        }
    }
    return 0;
}

}  // extern "C"

namespace {

// One query row against a sequence of key/value rows given by `key_row(j)` (pointer to the f16
// K row and V row of the j-th visited key), in visiting order. mode selects the precision model.
// Returns the natural-log sum-exp of the scaled scores (exact mode) through *lse.
template <class KeyRow>
void attend_one(const float *q, int head_dim, int64_t n_keys, KeyRow key_row, float scale, int mode, float *out,
                float *lse) {
    if (mode == ORC_MODE_GGML) {
        std::vector<float> qf(head_dim), acc32(head_dim);
        std::vector<f16> acc(head_dim, (f16) 0.0f);
        for (int d = 0; d < head_dim; d++) qf[d] = (float) (f16) q[d];
        float S = 0.0f;
        float M = -INFINITY;
        for (int64_t j = 0; j < n_keys; j++) {
            const uint16_t *kr;
            const uint16_t *vr;
            key_row(j, &kr, &vr);
            double dot = 0.0;
            for (int d = 0; d < head_dim; d++) dot += (double) (f16_bits_to_f32(kr[d]) * qf[d]);
            float s = (float) dot;
            s = s * scale;
            const float Mold = M;
            float ms = 1.0f;
            float vs = 1.0f;
            if (s > M) {
                M = s;
                ms = expf(Mold - M);
                for (int d = 0; d < head_dim; d++) acc[d] = (f16) ((float) acc[d] * ms);
            } else {
                vs = expf(s - M);
            }
            for (int d = 0; d < head_dim; d++) acc[d] = (f16) fmaf(f16_bits_to_f32(vr[d]), vs, (float) acc[d]);
            S = S * ms + vs;
        }
        const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
        for (int d = 0; d < head_dim; d++) out[d] = (float) acc[d] * S_inv;
        if (lse) *lse = (S == 0.0f) ? -INFINITY : (float) ((double) M + std::log((double) S));
        return;
    }
    // Exact: f32 Q, double scores and softmax (two passes), double V accumulation.
    std::vector<double> s(n_keys);
    double m = -INFINITY;
    for (int64_t j = 0; j < n_keys; j++) {
        const uint16_t *kr;
        const uint16_t *vr;
        key_row(j, &kr, &vr);
        double dot = 0.0;
        for (int d = 0; d < head_dim; d++) dot += (double) f16_bits_to_f32(kr[d]) * (double) q[d];
        s[j] = dot * (double) scale;
        m = std::max(m, s[j]);
    }
    std::vector<double> acc(head_dim, 0.0);
    double l = 0.0;
    for (int64_t j = 0; j < n_keys; j++) {
        const uint16_t *kr;
        const uint16_t *vr;
        key_row(j, &kr, &vr);
        const double p = std::exp(s[j] - m);
        l += p;
        for (int d = 0; d < head_dim; d++) acc[d] += p * (double) f16_bits_to_f32(vr[d]);
    }
    for (int d = 0; d < head_dim; d++) out[d] = l > 0.0 ? (float) (acc[d] / l) : 0.0f;
    if (lse) *lse = l > 0.0 ? (float) (m + std::log(l)) : -INFINITY;
}

}  // namespace

extern "C" {

// ggml_flash_attn_ext as attn_block calls it (src/qwen3.cpp:155-167): q [n_tokens][n_head][D] f32,
// caches [n_cells][n_head_kv][D] f16 viewed over cells [0, n_kv), mask [n_tokens][n_kv] f16 with
// 0 / -inf entries (KvCache::fill_mask, src/kv_cache.cpp:140-150), GQA head h -> kv head
// h / (n_head / n_head_kv). out [n_tokens][n_head][D] f32.
void orc_flash_attn_ext(const float *q, int n_tokens, int n_head, const uint16_t *k_cache, const uint16_t *v_cache,
                        int n_head_kv, int head_dim, int64_t n_kv, const uint16_t *mask, float scale, int mode,
                        float *out, int n_threads) {
    const int group = n_head / n_head_kv;
    const int64_t row = (int64_t) n_head_kv * head_dim;
    parallel_for((int64_t) n_tokens * n_head, n_threads, [&](int64_t task) {
        const int i = (int) (task / n_head);
        const int h = (int) (task % n_head);
        const int kvh = h / group;
        std::vector<int64_t> visible;
        visible.reserve(n_kv);
        for (int64_t c = 0; c < n_kv; c++) {
            const float mv = mask ? f16_bits_to_f32(mask[(int64_t) i * n_kv + c]) : 0.0f;
            if (mv != -INFINITY) visible.push_back(c);
        }
        auto key_row = [&](int64_t j, const uint16_t **kr, const uint16_t **vr) {
            const int64_t c = visible[j];
            *kr = k_cache + c * row + (int64_t) kvh * head_dim;
            *vr = v_cache + c * row + (int64_t) kvh * head_dim;
        };
        attend_one(q + ((int64_t) i * n_head + h) * head_dim, head_dim, (int64_t) visible.size(), key_row, scale, mode,
                   out + ((int64_t) i * n_head + h) * head_dim, nullptr);
    });
}

// Page-table attention: the same softmax(scale * q k^T) v, but the keys of query r are the
// positions 0 .. n_keys-1 of its sequence b = q_seq[r], read through the block table
// (cell = block_tables[b][p / block_size] * block_size + p % block_size), in position order.
// n_keys = min(q_pos[r] + 1, kv_lens[b]) when causal, else kv_lens[b]. This is the visibility
// KvCache::fill_mask grants (same sequence, cell_pos <= query pos), without the dense scan.
// q [n_q][n_head][D] f32; out [n_q][n_head][D]; lse_out [n_q][n_head] (natural log) or null.
void orc_paged_attn(const float *q, int n_q, const int32_t *q_seq, const int32_t *q_pos, int n_head,
                    const uint16_t *k_cache, const uint16_t *v_cache, int n_head_kv, int head_dim, int block_size,
                    const int32_t *block_tables, int max_blocks, const int32_t *kv_lens, int causal, float scale,
                    int mode, float *out, float *lse_out, int n_threads) {
    const int group = n_head / n_head_kv;
    const int64_t row = (int64_t) n_head_kv * head_dim;
    parallel_for((int64_t) n_q * n_head, n_threads, [&](int64_t task) {
        const int r = (int) (task / n_head);
        const int h = (int) (task % n_head);
        const int kvh = h / group;
        const int b = q_seq[r];
        int64_t n_keys = kv_lens[b];
        if (causal) n_keys = std::min<int64_t>(n_keys, (int64_t) q_pos[r] + 1);
        if (n_keys < 0) n_keys = 0;
        const int32_t *bt = block_tables + (int64_t) b * max_blocks;
        auto key_row = [&](int64_t p, const uint16_t **kr, const uint16_t **vr) {
            const int64_t c = (int64_t) bt[p / block_size] * block_size + p % block_size;
            *kr = k_cache + c * row + (int64_t) kvh * head_dim;
            *vr = v_cache + c * row + (int64_t) kvh * head_dim;
        };
        attend_one(q + ((int64_t) r * n_head + h) * head_dim, head_dim, n_keys, key_row, scale, mode,
                   out + ((int64_t) r * n_head + h) * head_dim, lse_out ? lse_out + (int64_t) r * n_head + h : nullptr);
    });
}

// Log-sum-exp merge of partial attention results over disjoint key ranges:
// o_parts [n_parts][n_rows][D] (each normalised by its own softmax sum), lse_parts [n_parts][n_rows]
// (natural log). out = sum_r exp(lse_r - M) o_r / sum_r exp(lse_r - M), in double.
void orc_lse_merge(const float *o_parts, const float *lse_parts, int n_parts, int64_t n_rows, int head_dim, float *out,
                   float *lse_out) {
    for (int64_t i = 0; i < n_rows; i++) {
        double M = -INFINITY;
        for (int r = 0; r < n_parts; r++) M = std::max(M, (double) lse_parts[(int64_t) r * n_rows + i]);
        std::vector<double> acc(head_dim, 0.0);
        double den = 0.0;
        if (M != -INFINITY) {
            for (int r = 0; r < n_parts; r++) {
                const double w = std::exp((double) lse_parts[(int64_t) r * n_rows + i] - M);
                den += w;
                const float *o = o_parts + ((int64_t) r * n_rows + i) * head_dim;
                for (int d = 0; d < head_dim; d++) acc[d] += w * (double) o[d];
            }
        }
        for (int d = 0; d < head_dim; d++) out[i * head_dim + d] = den > 0.0 ? (float) (acc[d] / den) : 0.0f;
        if (lse_out) lse_out[i] = den > 0.0 ? (float) (M + std::log(den)) : -INFINITY;
    }
}

// Timed CPU baseline: page-table decode attention in the ggml CPU precision model (Q rounded to
// f16, f32 dot, f16 V accumulator), with the n_head / n_head_kv query heads of a KV head sharing
// one pass over that head's K/V rows. One task per (sequence, kv head); n_threads workers.
void orc_paged_decode_ggml_fast(const float *q, int n_seqs, int n_head, const uint16_t *k_cache, const uint16_t *v_cache,
                                int n_head_kv, int head_dim, int block_size, const int32_t *block_tables,
                                int max_blocks, const int32_t *kv_lens, float scale, float *out, int n_threads) {
    const int group = n_head / n_head_kv;
    const int64_t row = (int64_t) n_head_kv * head_dim;
    parallel_for((int64_t) n_seqs * n_head_kv, n_threads, [&](int64_t task) {
        const int b = (int) (task / n_head_kv);
        const int kvh = (int) (task % n_head_kv);
        const int32_t *bt = block_tables + (int64_t) b * max_blocks;
        std::vector<float> qf((size_t) group * head_dim), kf(head_dim), vf(head_dim), tmp(head_dim);
        std::vector<f16> acc((size_t) group * head_dim, (f16) 0.0f);
        std::vector<float> M(group, -INFINITY), S(group, 0.0f);
        for (int g = 0; g < group; g++)
            for (int d = 0; d < head_dim; d++)
                qf[(size_t) g * head_dim + d] = (float) (f16) q[((int64_t) b * n_head + kvh * group + g) * head_dim + d];
        for (int64_t p = 0; p < kv_lens[b]; p++) {
            const int64_t c = (int64_t) bt[p / block_size] * block_size + p % block_size;
            const f16 *kr = (const f16 *) (k_cache + c * row + (int64_t) kvh * head_dim);
            const f16 *vr = (const f16 *) (v_cache + c * row + (int64_t) kvh * head_dim);
            for (int d = 0; d < head_dim; d++) kf[d] = (float) kr[d];
            for (int d = 0; d < head_dim; d++) vf[d] = (float) vr[d];
            for (int g = 0; g < group; g++) {
                const float *qg = qf.data() + (size_t) g * head_dim;
                float part[16] = {0};
                for (int d = 0; d < head_dim; d += 16)
                    for (int u = 0; u < 16; u++) part[u] = fmaf(kf[d + u], qg[d + u], part[u]);
                float s = 0.0f;
                for (int u = 0; u < 16; u++) s += part[u];
                s = s * scale;
                f16 *ag = acc.data() + (size_t) g * head_dim;
                float ms = 1.0f, vs = 1.0f;
                if (s > M[g]) {
                    ms = expf(M[g] - s);
                    M[g] = s;
                    for (int d = 0; d < head_dim; d++) ag[d] = (f16) ((float) ag[d] * ms);
                } else {
                    vs = expf(s - M[g]);
                }
                for (int d = 0; d < head_dim; d++) ag[d] = (f16) fmaf(vf[d], vs, (float) ag[d]);
                S[g] = S[g] * ms + vs;
            }
        }
        for (int g = 0; g < group; g++) {
            const float inv = S[g] == 0.0f ? 0.0f : 1.0f / S[g];
            float *o = out + ((int64_t) b * n_head + kvh * group + g) * head_dim;
            for (int d = 0; d < head_dim; d++) o[d] = (float) acc[(size_t) g * head_dim + d] * inv;
        }
    });
}

// ---- q8_0 KV cache (the reference's planned option, docs/plan.md:389-395) ----------------------
// Quantisation of ggml's block_q8_0 (ggml-quants quantize_row_q8_0): per 32 consecutive values
// amax = max |x|, d = amax / 127, id = d ? 1 / d : 0, q = round(x * id) as int8 and the f16 of d
// kept as the block's scale. The rounding is to nearest with ties to even, as the ARM NEON form
// (vcvtnq_s32_f32) computes it on the reference's platform (the generic C form rounds ties away
// from zero). The cache keeps ggml's values in two planes: qs int8 [n_cells][n_head_kv][D] and
// d f16 bits [n_cells][n_head_kv][D / 32].
static void quantize_q8_0_row(const float *x, int n, int8_t *qs, uint16_t *d) {
    for (int b = 0; b < n / 32; b++) {
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) amax = std::max(amax, std::fabs(x[b * 32 + j]));
        const float dd = amax / 127.0f;
        const float id = dd != 0.0f ? 1.0f / dd : 0.0f;
        d[b] = f32_to_f16_bits(dd);
        for (int j = 0; j < 32; j++) qs[b * 32 + j] = (int8_t) std::lrintf(x[b * 32 + j] * id);
    }
}

int orc_quantize_q8_0(const float *x, int64_t n_rows, int row_elems, int8_t *qs, uint16_t *d) {
    if (row_elems % 32) return -1;
    for (int64_t r = 0; r < n_rows; r++)
        quantize_q8_0_row(x + r * row_elems, row_elems, qs + r * row_elems, d + r * (row_elems / 32));
    return 0;
}

// orc_kv_append with the K and V rows stored as q8_0 planes instead of f16 rows.
int orc_kv_append_q8(const void *q_in, const void *k_in, const void *v_in, int in_dtype, int64_t q_stride,
                     int64_t k_stride, int64_t v_stride, int n_tokens, int n_head, int n_head_kv, int head_dim,
                     const int32_t *positions, const int64_t *cells, const float *q_gamma, const float *k_gamma,
                     float eps, float freq_base, float freq_scale, int8_t *k_qs, uint16_t *k_d, int8_t *v_qs,
                     uint16_t *v_d, int64_t n_cells, float *q_out) {
    auto load = [&](const void *base, int64_t off) -> float {
        if (in_dtype == ORC_BF16) return bf16_bits_to_f32(((const uint16_t *) base)[off]);
        return ((const float *) base)[off];
    };
    if (head_dim % 32) return -1;
    std::vector<float> row(head_dim), normed(head_dim), cs(head_dim);
    for (int t = 0; t < n_tokens; t++) {
        if (cells[t] < 0 || cells[t] >= n_cells) return -1;
        rope_cache(positions[t], head_dim, freq_base, freq_scale, cs.data());
        for (int h = 0; h < n_head; h++) {
            for (int i = 0; i < head_dim; i++) row[i] = load(q_in, t * q_stride + (int64_t) h * head_dim + i);
            if (q_gamma) rms_norm_mul_row(row.data(), normed.data(), head_dim, q_gamma, eps);
            else normed = row;
            rope_neox_row(normed.data(), head_dim, cs.data());
            std::memcpy(q_out + ((int64_t) t * n_head + h) * head_dim, normed.data(), sizeof(float) * head_dim);
        }
        for (int h = 0; h < n_head_kv; h++) {
            const int64_t r = cells[t] * n_head_kv + h;
            for (int i = 0; i < head_dim; i++) row[i] = load(k_in, t * k_stride + (int64_t) h * head_dim + i);
            if (k_gamma) rms_norm_mul_row(row.data(), normed.data(), head_dim, k_gamma, eps);
            else normed = row;
            rope_neox_row(normed.data(), head_dim, cs.data());
            quantize_q8_0_row(normed.data(), head_dim, k_qs + r * head_dim, k_d + r * (head_dim / 32));
            for (int i = 0; i < head_dim; i++) row[i] = load(v_in, t * v_stride + (int64_t) h * head_dim + i);
            quantize_q8_0_row(row.data(), head_dim, v_qs + r * head_dim, v_d + r * (head_dim / 32));
        }
    }
    return 0;
}

// Page-table attention over a q8_0 cache (orc_paged_attn's visibility and arguments otherwise).
// ORC_MODE_GGML follows ggml's CPU flash_attn_ext for a q8_0 K / V cache: the query row is itself
// quantised to q8_0 (K's vec_dot type), a score is sum over blocks of the block's integer dot
// product times (d_k * d_q) in block order, scaled; softmax online with expf; V rows dequantised
// to f32 (d * q) and accumulated in f32 (the non-f16 V path). ORC_MODE_EXACT: f32 query, the
// dequantised K and V, softmax and accumulation in double.
void orc_paged_attn_q8(const float *q, int n_q, const int32_t *q_seq, const int32_t *q_pos, int n_head,
                       const int8_t *k_qs, const uint16_t *k_d, const int8_t *v_qs, const uint16_t *v_d,
                       int n_head_kv, int head_dim, int block_size, const int32_t *block_tables, int max_blocks,
                       const int32_t *kv_lens, int causal, float scale, int mode, float *out, float *lse_out,
                       int n_threads) {
    const int group = n_head / n_head_kv;
    const int nb = head_dim / 32;
    parallel_for((int64_t) n_q * n_head, n_threads, [&](int64_t task) {
        const int r = (int) (task / n_head);
        const int h = (int) (task % n_head);
        const int kvh = h / group;
        const int b = q_seq[r];
        int64_t n_keys = kv_lens[b];
        if (causal) n_keys = std::min<int64_t>(n_keys, (int64_t) q_pos[r] + 1);
        if (n_keys < 0) n_keys = 0;
        const int32_t *bt = block_tables + (int64_t) b * max_blocks;
        const float *qr = q + ((int64_t) r * n_head + h) * head_dim;
        float *o = out + ((int64_t) r * n_head + h) * head_dim;
        auto cell_row = [&](int64_t p) {
            return ((int64_t) bt[p / block_size] * block_size + p % block_size) * n_head_kv + kvh;
        };
        if (mode == ORC_MODE_GGML) {
            std::vector<int8_t> qq(head_dim);
            std::vector<uint16_t> qd(nb);
            quantize_q8_0_row(qr, head_dim, qq.data(), qd.data());
            std::vector<float> acc(head_dim, 0.0f), v32(head_dim);
            float S = 0.0f, M = -INFINITY;
            for (int64_t p = 0; p < n_keys; p++) {
                const int64_t row = cell_row(p);
                const int8_t *kq = k_qs + row * head_dim;
                const uint16_t *kd = k_d + row * nb;
                float s = 0.0f;
                for (int blk = 0; blk < nb; blk++) {
                    int sumi = 0;
                    for (int j = 0; j < 32; j++) sumi += (int) kq[blk * 32 + j] * (int) qq[blk * 32 + j];
                    s += (float) sumi * (f16_bits_to_f32(kd[blk]) * f16_bits_to_f32(qd[blk]));
                }
                s = s * scale;
                const float Mold = M;
                float ms = 1.0f, vs = 1.0f;
                if (s > M) {
                    M = s;
                    ms = expf(Mold - M);
                    for (int d = 0; d < head_dim; d++) acc[d] *= ms;
                } else {
                    vs = expf(s - M);
                }
                const int8_t *vq = v_qs + row * head_dim;
                const uint16_t *vd = v_d + row * nb;
                for (int d = 0; d < head_dim; d++) v32[d] = f16_bits_to_f32(vd[d / 32]) * (float) vq[d];
                for (int d = 0; d < head_dim; d++) acc[d] = fmaf(v32[d], vs, acc[d]);
                S = S * ms + vs;
            }
            const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
            for (int d = 0; d < head_dim; d++) o[d] = acc[d] * S_inv;
            if (lse_out) lse_out[(int64_t) r * n_head + h] = S == 0.0f ? -INFINITY : (float) ((double) M + std::log((double) S));
            return;
        }
        std::vector<double> s(n_keys);
        double m = -INFINITY;
        for (int64_t p = 0; p < n_keys; p++) {
            const int64_t row = cell_row(p);
            double dot = 0.0;
            for (int d = 0; d < head_dim; d++)
                dot += (double) f16_bits_to_f32(k_d[row * nb + d / 32]) * (double) k_qs[row * head_dim + d] * (double) qr[d];
            s[p] = dot * (double) scale;
            m = std::max(m, s[p]);
        }
        std::vector<double> acc(head_dim, 0.0);
        double l = 0.0;
        for (int64_t p = 0; p < n_keys; p++) {
            const int64_t row = cell_row(p);
            const double w = std::exp(s[p] - m);
            l += w;
            for (int d = 0; d < head_dim; d++)
                acc[d] += w * (double) f16_bits_to_f32(v_d[row * nb + d / 32]) * (double) v_qs[row * head_dim + d];
        }
        for (int d = 0; d < head_dim; d++) o[d] = l > 0.0 ? (float) (acc[d] / l) : 0.0f;
        if (lse_out) lse_out[(int64_t) r * n_head + h] = l > 0.0 ? (float) (m + std::log(l)) : -INFINITY;
    });
}

int orc_hardware_threads(void) { return (int) std::thread::hardware_concurrency(); }

}  // extern "C"
