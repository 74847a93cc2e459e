// kv_append.cuh - fused QK-RMSNorm + NEOX RoPE + f16 scatter of K/V rows into the paged cache.
//
// Replaces attn_block's rms_norm/mul (src/qwen3.cpp:139-140), rope_ext (:143-146) and the two
// set_rows (:150-153). HBM-bound byte work: per token it reads (Hq + 2 Hkv) * 128 inputs and
// writes 2 Hkv * 128 f16 cache values plus Hq * 128 Q values.
//
// Bit-exactness. Every floating-point step uses an explicitly rounded intrinsic so nothing is
// contracted into an FMA, and the RMS sum of squares is accumulated in double in index order,
// the order ggml's CPU rms_norm uses. With the same (cos, sin) table the f16 cache bytes equal
// a CPU evaluation of the ggml op sequence.
//
// Work decomposition. A "row" is one (token, head) vector of 128 values; rows are numbered
// token-major: for token t, rows [t*R, t*R + R) with R = Hq + 2*Hkv are Hq query heads, Hkv key
// heads, Hkv value heads. Each warp takes 8 consecutive rows. Lane l owns elements
// {2l, 2l+1, 64+2l, 65+2l} of every row - exactly its two NEOX pairs - so loads and stores are
// 8-byte vectors, coalesced across the warp. The warp's rows are staged into shared memory (row
// stride 129 floats) with all loads issued before any store, so a warp has 16 loads in flight.
// Lane r then sums row r's squares sequentially in double (conflict-free thanks to the padding),
// and the warp writes the rows out, lane r's row metadata broadcast by shuffle. The kernel is
// latency-bound at decode sizes (a few hundred rows), so the group is kept short: the serial
// parts per warp are one round of loads, a 128-term double sum and 8 row writes.
#pragma once

#include "common.cuh"

namespace lstk {
namespace append {

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kRowsPerWarp = 8;
constexpr int kRowStride = kD + 1;  // padded shared-memory row
constexpr int kBatch = 8;           // rows whose loads are in flight together

struct Params {
    const void *q_in;
    const void *k_in;
    const void *v_in;
    int64_t q_stride, k_stride, v_stride;  // elements between consecutive tokens
    int in_bf16;
    int n_tokens, n_head, n_head_kv;
    const int32_t *positions;
    const int64_t *cells;
    const float *q_gamma;
    const float *k_gamma;
    float eps;
    const float2 *rope;  // [rope_n_pos][64] (cos, sin)
    int rope_n_pos;
    __half *k_cache;
    __half *v_cache;
    int64_t n_cells;
    void *q_out;
    int q_out_f16;
    DeviceStatus *status;
};

// Elements (2l, 2l+1) and (64+2l, 65+2l) of one input row.
__device__ __forceinline__ void load_row4(const Params &p, int64_t t, int j, int lane, float v[4]) {
    const void *base;
    int64_t off;
    if (j < p.n_head) {
        base = p.q_in;
        off = t * p.q_stride + (int64_t) j * kD;
    } else if (j < p.n_head + p.n_head_kv) {
        base = p.k_in;
        off = t * p.k_stride + (int64_t) (j - p.n_head) * kD;
    } else {
        base = p.v_in;
        off = t * p.v_stride + (int64_t) (j - p.n_head - p.n_head_kv) * kD;
    }
    off += 2 * lane;
    if (p.in_bf16) {
        const uint16_t *b = reinterpret_cast<const uint16_t *>(base) + off;
        const uint32_t a = *reinterpret_cast<const uint32_t *>(b);
        const uint32_t c = *reinterpret_cast<const uint32_t *>(b + 64);
        v[0] = __uint_as_float(a << 16);
        v[1] = __uint_as_float(a & 0xffff0000u);
        v[2] = __uint_as_float(c << 16);
        v[3] = __uint_as_float(c & 0xffff0000u);
    } else {
        const float *f = reinterpret_cast<const float *>(base) + off;
        const float2 a = *reinterpret_cast<const float2 *>(f);
        const float2 c = *reinterpret_cast<const float2 *>(f + 64);
        v[0] = a.x;
        v[1] = a.y;
        v[2] = c.x;
        v[3] = c.y;
    }
}

__device__ __forceinline__ __half2 h2(float a, float b) { return __halves2half2(__float2half_rn(a), __float2half_rn(b)); }

__global__ void __launch_bounds__(kWarps * 32) kv_append_kernel(const Params p) {
    __shared__ float stage[kWarps][kRowsPerWarp * kRowStride];

    // Inputs may come from the previous kernel in the stream (programmatic dependent launch);
    // the decode launched after this kernel may be staged right away (it waits for completion).
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int R = p.n_head + 2 * p.n_head_kv;
    const int n_qk = p.n_head + p.n_head_kv;
    const int64_t n_rows = (int64_t) p.n_tokens * R;
    const int64_t n_groups = (n_rows + kRowsPerWarp - 1) / kRowsPerWarp;
    float *srow = stage[warp];

    // This lane's weight elements (2l, 2l+1, 64+2l, 65+2l) for Q and K rows.
    float qg[4] = {1.f, 1.f, 1.f, 1.f}, kg[4] = {1.f, 1.f, 1.f, 1.f};
    if (p.q_gamma != nullptr) {
        qg[0] = p.q_gamma[2 * lane];
        qg[1] = p.q_gamma[2 * lane + 1];
        qg[2] = p.q_gamma[64 + 2 * lane];
        qg[3] = p.q_gamma[65 + 2 * lane];
    }
    if (p.k_gamma != nullptr) {
        kg[0] = p.k_gamma[2 * lane];
        kg[1] = p.k_gamma[2 * lane + 1];
        kg[2] = p.k_gamma[64 + 2 * lane];
        kg[3] = p.k_gamma[65 + 2 * lane];
    }

    for (int64_t grp = (int64_t) blockIdx.x * kWarps + warp; grp < n_groups; grp += (int64_t) gridDim.x * kWarps) {
        const int64_t row0 = grp * kRowsPerWarp;
        const int nr = (int) (n_rows - row0 < kRowsPerWarp ? n_rows - row0 : kRowsPerWarp);

        // Lane r: metadata of row r (token, head slot, position, cell), loaded in parallel.
        int64_t my_t = 0, my_cell = 0;
        int my_j = 0, my_pos = 0;
        if (lane < nr) {
            my_t = (row0 + lane) / R;
            my_j = (int) (row0 + lane - my_t * R);
            if (my_j < n_qk) my_pos = p.positions[my_t];
            if (my_j >= p.n_head) my_cell = p.cells[my_t];
        }

        // RoPE rows of the group's first two tokens, loaded while the rows are staged (a group of
        // 8 rows spans at most two tokens whenever a token has 8 or more rows, as every Qwen3
        // shape does; rows of any further token load theirs in the write loop).
        const int64_t t_first = row0 / R;
        float4 cs_pre[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
#pragma unroll
        for (int u = 0; u < 2; u++) {
            if (t_first + u < p.n_tokens) {
                const int pos = p.positions[t_first + u];
                if (pos >= 0 && pos < p.rope_n_pos)
                    cs_pre[u] = *reinterpret_cast<const float4 *>(p.rope + (int64_t) pos * (kD / 2) + 2 * lane);
            }
        }

        // Stage rows, kBatch at a time: all loads of a batch issued before its stores.
        for (int r0 = 0; r0 < nr; r0 += kBatch) {
            float v[kBatch][4];
#pragma unroll
            for (int k = 0; k < kBatch; k++) {
                const int64_t t = __shfl_sync(0xffffffffu, my_t, (r0 + k) & 31);
                const int j = __shfl_sync(0xffffffffu, my_j, (r0 + k) & 31);
                if (r0 + k < nr) load_row4(p, t, j, lane, v[k]);
            }
#pragma unroll
            for (int k = 0; k < kBatch; k++) {
                if (r0 + k < nr) {
                    float *row = srow + (r0 + k) * kRowStride;
                    row[2 * lane] = v[k][0];
                    row[2 * lane + 1] = v[k][1];
                    row[64 + 2 * lane] = v[k][2];
                    row[65 + 2 * lane] = v[k][3];
                }
            }
        }
        __syncwarp();

        // Lane r: ggml rms_norm scale of row r (Q and K rows with a weight), sequential double sum.
        float my_scale = 1.0f;
        if (lane < nr && my_j < n_qk) {
            const float *gamma = my_j < p.n_head ? p.q_gamma : p.k_gamma;
            if (gamma != nullptr) {
                const float *row = srow + lane * kRowStride;
                double sum = 0.0;
                for (int i = 0; i < kD; i++) sum = __dadd_rn(sum, (double) __fmul_rn(row[i], row[i]));
                const float mean = __double2float_rn(__ddiv_rn(sum, (double) kD));
                my_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
            }
        }

        // Write out row by row; lane l produces its two NEOX pairs (2l, 64+2l), (2l+1, 65+2l).
#pragma unroll 4
        for (int r = 0; r < nr; r++) {
            const int64_t t = __shfl_sync(0xffffffffu, my_t, r);
            const int j = __shfl_sync(0xffffffffu, my_j, r);
            const int pos = __shfl_sync(0xffffffffu, my_pos, r);
            const int64_t cell = __shfl_sync(0xffffffffu, my_cell, r);
            const float scale = __shfl_sync(0xffffffffu, my_scale, r);
            const float *row = srow + r * kRowStride;
            float x[4] = {row[2 * lane], row[2 * lane + 1], row[64 + 2 * lane], row[65 + 2 * lane]};
            if (j >= p.n_head && (cell < 0 || cell >= p.n_cells)) {
                if (lane == 0 && j == p.n_head) report(p.status, kStatusBadIndex, kSiteAppendCell, (int) t);
                continue;
            }
            if (j >= n_qk) {  // V row: f16 only
                __half *dst = p.v_cache + (cell * p.n_head_kv + (j - n_qk)) * kD;
                *reinterpret_cast<__half2 *>(dst + 2 * lane) = h2(x[0], x[1]);
                *reinterpret_cast<__half2 *>(dst + 64 + 2 * lane) = h2(x[2], x[3]);
                continue;
            }
            if (pos < 0 || pos >= p.rope_n_pos) {
                if (lane == 0 && j == 0) report(p.status, kStatusBadIndex, kSiteAppendPos, (int) t);
                continue;
            }
            const bool is_q = j < p.n_head;
            const float *gamma = is_q ? p.q_gamma : p.k_gamma;
            if (gamma != nullptr) {
#pragma unroll
                for (int e = 0; e < 4; e++) x[e] = __fmul_rn(__fmul_rn(x[e], scale), is_q ? qg[e] : kg[e]);
            }
            const float4 cs = t == t_first       ? cs_pre[0]
                              : t == t_first + 1 ? cs_pre[1]
                                                 : *reinterpret_cast<const float4 *>(p.rope + (int64_t) pos * (kD / 2) + 2 * lane);
            // pair (2l, 64+2l) uses (cs.x, cs.y); pair (2l+1, 65+2l) uses (cs.z, cs.w)
            float o[4];
            o[0] = __fsub_rn(__fmul_rn(x[0], cs.x), __fmul_rn(x[2], cs.y));
            o[2] = __fadd_rn(__fmul_rn(x[0], cs.y), __fmul_rn(x[2], cs.x));
            o[1] = __fsub_rn(__fmul_rn(x[1], cs.z), __fmul_rn(x[3], cs.w));
            o[3] = __fadd_rn(__fmul_rn(x[1], cs.w), __fmul_rn(x[3], cs.z));
            if (is_q) {
                const int64_t off = (t * p.n_head + j) * kD;
                if (p.q_out_f16) {
                    __half *dst = reinterpret_cast<__half *>(p.q_out) + off;
                    *reinterpret_cast<__half2 *>(dst + 2 * lane) = h2(o[0], o[1]);
                    *reinterpret_cast<__half2 *>(dst + 64 + 2 * lane) = h2(o[2], o[3]);
                } else {
                    float *dst = reinterpret_cast<float *>(p.q_out) + off;
                    *reinterpret_cast<float2 *>(dst + 2 * lane) = make_float2(o[0], o[1]);
                    *reinterpret_cast<float2 *>(dst + 64 + 2 * lane) = make_float2(o[2], o[3]);
                }
            } else {
                __half *dst = p.k_cache + (cell * p.n_head_kv + (j - p.n_head)) * kD;
                *reinterpret_cast<__half2 *>(dst + 2 * lane) = h2(o[0], o[1]);
                *reinterpret_cast<__half2 *>(dst + 64 + 2 * lane) = h2(o[2], o[3]);
            }
        }
        __syncwarp();
    }
}

}  // namespace append
}  // namespace lstk
