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
// heads, Hkv value heads. Each warp takes 32 consecutive rows: it stages them in shared memory
// (coalesced 512-byte row loads, stored with a per-row rotation so that lane r later reads its
// own row without bank conflicts), lane r reduces row r's sum of squares sequentially in double,
// then the warp writes the rows out cooperatively (each lane owns the NEOX pairs (l, l+64) and
// (l+32, l+96) of every row), so global stores stay coalesced.
#pragma once

#include "common.cuh"

namespace lstk {
namespace append {

constexpr int kD = 128;
constexpr int kWarps = 2;  // 2 x 16 KiB of staged rows per CTA
constexpr int kRowsPerWarp = 32;

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

__device__ __forceinline__ void load4(const void *base, int64_t off, int bf16, float v[4]) {
    if (bf16) {
        const uint2 raw = *reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(base) + off);
        v[0] = __uint_as_float(raw.x << 16);
        v[1] = __uint_as_float(raw.x & 0xffff0000u);
        v[2] = __uint_as_float(raw.y << 16);
        v[3] = __uint_as_float(raw.y & 0xffff0000u);
    } else {
        const float4 f = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(base) + off);
        v[0] = f.x;
        v[1] = f.y;
        v[2] = f.z;
        v[3] = f.w;
    }
}

__global__ void __launch_bounds__(kWarps * 32) kv_append_kernel(const Params p) {
    __shared__ float stage[kWarps][kRowsPerWarp * kD];
    __shared__ float row_scale[kWarps][kRowsPerWarp];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int R = p.n_head + 2 * p.n_head_kv;
    const int64_t n_rows = (int64_t) p.n_tokens * R;
    const int64_t n_groups = (n_rows + kRowsPerWarp - 1) / kRowsPerWarp;
    float *srow = stage[warp];

    for (int64_t grp = (int64_t) blockIdx.x * kWarps + warp; grp < n_groups; grp += (int64_t) gridDim.x * kWarps) {
        const int64_t row0 = grp * kRowsPerWarp;
        const int nr = (int) (n_rows - row0 < kRowsPerWarp ? n_rows - row0 : kRowsPerWarp);

        // Stage: row r element i at srow[r*128 + ((i + r) & 127)].
        for (int r = 0; r < nr; r++) {
            const int64_t row = row0 + r;
            const int64_t t = row / R;
            const int j = (int) (row - t * R);
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
            float v[4];
            load4(base, off + lane * 4, p.in_bf16, v);
#pragma unroll
            for (int e = 0; e < 4; e++) srow[r * kD + ((lane * 4 + e + r) & (kD - 1))] = v[e];
        }
        __syncwarp();

        // Lane r: ggml rms_norm scale of row r (Q and K rows only), sequential double sum.
        if (lane < nr) {
            const int64_t row = row0 + lane;
            const int j = (int) (row % R);
            float scale = 1.0f;
            if (j < p.n_head + p.n_head_kv) {
                const float *gamma = j < p.n_head ? p.q_gamma : p.k_gamma;
                if (gamma != nullptr) {
                    double sum = 0.0;
                    for (int i = 0; i < kD; i++) {
                        const float x = srow[lane * kD + ((i + lane) & (kD - 1))];
                        sum = __dadd_rn(sum, (double) __fmul_rn(x, x));
                    }
                    const float mean = __double2float_rn(__ddiv_rn(sum, (double) kD));
                    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
                }
            }
            row_scale[warp][lane] = scale;
        }
        __syncwarp();

        // Write out: lane owns dims l, l+32 (first half of each NEOX pair) and l+64, l+96.
        for (int r = 0; r < nr; r++) {
            const int64_t row = row0 + r;
            const int64_t t = row / R;
            const int j = (int) (row - t * R);
            const float *xr = srow + r * kD;
            auto X = [&](int i) { return xr[(i + r) & (kD - 1)]; };
            const bool is_v = j >= p.n_head + p.n_head_kv;
            int64_t cell = 0;
            if (j >= p.n_head) {
                cell = p.cells[t];
                if (cell < 0 || cell >= p.n_cells) {
                    if (lane == 0 && j == p.n_head) report(p.status, kStatusBadIndex, kSiteAppendCell, (int) t);
                    continue;
                }
            }
            if (is_v) {
                const int h = j - p.n_head - p.n_head_kv;
                __half *dst = p.v_cache + (cell * p.n_head_kv + h) * kD;
#pragma unroll
                for (int e = 0; e < 4; e++) dst[lane + 32 * e] = __float2half_rn(X(lane + 32 * e));
                continue;
            }
            const int32_t pos = p.positions[t];
            if (pos < 0 || pos >= p.rope_n_pos) {
                if (lane == 0 && j == 0) report(p.status, kStatusBadIndex, kSiteAppendPos, (int) t);
                continue;
            }
            const float scale = row_scale[warp][r];
            const bool is_q = j < p.n_head;
            const float *gamma = is_q ? p.q_gamma : p.k_gamma;
            const float2 *cs = p.rope + (int64_t) pos * (kD / 2);
            float out[4];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int i = lane + 32 * e;  // pair (i, i + 64)
                float x0 = X(i);
                float x1 = X(i + 64);
                if (gamma != nullptr) {
                    x0 = __fmul_rn(__fmul_rn(x0, scale), gamma[i]);
                    x1 = __fmul_rn(__fmul_rn(x1, scale), gamma[i + 64]);
                }
                const float2 c = cs[i];
                out[e] = __fsub_rn(__fmul_rn(x0, c.x), __fmul_rn(x1, c.y));
                out[e + 2] = __fadd_rn(__fmul_rn(x0, c.y), __fmul_rn(x1, c.x));
            }
            if (is_q) {
                const int64_t o = (t * p.n_head + j) * kD;
                if (p.q_out_f16) {
                    __half *dst = reinterpret_cast<__half *>(p.q_out) + o;
#pragma unroll
                    for (int e = 0; e < 4; e++) dst[lane + 32 * e] = __float2half_rn(out[e]);
                } else {
                    float *dst = reinterpret_cast<float *>(p.q_out) + o;
#pragma unroll
                    for (int e = 0; e < 4; e++) dst[lane + 32 * e] = out[e];
                }
            } else {
                __half *dst = p.k_cache + (cell * p.n_head_kv + (j - p.n_head)) * kD;
#pragma unroll
                for (int e = 0; e < 4; e++) dst[lane + 32 * e] = __float2half_rn(out[e]);
            }
        }
        __syncwarp();
    }
}

}  // namespace append
}  // namespace lstk
