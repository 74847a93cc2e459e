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
// heads, Hkv value heads. Each warp takes up to 32 consecutive rows (8 or 16 for short appends,
// whose time is one warp's chain of dependent steps; at most 16 with f32 data). The rows, and
// the RoPE rows of the group's first four tokens, are staged into shared memory with 16-byte
// cp.async copies (a bf16 row is 16 chunks, so one warp instruction moves two rows), every copy
// of the group in flight at once and no registers held. Lane r then sums row r's squares
// sequentially in double: independent chains across the lanes, where the sequential order
// leaves no parallelism inside a row; it also prepares row r's kind, destination and RoPE slot.
// The warp writes four rows per step: lanes 8s..8s+7 take one row, lane c its NEOX pairs
// [8c, 8c+8) (elements 8c..8c+7 and 64+8c..64+8c+7), loaded and stored as 16-byte vectors with
// branch-free arithmetic, so the per-row shuffles and address work are shared by four rows.
#pragma once

#include "common.cuh"

namespace lstk {
namespace append {

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kRowsPerWarp = 32;  // at most; the launch picks 8, 16 or 32 (Params::rows_per_warp)
// Staged rows keep the input type and layout, 16 bytes of padding after each (16-byte aligned
// rows for the 16-byte copies): bf16 rows of 68 32-bit words, f32 rows of 132 floats. Lanes
// reading one row in the write phase hit distinct banks, and so do lanes reading their own rows
// 16 bytes at a time for the sum (row starts are 17 or 33 16-byte units apart).
constexpr int kStrideBf16Words = 68;
constexpr int kStrideF32 = 132;
constexpr int kRowBytes = 32 * kStrideBf16Words * 4;  // rows of one group: 32 bf16 rows or 16 f32 rows
static_assert(kRowBytes >= 16 * kStrideF32 * 4, "f32 groups hold at most 16 rows");
constexpr int kCsTokens = 4;                               // RoPE rows staged per group
constexpr int kWarpStageBytes = kRowBytes + kCsTokens * kD * 4;
constexpr int kGammaBytes = 2 * kD * 4;
constexpr int kSmemBytes = kGammaBytes + kWarps * kWarpStageBytes;

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
    int rows_per_warp;  // 8, 16 or 32
    DeviceStatus *status;
};

__device__ __forceinline__ __half2 h2(float a, float b) { return __halves2half2(__float2half_rn(a), __float2half_rn(b)); }

// Input row (t, j) as the 32-bit words lane `lane` needs: bf16 -> w[0] = elements (2l, 2l+1),
// w[1] = (64+2l, 65+2l); f32 -> w[0..3] = elements 2l, 2l+1, 64+2l, 65+2l.
__device__ __forceinline__ const void *row_ptr(const Params &p, int64_t t, int j) {
    if (j < p.n_head) return p.in_bf16 ? (const void *) ((const uint16_t *) p.q_in + t * p.q_stride + (int64_t) j * kD)
                                       : (const void *) ((const float *) p.q_in + t * p.q_stride + (int64_t) j * kD);
    if (j < p.n_head + p.n_head_kv) {
        const int64_t o = t * p.k_stride + (int64_t) (j - p.n_head) * kD;
        return p.in_bf16 ? (const void *) ((const uint16_t *) p.k_in + o) : (const void *) ((const float *) p.k_in + o);
    }
    const int64_t o = t * p.v_stride + (int64_t) (j - p.n_head - p.n_head_kv) * kD;
    return p.in_bf16 ? (const void *) ((const uint16_t *) p.v_in + o) : (const void *) ((const float *) p.v_in + o);
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Shared-memory layouts chosen so that the write loop's 16-byte reads are free of bank conflicts.
// In the write loop lane c (of eight per row) reads gamma chunks 2c + q + 16h (four floats each)
// and the (cos, sin) chunks 4c + q of a RoPE row; eight lanes of a quarter-warp then hit the
// same banks two (gamma) or four (RoPE) at a time in the natural order. Gamma chunk k is stored
// at slot k ^ ((k >> 3) & 1), RoPE chunk 4c + q at 4c + ((q + (c >> 1)) & 3).
__device__ __forceinline__ int gamma_slot(int k) { return k ^ ((k >> 3) & 1); }
__device__ __forceinline__ int rope_slot(int k) { return (k & ~3) | (((k & 3) + ((k >> 3) & 3)) & 3); }

__global__ void __launch_bounds__(kWarps * 32) kv_append_kernel(const Params p) {
    extern __shared__ __align__(16) uint8_t stage_smem[];
    float *s_gamma = reinterpret_cast<float *>(stage_smem);  // [2][128]: q_gamma, k_gamma (1 when absent)

    // Inputs may come from the previous kernel in the stream (programmatic dependent launch);
    // the decode launched after this kernel may be staged right away (it waits for completion).
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kD; i += blockDim.x) {
        const int at = gamma_slot(i >> 2) * 4 + (i & 3);
        s_gamma[at] = p.q_gamma != nullptr ? p.q_gamma[i] : 1.f;
        s_gamma[kD + at] = p.k_gamma != nullptr ? p.k_gamma[i] : 1.f;
    }
    __syncthreads();
    const int R = p.n_head + 2 * p.n_head_kv;
    const int n_qk = p.n_head + p.n_head_kv;
    const int64_t n_rows = (int64_t) p.n_tokens * R;
    const int rpw = p.rows_per_warp;
    const int64_t n_groups = (n_rows + rpw - 1) / rpw;
    uint8_t *stage = stage_smem + kGammaBytes + warp * kWarpStageBytes;
    const uint32_t stage_u32 = smem_u32(stage);
    const uint32_t *sw = reinterpret_cast<const uint32_t *>(stage);  // bf16 pairs
    const float *sf = reinterpret_cast<const float *>(stage);        // f32
    const float *s_cs = reinterpret_cast<const float *>(stage + kRowBytes);  // [kCsTokens][64] (cos, sin)

    for (int64_t grp = (int64_t) blockIdx.x * kWarps + warp; grp < n_groups; grp += (int64_t) gridDim.x * kWarps) {
        const int64_t row0 = grp * rpw;
        const int nr = (int) (n_rows - row0 < rpw ? n_rows - row0 : rpw);
        const int64_t t_first = row0 / R;
        const int j_first = (int) (row0 - t_first * R);

        // Lane r: metadata of row r (token, head slot, position, cell), loaded in parallel.
        int64_t my_t = 0, my_cell = 0;
        int my_j = 0, my_pos = 0;
        if (lane < nr) {
            my_t = (row0 + lane) / R;
            my_j = (int) (row0 + lane - my_t * R);
            my_pos = p.positions[my_t];
            if (my_j >= p.n_head) my_cell = p.cells[my_t];
        }

        // Stage the rows straight into shared memory with 16-byte cp.async copies (every copy of
        // the group in flight at once, no registers held): a bf16 row is 16 chunks, so a warp
        // instruction moves two rows; an f32 row is 32 chunks. (t, j) walk the rows token-major.
        {
            const int cpr = p.in_bf16 ? 16 : 32;  // 16-byte chunks per row
            const int stride_bytes = p.in_bf16 ? kStrideBf16Words * 4 : kStrideF32 * 4;
            const int sub = lane / cpr;            // which row of the instruction's pair (bf16)
            const int chunk = lane % cpr;
            const int step = 32 / cpr;             // rows per instruction
            int64_t t = t_first;
            int j = j_first + sub;
            while (j >= R) {
                j -= R;
                t++;
            }
            for (int k = sub; k < nr; k += step) {
                const uint8_t *src = reinterpret_cast<const uint8_t *>(row_ptr(p, t, j)) + chunk * 16;
                cp_async_16(stage_u32 + (uint32_t) (k * stride_bytes + chunk * 16), src);
                j += step;
                while (j >= R) {
                    j -= R;
                    t++;
                }
            }
        }
        // RoPE rows (64 (cos, sin) pairs, 512 B) of the group's first kCsTokens tokens, staged the
        // same way; the position of token t_first + u comes from the lane holding that token's
        // first row in the group. Rows of a token with a bad position are never read.
#pragma unroll
        for (int u = 0; u < kCsTokens; u++) {
            const int64_t first_row = (t_first + u) * R - row0;
            const int src = (int) (first_row < 0 ? 0 : (first_row > 31 ? 31 : first_row));
            const int pos = __shfl_sync(0xffffffffu, my_pos, src);
            if (first_row < nr && pos >= 0 && pos < p.rope_n_pos)
                cp_async_16(stage_u32 + (uint32_t) (kRowBytes + u * kD * 4 + rope_slot(lane) * 16),
                            p.rope + (int64_t) pos * (kD / 2) + 2 * lane);
        }
        cp_async_wait_all();
        __syncwarp();

        // Lane r: ggml rms_norm scale of row r (Q and K rows with a weight), sequential double sum.
        float my_scale = 1.0f;
        if (lane < nr && my_j < n_qk) {
            const float *gamma = my_j < p.n_head ? p.q_gamma : p.k_gamma;
            if (gamma != nullptr) {
                double sum = 0.0;
                // 16-byte reads (rows start 272 or 528 bytes apart: the eight lanes of a quarter-warp
                // cover all 32 banks), summed in index order.
                if (p.in_bf16) {
                    const uint4 *row = reinterpret_cast<const uint4 *>(sw + lane * kStrideBf16Words);
                    for (int i4 = 0; i4 < kD / 8; i4++) {
                        const uint4 w4 = row[i4];
                        const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const float a = __uint_as_float(ws[e] << 16), b = __uint_as_float(ws[e] & 0xffff0000u);
                            sum = __dadd_rn(sum, (double) __fmul_rn(a, a));
                            sum = __dadd_rn(sum, (double) __fmul_rn(b, b));
                        }
                    }
                } else {
                    const float4 *row = reinterpret_cast<const float4 *>(sf + lane * kStrideF32);
                    for (int i4 = 0; i4 < kD / 4; i4++) {
                        const float4 v4 = row[i4];
                        sum = __dadd_rn(sum, (double) __fmul_rn(v4.x, v4.x));
                        sum = __dadd_rn(sum, (double) __fmul_rn(v4.y, v4.y));
                        sum = __dadd_rn(sum, (double) __fmul_rn(v4.z, v4.z));
                        sum = __dadd_rn(sum, (double) __fmul_rn(v4.w, v4.w));
                    }
                }
                const float mean = __double2float_rn(__ddiv_rn(sum, (double) kD));
                my_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
            }
        }

        // Lane r prepares row r's output: kind (0 Q, 1 K, 2 V, 3 nothing to write: a bad cell or
        // position, reported here), destination, and which prefetched RoPE row it uses.
        int my_kind = 3;
        int64_t my_dst = 0;  // element offset into q_out / k_cache / v_cache
        if (lane < nr) {
            if (my_j >= p.n_head && (my_cell < 0 || my_cell >= p.n_cells)) {
                if (my_j == p.n_head) report(p.status, kStatusBadIndex, kSiteAppendCell, (int) my_t);
            } else if (my_j >= n_qk) {
                my_kind = 2;
                my_dst = (my_cell * p.n_head_kv + (my_j - n_qk)) * kD;
            } else if (my_pos < 0 || my_pos >= p.rope_n_pos) {
                if (my_j == 0) report(p.status, kStatusBadIndex, kSiteAppendPos, (int) my_t);
            } else if (my_j < p.n_head) {
                my_kind = 0;
                my_dst = (my_t * p.n_head + my_j) * kD;
            } else {
                my_kind = 1;
                my_dst = (my_cell * p.n_head_kv + (my_j - p.n_head)) * kD;
            }
        }
        const int my_u = (int) (my_t - t_first);  // RoPE slot (>= 4: loaded in the loop)

        // Write out: lanes 8s..8s+7 take row r0 + s, four rows per warp instruction; lane c = lane & 7
        // owns NEOX pairs [8c, 8c+8) - elements 8c..8c+7 and 64+8c..64+8c+7 - moved as 16-byte
        // vectors. Branch-free arithmetic per element (selects).
        const int sub = lane >> 3, c = lane & 7;
        int goff[4], coff[4];  // float offsets of this lane's gamma chunks and staged RoPE chunks
#pragma unroll
        for (int q = 0; q < 4; q++) {
            goff[q] = gamma_slot(2 * c + (q & 1) + 16 * (q >> 1)) * 4;
            coff[q] = rope_slot(4 * c + q) * 4;
        }
        for (int r0 = 0; r0 < nr; r0 += 4) {
            const int r = r0 + sub;
            const int from = r < nr ? r : r0;
            const int kind = __shfl_sync(0xffffffffu, my_kind, from);
            const int64_t dst = __shfl_sync(0xffffffffu, my_dst, from);
            const float scale = __shfl_sync(0xffffffffu, my_scale, from);
            const int u = __shfl_sync(0xffffffffu, my_u, from);
            const int pos = __shfl_sync(0xffffffffu, my_pos, from);
            if (r >= nr || kind == 3) continue;  // no warp collective below
            float x[16];
            if (p.in_bf16) {
                const uint8_t *row = stage + r * (kStrideBf16Words * 4);
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(row + h * 128 + c * 16);
                    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        x[8 * h + 2 * e] = __uint_as_float(ws[e] << 16);
                        x[8 * h + 2 * e + 1] = __uint_as_float(ws[e] & 0xffff0000u);
                    }
                }
            } else {
                const float *row = sf + r * kStrideF32;
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        const float4 v = *reinterpret_cast<const float4 *>(row + h * 64 + c * 8 + q * 4);
                        x[8 * h + 4 * q] = v.x;
                        x[8 * h + 4 * q + 1] = v.y;
                        x[8 * h + 4 * q + 2] = v.z;
                        x[8 * h + 4 * q + 3] = v.w;
                    }
            }
            const bool is_q = kind == 0, is_v = kind == 2;
            const bool normed = is_q ? p.q_gamma != nullptr : p.k_gamma != nullptr;
            const float *g = s_gamma + (is_q ? 0 : kD);
            // (cos, sin) of pairs 8c..8c+7: staged for the group's first tokens, else from the table
            // (Q / K rows have a checked position; V rows use none of it)
            const bool staged = u < kCsTokens || is_v;
            const float *csr = u < kCsTokens ? s_cs + u * kD
                                             : is_v ? s_cs
                                                    : reinterpret_cast<const float *>(p.rope + (int64_t) pos * (kD / 2));
            // gamma of elements 8c..8c+7 and 64+8c..64+8c+7; (cos, sin) of pairs 8c..8c+7 (pair
            // e: elements e and 64 + e of the lane's slice), as 16-byte reads
            float gm[16], cs[16];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float4 gv = *reinterpret_cast<const float4 *>(g + goff[q]);
                gm[4 * q] = gv.x;
                gm[4 * q + 1] = gv.y;
                gm[4 * q + 2] = gv.z;
                gm[4 * q + 3] = gv.w;
                const float4 cv = *reinterpret_cast<const float4 *>(csr + (staged ? coff[q] : 16 * c + 4 * q));
                cs[4 * q] = cv.x;
                cs[4 * q + 1] = cv.y;
                cs[4 * q + 2] = cv.z;
                cs[4 * q + 3] = cv.w;
            }
            float o[16];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                float a = x[e], b = x[8 + e];
                const float ya = __fmul_rn(__fmul_rn(a, scale), gm[e]);
                const float yb = __fmul_rn(__fmul_rn(b, scale), gm[8 + e]);
                a = normed ? ya : a;
                b = normed ? yb : b;
                const float cx = cs[2 * e], sy = cs[2 * e + 1];
                const float oa = __fsub_rn(__fmul_rn(a, cx), __fmul_rn(b, sy));
                const float ob = __fadd_rn(__fmul_rn(a, sy), __fmul_rn(b, cx));
                o[e] = is_v ? x[e] : oa;  // V rows are stored as read
                o[8 + e] = is_v ? x[8 + e] : ob;
            }
            if (is_q && !p.q_out_f16) {
                float *d = reinterpret_cast<float *>(p.q_out) + dst;
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int q = 0; q < 2; q++)
                        *reinterpret_cast<float4 *>(d + h * 64 + c * 8 + q * 4) =
                            make_float4(o[8 * h + 4 * q], o[8 * h + 4 * q + 1], o[8 * h + 4 * q + 2], o[8 * h + 4 * q + 3]);
            } else {
                __half *d = (is_q ? reinterpret_cast<__half *>(p.q_out) : is_v ? p.v_cache : p.k_cache) + dst;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    uint4 v;
                    uint32_t *vw = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const __half2 hh = h2(o[8 * h + 2 * e], o[8 * h + 2 * e + 1]);
                        vw[e] = *reinterpret_cast<const uint32_t *>(&hh);
                    }
                    *reinterpret_cast<uint4 *>(d + h * 64 + c * 8) = v;
                }
            }
        }
        __syncwarp();
    }
}

}  // namespace append
}  // namespace lstk
