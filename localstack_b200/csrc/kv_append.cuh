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
// whose time is one warp's chain of dependent steps). Lane l owns elements
// {2l, 2l+1, 64+2l, 65+2l} of every row - exactly its two NEOX pairs - so stores are coalesced
// across the warp. The rows are staged into shared memory with 16-byte cp.async copies (a bf16
// row is 16 chunks, so one warp instruction moves two rows), every copy of the group in flight
// at once and no registers held, keeping the input type. Lane r then sums row r's squares
// sequentially in double: independent chains across the lanes, where the sequential order
// leaves no parallelism inside a row. Lane r also prepares row r's kind, destination and RoPE
// slot, so the warp's write loop over the rows is shuffles and branch-free arithmetic; the RoPE
// rows of the group's first four tokens are loaded up front.
#pragma once

#include "common.cuh"

namespace lstk {
namespace append {

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kRowsPerWarp = 32;  // at most; the launch picks 8, 16 or 32 (Params::rows_per_warp)
// Staged rows keep the input type and layout, 16 bytes of padding after each (16-byte aligned
// rows for the 16-byte copies): bf16 rows of 68 32-bit words, f32 rows of 132 floats. Lanes
// reading one row in the write phase hit distinct banks; lane r reading its own row r word by
// word (the sum) has 4-way conflicts, small next to the sum's dependent double adds.
constexpr int kStrideBf16Words = 68;
constexpr int kStrideF32 = 132;
constexpr int kWarpStageBytes = kRowsPerWarp * kStrideF32 * 4;
constexpr int kSmemBytes = kWarps * kWarpStageBytes;

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

__global__ void __launch_bounds__(kWarps * 32) kv_append_kernel(const Params p) {
    extern __shared__ float stage_smem[];

    // Inputs may come from the previous kernel in the stream (programmatic dependent launch);
    // the decode launched after this kernel may be staged right away (it waits for completion).
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int R = p.n_head + 2 * p.n_head_kv;
    const int n_qk = p.n_head + p.n_head_kv;
    const int64_t n_rows = (int64_t) p.n_tokens * R;
    const int rpw = p.rows_per_warp;
    const int64_t n_groups = (n_rows + rpw - 1) / rpw;
    uint8_t *stage = reinterpret_cast<uint8_t *>(stage_smem) + warp * kWarpStageBytes;
    const uint32_t stage_u32 = smem_u32(stage);
    const uint32_t *sw = reinterpret_cast<const uint32_t *>(stage);  // bf16 pairs
    const float *sf = reinterpret_cast<const float *>(stage);        // f32

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
            cp_async_wait_all();
        }

        // RoPE rows (cos, sin) of the group's first four tokens; the position of token t_first + u
        // comes from the lane holding that token's first row in the group.
        float4 cs_pre[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int64_t first_row = (t_first + u) * R - row0;
            const int src = (int) (first_row < 0 ? 0 : (first_row > 31 ? 31 : first_row));
            const int pos = __shfl_sync(0xffffffffu, my_pos, src);
            cs_pre[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (first_row < nr && pos >= 0 && pos < p.rope_n_pos)
                cs_pre[u] = *reinterpret_cast<const float4 *>(p.rope + (int64_t) pos * (kD / 2) + 2 * lane);
        }
        __syncwarp();

        // Lane r: ggml rms_norm scale of row r (Q and K rows with a weight), sequential double sum.
        float my_scale = 1.0f;
        if (lane < nr && my_j < n_qk) {
            const float *gamma = my_j < p.n_head ? p.q_gamma : p.k_gamma;
            if (gamma != nullptr) {
                double sum = 0.0;
                if (p.in_bf16) {
                    const uint32_t *row = sw + lane * kStrideBf16Words;
                    for (int i = 0; i < kD / 2; i++) {
                        const uint32_t w = row[i];
                        const float a = __uint_as_float(w << 16), b = __uint_as_float(w & 0xffff0000u);
                        sum = __dadd_rn(sum, (double) __fmul_rn(a, a));
                        sum = __dadd_rn(sum, (double) __fmul_rn(b, b));
                    }
                } else {
                    const float *row = sf + lane * kStrideF32;
                    for (int i = 0; i < kD; i++) sum = __dadd_rn(sum, (double) __fmul_rn(row[i], row[i]));
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

        // Write out row by row; lane l produces its two NEOX pairs (2l, 64+2l), (2l+1, 65+2l).
        // Branch-free arithmetic per row (selects), so unrolled rows overlap.
#pragma unroll 4
        for (int r = 0; r < nr; r++) {
            const int kind = __shfl_sync(0xffffffffu, my_kind, r);
            const int64_t dst = __shfl_sync(0xffffffffu, my_dst, r);
            const float scale = __shfl_sync(0xffffffffu, my_scale, r);
            const int u = __shfl_sync(0xffffffffu, my_u, r);
            float x[4];
            if (p.in_bf16) {
                const uint32_t w0 = sw[r * kStrideBf16Words + lane], w1 = sw[r * kStrideBf16Words + 32 + lane];
                x[0] = __uint_as_float(w0 << 16);
                x[1] = __uint_as_float(w0 & 0xffff0000u);
                x[2] = __uint_as_float(w1 << 16);
                x[3] = __uint_as_float(w1 & 0xffff0000u);
            } else {
                const float2 a = *reinterpret_cast<const float2 *>(sf + r * kStrideF32 + 2 * lane);
                const float2 b = *reinterpret_cast<const float2 *>(sf + r * kStrideF32 + 64 + 2 * lane);
                x[0] = a.x;
                x[1] = a.y;
                x[2] = b.x;
                x[3] = b.y;
            }
            if (kind == 3) continue;
            const bool is_q = kind == 0;
            const bool normed = is_q ? p.q_gamma != nullptr : p.k_gamma != nullptr;
            float y[4];
#pragma unroll
            for (int e = 0; e < 4; e++) y[e] = __fmul_rn(__fmul_rn(x[e], scale), is_q ? qg[e] : kg[e]);
            float4 cs = u == 0 ? cs_pre[0] : u == 1 ? cs_pre[1] : u == 2 ? cs_pre[2] : cs_pre[3];
            if (u >= 4 && kind != 2) {  // Q / K rows have a checked position; V rows need none
                const int pos = __shfl_sync(0xffffffffu, my_pos, r);
                cs = *reinterpret_cast<const float4 *>(p.rope + (int64_t) pos * (kD / 2) + 2 * lane);
            }
            float w[4];
#pragma unroll
            for (int e = 0; e < 4; e++) w[e] = normed ? y[e] : x[e];
            // pair (2l, 64+2l) uses (cs.x, cs.y); pair (2l+1, 65+2l) uses (cs.z, cs.w)
            float o[4];
            o[0] = __fsub_rn(__fmul_rn(w[0], cs.x), __fmul_rn(w[2], cs.y));
            o[2] = __fadd_rn(__fmul_rn(w[0], cs.y), __fmul_rn(w[2], cs.x));
            o[1] = __fsub_rn(__fmul_rn(w[1], cs.z), __fmul_rn(w[3], cs.w));
            o[3] = __fadd_rn(__fmul_rn(w[1], cs.w), __fmul_rn(w[3], cs.z));
            const bool is_v = kind == 2;
#pragma unroll
            for (int e = 0; e < 4; e++) o[e] = is_v ? x[e] : o[e];  // V rows are stored as read
            if (is_q && !p.q_out_f16) {
                float *d = reinterpret_cast<float *>(p.q_out) + dst;
                *reinterpret_cast<float2 *>(d + 2 * lane) = make_float2(o[0], o[1]);
                *reinterpret_cast<float2 *>(d + 64 + 2 * lane) = make_float2(o[2], o[3]);
            } else {
                __half *d = (is_q ? reinterpret_cast<__half *>(p.q_out) : is_v ? p.v_cache : p.k_cache) + dst;
                *reinterpret_cast<__half2 *>(d + 2 * lane) = h2(o[0], o[1]);
                *reinterpret_cast<__half2 *>(d + 64 + 2 * lane) = h2(o[2], o[3]);
            }
        }
        __syncwarp();
    }
}

}  // namespace append
}  // namespace lstk
