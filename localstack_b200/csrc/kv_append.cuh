// kv_append.cuh - fused QK-RMSNorm + NEOX RoPE + f16 scatter of K/V rows into the paged cache.
//
// Replaces attn_block's rms_norm/mul (src/qwen3.cpp:139-140), rope_ext (:143-146) and the two
// set_rows (:150-153). HBM-bound byte work: per token it reads (Hq + 2 Hkv) * 128 inputs and
// writes 2 Hkv * 128 f16 cache values plus Hq * 128 Q values.
//
// Bit-exactness. Every floating-point step uses an explicitly rounded intrinsic so nothing is
// contracted into an FMA, and the RMS sum of squares equals ggml's CPU rms_norm sum (f32
// squares added in double in index order): rows whose partial sums cannot round are summed in
// parallel (any order gives the exact total), every other row sequentially in index order. With
// the same (cos, sin) table the f16 cache bytes equal a CPU evaluation of the ggml op sequence.
//
// Work decomposition. A "row" is one (token, head) vector of 128 values; token t has R = Hq +
// 2 Hkv rows: Hq query heads, Hkv key heads, Hkv value heads. A group is G consecutive rows of
// one token (G a multiple of 4, at most 32 bf16 or 16 f32 rows; the launch picks G so there are
// enough groups for the grid), and a warp takes a grid-stride sequence of groups on a grid sized
// to the resident warps. A group's rows are at most three contiguous pieces of the inputs (its
// Q, K and V rows), copied into shared memory by bulk async copies together with the RoPE row of
// the token's position, completing on one mbarrier; two stage buffers per warp keep the next
// group's copies in flight while the current group is processed. Four rows per step: lanes
// 8s..8s+7 take one row, lane c its NEOX pairs [8c, 8c+8) (elements 8c..8c+7 and 64+8c..64+8c+7)
// as 16-byte vectors; the row's sum of squares is reduced across its eight lanes by shuffles, the
// scale of row r is computed by lane r, and lane c keeps the token's cos / sin of its pairs in
// registers for the whole group.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace lstk {
namespace append {

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kMaxGroupRows = 32;  // bf16 rows; f32 groups hold at most 16
constexpr int kGammaBytes = 2 * kD * 4;
// One stage buffer: the group's rows back to back in the input type, then the RoPE row (64
// (cos, sin) pairs). Rows are 256 or 512 bytes, so every piece starts 16-byte aligned.
__host__ __device__ constexpr int buf_bytes(int group_rows, bool bf16) { return group_rows * kD * (bf16 ? 2 : 4) + kD * 4; }
// A warp's shared memory: two stage buffers, then per row the eight partial sums of squares
// (double) and the eight smallest |x| (32 bits) of its lanes.
__host__ __device__ constexpr int warp_bytes(int group_rows, bool bf16) {
    return 2 * buf_bytes(group_rows, bf16) + group_rows * 8 * (8 + 4);
}
__host__ __device__ constexpr int smem_bytes(int group_rows, bool bf16) {
    return kGammaBytes + kWarps * warp_bytes(group_rows, bf16);
}
constexpr int kSmemBytes = smem_bytes(kMaxGroupRows, true);  // the largest launch

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
    // q8_0 cache (kv_append_kernel<.., .., true>): K / V rows quantised into planes qs int8
    // [n_cells][n_head_kv][128] and d f16 [n_cells][n_head_kv][4] instead of k_cache / v_cache.
    int8_t *k_qs, *v_qs;
    __half *k_d, *v_d;
    int group_rows;        // G: a multiple of 4, at most 32 (bf16) or 16 (f32)
    int groups_per_token;  // ceil(R / G)
    DeviceStatus *status;
};

// Packed f32 pairs (one 64-bit register pair): each lane of mul.rn.f32x2 is an IEEE round-to-
// nearest multiply on its own, the same as the scalar __fmul_rn.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void uf2(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ void uf2u(uint64_t v, uint32_t &lo, uint32_t &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// Two floats as an f16 pair, each rounded to nearest even (lower half = lo).
__device__ __forceinline__ uint32_t f16x2_bits(float lo, float hi) {
    uint32_t h;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(hi), "f"(lo));
    return h;
}


// One contiguous global -> shared copy by the async proxy, completing on `bar` (addresses and
// size multiples of 16 bytes).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// min(|a|, |b|) of each bf16 half (the result's sign bits are not used).
__device__ __forceinline__ uint32_t min_abs_bf16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("min.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// The write loop's 16-byte gamma reads are free of bank conflicts with gamma chunk k stored at
// slot k ^ ((k >> 3) & 1): lane c (of eight per row) reads chunks 2c + q + 16h, which would hit
// the same banks two at a time in the natural order.
__device__ __forceinline__ int gamma_slot(int k) { return k ^ ((k >> 3) & 1); }

// kBf16: bf16 inputs (else f32); kQ16: Q written as f16 (else f32); kQ8: K and V stored as
// q8_0 planes (else f16 rows). Params::in_bf16 and q_out_f16 match the instantiation.
template <bool kBf16, bool kQ16, bool kQ8>
__global__ void __launch_bounds__(kWarps * 32) kv_append_kernel(const Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t s_bar[kWarps][2];    // per warp, per stage buffer
    float *s_gamma = reinterpret_cast<float *>(smem);     // [2][128]: q_gamma, k_gamma (1 when absent)

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
    if (lane == 0) {
        mbar_init(smem_u32(&s_bar[warp][0]), 1);
        mbar_init(smem_u32(&s_bar[warp][1]), 1);
        fence_barrier_init();
    }
    __syncthreads();

    const int R = p.n_head + 2 * p.n_head_kv;
    const int n_qk = p.n_head + p.n_head_kv;
    const int G = p.group_rows, gpt = p.groups_per_token;
    const int n_groups = p.n_tokens * gpt;  // below 2^31 (checked by the launch)
    const int es = kBf16 ? 2 : 4;  // input element bytes
    const int row_bytes = kD * es;
    const int rope_off = G * row_bytes;
    const int bbytes = rope_off + kD * 4;
    uint8_t *bufs = smem + kGammaBytes + warp * warp_bytes(G, kBf16);
    double *part_sum = reinterpret_cast<double *>(bufs + 2 * bbytes);              // [G][8]
    uint32_t *part_min = reinterpret_cast<uint32_t *>(bufs + 2 * bbytes + G * 64);  // [G][8]
    // Groups g = blockIdx.x * kWarps + warp + k * gs, walked as (token, part) without dividing.
    const int gs = gridDim.x * kWarps;
    const int dq = gs / gpt, dr = gs - dq * gpt;
    struct Cursor {
        int g, t, part;
    };
    auto advance = [&](Cursor &k) {
        k.g += gs;
        k.t += dq;
        k.part += dr;
        if (k.part >= gpt) k.part -= gpt, k.t++;
    };
    struct Group {  // token, its first row, rows, the token's position and cell
        int64_t cell;
        int t, j0, nr, pos;
    };
    auto locate = [&](const Cursor &k, Group &m) {
        m.t = 0, m.cell = -1, m.j0 = 0, m.nr = 0, m.pos = -1;
        if (k.g >= n_groups) return;
        m.t = k.t;
        m.j0 = k.part * G;
        m.nr = min(G, R - m.j0);
        m.pos = p.positions[m.t];
        m.cell = p.cells[m.t];
    };
    // Lane 0 issues the group's copies into buffer b: its Q, K and V rows (each a contiguous
    // piece of its input) and the RoPE row of the token's position when the group has Q / K rows
    // and the position is valid; all complete on the buffer's barrier.
    auto issue = [&](const Group &m, int b) {
        if (lane != 0) return;
        const uint32_t bar = smem_u32(&s_bar[warp][b]);
        const uint32_t dst = smem_u32(bufs + b * bbytes);
        const bool rope = m.j0 < n_qk && m.pos >= 0 && m.pos < p.rope_n_pos;
        fence_proxy_async_smem();  // the buffer's last reads (generic proxy) come before the copies
        mbar_arrive_expect_tx(bar, (uint32_t) (m.nr * row_bytes + (rope ? kD * 4 : 0)));
        int j = m.j0;
        const int end = m.j0 + m.nr;
        uint32_t d = dst;
        if (j < p.n_head) {
            const int n = min(end, p.n_head) - j;
            bulk_load(d, (const uint8_t *) p.q_in + ((int64_t) m.t * p.q_stride + (int64_t) j * kD) * es, (uint32_t) (n * row_bytes), bar);
            d += n * row_bytes;
            j += n;
        }
        if (j < end && j < n_qk) {
            const int n = min(end, n_qk) - j;
            bulk_load(d, (const uint8_t *) p.k_in + ((int64_t) m.t * p.k_stride + (int64_t) (j - p.n_head) * kD) * es,
                      (uint32_t) (n * row_bytes), bar);
            d += n * row_bytes;
            j += n;
        }
        if (j < end)
            bulk_load(d, (const uint8_t *) p.v_in + ((int64_t) m.t * p.v_stride + (int64_t) (j - n_qk) * kD) * es,
                      (uint32_t) ((end - j) * row_bytes), bar);
        if (rope) bulk_load(dst + rope_off, p.rope + (int64_t) m.pos * (kD / 2), kD * 4, bar);
    };

    const int sub = lane >> 3, c = lane & 7;
    int goff[4];  // float offsets of this lane's gamma chunks
#pragma unroll
    for (int q = 0; q < 4; q++) goff[q] = gamma_slot(2 * c + (q & 1) + 16 * (q >> 1)) * 4;
    const int sig = kBf16 ? 16 : 24;  // significant bits of a square of an input value

    const int g0 = blockIdx.x * kWarps + warp;
    Cursor ahead = {g0, g0 / gpt, g0 % gpt};  // two groups ahead of the current one, once started
    Group cur, nxt, nxt2;
    locate(ahead, cur);
    advance(ahead);
    locate(ahead, nxt);
    advance(ahead);
    if (g0 < n_groups) issue(cur, 0);
    uint32_t parity = 0;  // bit b: parity of buffer b's next completion
    for (int b = 0, g = g0; g < n_groups; g += gs, b ^= 1) {
        locate(ahead, nxt2);  // used two groups from now
        advance(ahead);
        const bool more = g + gs < n_groups;
        if (more) issue(nxt, b ^ 1);
        if (!mbar_wait_bounded(smem_u32(&s_bar[warp][b]), (parity >> b) & 1u, nullptr)) {
            report(p.status, kStatusTimeout, kSiteAppendWait, g);
            // leave no copy in flight into this CTA's shared memory
            mbar_wait_bounded(smem_u32(&s_bar[warp][b]), (parity >> b) & 1u, nullptr);
            if (more) mbar_wait_bounded(smem_u32(&s_bar[warp][b ^ 1]), (parity >> (b ^ 1)) & 1u, nullptr);
            return;
        }
        parity ^= 1u << b;
        const uint8_t *buf = bufs + b * bbytes;
        const bool pos_ok = cur.pos >= 0 && cur.pos < p.rope_n_pos;
        const bool cell_ok = cur.cell >= 0 && cur.cell < p.n_cells;
        if (lane == 0 && cur.j0 == 0) {  // once per token
            if (!pos_ok) report(p.status, kStatusBadIndex, kSiteAppendPos, cur.t);
            if (!cell_ok) report(p.status, kStatusBadIndex, kSiteAppendCell, cur.t);
        }

        // ggml rms_norm sum of each Q / K row's squares (f32 squares added in double in index
        // order). If no partial sum of a row's squares can round, every order of summation gives
        // the exact total: each of the row's eight lanes sums its 16 squares (four chains) and
        // lane r adds row r's eight partials. With |x| >= 2^e for every element, each square is a multiple of
        // 2^(2e - sig + 1) (sig significant bits: 16 for bf16 inputs, 24 for f32), so a total
        // below 2^(2e + 53 - sig) - one bit of margin, so a rounded total fails too - is exact;
        // e >= -63 keeps every square a normal f32 and the total must stay below 2^128. The squares
        // are added as doubles scaled by 2^-896: the f32 bits shifted into a double's bits (exact
        // for every finite f32, and an f32 inf or NaN lands at or above 2^128 once unscaled). Rows
        // failing the test (zeros, tiny or huge values, inf, NaN, a wide spread of magnitudes) are
        // summed again sequentially by lane r.
#pragma unroll 2
        for (int r0 = 0; r0 < cur.nr; r0 += 4) {
            const int r = r0 + sub;
            const int j = cur.j0 + r;
            const bool norm = r < cur.nr && (j < p.n_head ? p.q_gamma != nullptr : (j < n_qk && p.k_gamma != nullptr));
            double part[4] = {0.0, 0.0, 0.0, 0.0};  // four independent chains
            uint32_t mn = 0x7f7f7f7fu;                 // smallest |x| (bf16 pair or f32 bits)
            if (norm) {
                const uint8_t *row = buf + r * row_bytes;
                if constexpr (kBf16) {
                    const uint4 a = *reinterpret_cast<const uint4 *>(row + c * 16);
                    const uint4 bq = *reinterpret_cast<const uint4 *>(row + 128 + c * 16);
                    const uint32_t w[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
                    uint32_t mn2 = 0x7f7f7f7fu;
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        uint32_t s0, s1;
                        uf2u(mul2(f2(__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xffff0000u)),
                                  f2(__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xffff0000u))), s0, s1);
                        // a normal square of a bf16 value has zero low mantissa bits: the low word is 0
                        part[(2 * e) & 3] = __dadd_rn(part[(2 * e) & 3], __hiloint2double((int) (s0 >> 3), 0));
                        part[(2 * e + 1) & 3] = __dadd_rn(part[(2 * e + 1) & 3], __hiloint2double((int) (s1 >> 3), 0));
                        if (e & 1) mn2 = min_abs_bf16x2(mn2, w[e]);
                        else mn = min_abs_bf16x2(mn, w[e]);
                    }
                    mn = min_abs_bf16x2(mn, mn2);
                } else {
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int q = 0; q < 2; q++) {
                            const float4 v = *reinterpret_cast<const float4 *>(row + (h * 64 + c * 8 + q * 4) * 4);
                            const float vs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                const uint32_t s0 = __float_as_uint(__fmul_rn(vs[e], vs[e]));
                                part[e] = __dadd_rn(part[e], __hiloint2double((int) (s0 >> 3), (int) (s0 << 29)));
                                mn = min(mn, __float_as_uint(vs[e]) & 0x7fffffffu);
                            }
                        }
                }
            }
            // this lane's partial sum and minimum, combined per row by lane r below
            part_sum[r * 8 + c] = __dadd_rn(__dadd_rn(part[0], part[1]), __dadd_rn(part[2], part[3]));
            part_min[r * 8 + c] = mn;
        }
        __syncwarp();

        // Lane r: the scale of row r, 1 / sqrt(mean + eps) with each step rounded as ggml's. The
        // mean is the total / 128, exact or rounded once either way, so a multiply by the power
        // of two equals the divide.
        float my_scale = 1.0f;
        {
            const int j = cur.j0 + lane;
            const bool norm = lane < cur.nr && (j < p.n_head ? p.q_gamma != nullptr : (j < n_qk && p.k_gamma != nullptr));
            if (norm) {
                // the row's eight partials, read in a lane-rotated order (conflict-free 16-byte reads)
                double ps[8];
                uint32_t ms[8];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int q = (k + (lane >> 1)) & 3;
                    const double2 d2 = *reinterpret_cast<const double2 *>(part_sum + lane * 8 + 2 * q);
                    ps[2 * k] = d2.x, ps[2 * k + 1] = d2.y;
                }
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const int q = (k + (lane >> 2)) & 1;
                    const uint4 m4 = *reinterpret_cast<const uint4 *>(part_min + lane * 8 + 4 * q);
                    ms[4 * k] = m4.x, ms[4 * k + 1] = m4.y, ms[4 * k + 2] = m4.z, ms[4 * k + 3] = m4.w;
                }
                const double sum = __dadd_rn(__dadd_rn(__dadd_rn(ps[0], ps[1]), __dadd_rn(ps[2], ps[3])),
                                             __dadd_rn(__dadd_rn(ps[4], ps[5]), __dadd_rn(ps[6], ps[7])));
                int fx;  // biased exponent field of the smallest |x|
                if constexpr (kBf16) {
                    uint32_t m = min_abs_bf16x2(min_abs_bf16x2(min_abs_bf16x2(ms[0], ms[1]), min_abs_bf16x2(ms[2], ms[3])),
                                                min_abs_bf16x2(min_abs_bf16x2(ms[4], ms[5]), min_abs_bf16x2(ms[6], ms[7])));
                    m &= 0x7fff7fffu;
                    fx = (int) (min(m & 0xffffu, m >> 16) >> 7);
                } else {
                    fx = (int) (min(min(min(ms[0], ms[1]), min(ms[2], ms[3])), min(min(ms[4], ms[5]), min(ms[6], ms[7]))) >> 23);
                }
                const int fs = (int) ((uint32_t) __double2hiint(sum) >> 20);  // biased exponent of sum * 2^-896
                // unscaled: fs - 127 = floor(log2(total)); the bound 2^(2e + 53 - sig) with e = fx - 127
                double mean;
                if (fx >= 64 && fs < 255 && fs < 2 * fx - 74 - sig) {
                    mean = __dmul_rn(sum, 0x1p889);  // * 2^896 / 128
                } else {
                    double seq = 0.0;
                    const uint8_t *row = buf + lane * row_bytes;
                    if constexpr (kBf16) {
                        const uint32_t *w = reinterpret_cast<const uint32_t *>(row);
                        for (int i = 0; i < kD / 2; i++) {
                            const float a = __uint_as_float(w[i] << 16), bb = __uint_as_float(w[i] & 0xffff0000u);
                            seq = __dadd_rn(seq, (double) __fmul_rn(a, a));
                            seq = __dadd_rn(seq, (double) __fmul_rn(bb, bb));
                        }
                    } else {
                        const float *f = reinterpret_cast<const float *>(row);
                        for (int i = 0; i < kD; i++) seq = __dadd_rn(seq, (double) __fmul_rn(f[i], f[i]));
                    }
                    mean = __dmul_rn(seq, 1.0 / kD);
                }
                my_scale = __frcp_rn(__fsqrt_rn(__fadd_rn(__double2float_rn(mean), p.eps)));
            }
        }

        // cos / sin of this lane's pairs 8c..8c+7 at the token's position, for the whole group,
        // as packed pairs (C, S of pairs 2k, 2k+1)
        uint64_t Cp[4], Sp[4];
        if (cur.j0 < n_qk && pos_ok) {
            const float4 *cs = reinterpret_cast<const float4 *>(buf + rope_off) + 4 * c;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float4 t = cs[q];
                Cp[q] = f2(t.x, t.z);
                Sp[q] = f2(t.y, t.w);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; q++) Cp[q] = Sp[q] = 0;
        }

        // Write out. Q / K rows: RMSNorm scale and weight, then the rotation, on packed f32 pairs
        // of neighbouring elements (A = (a_e, a_e+1) of the first half, B of the second half):
        //   A' = A * C - B * S,  B' = A * S + B * C   (C, S: cos / sin of pairs e, e+1)
        // every multiply and add rounded on its own, as ggml's CPU rope computes them (the
        // differences and sums are scalar, see below). V rows are converted and stored as read.
        // One loop per kind over the group's rows of that kind; a row is written only when its
        // index is valid: Q needs the position, K the position and the cell, V the cell.
        auto write_rows = [&](auto kind, int lo, int hi, int64_t dst_row0) {
            constexpr int K = decltype(kind)::value;  // 0 Q, 1 K, 2 V
            const bool norm = K == 0 ? p.q_gamma != nullptr : K == 1 ? p.k_gamma != nullptr : false;
            const float *gm = s_gamma + (K == 0 ? 0 : kD);
#pragma unroll 2
            for (int r0 = lo; r0 < hi; r0 += 4) {
                const int r = r0 + sub;
                const float scale = __shfl_sync(0xffffffffu, my_scale, r < hi ? r : lo);
                if (r >= hi) continue;
                float x[16];
                const uint8_t *row = buf + r * row_bytes;
                if constexpr (kBf16) {
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
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int q = 0; q < 2; q++) {
                            const float4 v = *reinterpret_cast<const float4 *>(row + (h * 64 + c * 8 + q * 4) * 4);
                            x[8 * h + 4 * q] = v.x;
                            x[8 * h + 4 * q + 1] = v.y;
                            x[8 * h + 4 * q + 2] = v.z;
                            x[8 * h + 4 * q + 3] = v.w;
                        }
                }
                float o[16];
                if constexpr (K == 2) {
#pragma unroll
                    for (int i = 0; i < 16; i++) o[i] = x[i];
                } else {
                    uint64_t A[4], B[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        A[k] = f2(x[2 * k], x[2 * k + 1]);
                        B[k] = f2(x[8 + 2 * k], x[9 + 2 * k]);
                    }
                    if (norm) {
                        const uint64_t sc = f2(scale, scale);
#pragma unroll
                        for (int q = 0; q < 2; q++) {
                            const float4 ga = *reinterpret_cast<const float4 *>(gm + goff[q]);      // first half
                            const float4 gb = *reinterpret_cast<const float4 *>(gm + goff[2 + q]);  // second half
                            A[2 * q] = mul2(mul2(A[2 * q], sc), f2(ga.x, ga.y));
                            A[2 * q + 1] = mul2(mul2(A[2 * q + 1], sc), f2(ga.z, ga.w));
                            B[2 * q] = mul2(mul2(B[2 * q], sc), f2(gb.x, gb.y));
                            B[2 * q + 1] = mul2(mul2(B[2 * q + 1], sc), f2(gb.z, gb.w));
                        }
                    }
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        // packed products, scalar differences and sums: ptxas contracts a packed
                        // multiply feeding a packed add or subtract into a packed FMA (one rounding
                        // instead of two), even when the product is written as fma(a, b, -0), but
                        // not into a scalar one
                        float ac0, ac1, bs0, bs1, as0, as1, bc0, bc1;
                        uf2(mul2(A[k], Cp[k]), ac0, ac1);
                        uf2(mul2(B[k], Sp[k]), bs0, bs1);
                        uf2(mul2(A[k], Sp[k]), as0, as1);
                        uf2(mul2(B[k], Cp[k]), bc0, bc1);
                        o[2 * k] = __fsub_rn(ac0, bs0);
                        o[2 * k + 1] = __fsub_rn(ac1, bs1);
                        o[8 + 2 * k] = __fadd_rn(as0, bc0);
                        o[9 + 2 * k] = __fadd_rn(as1, bc1);
                    }
                }
                const int64_t at = dst_row0 + r * kD + c * 8;
                if constexpr (K == 0 && !kQ16) {
                    float *d = reinterpret_cast<float *>(p.q_out) + at;
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int q = 0; q < 2; q++)
                            *reinterpret_cast<float4 *>(d + h * 64 + q * 4) =
                                make_float4(o[8 * h + 4 * q], o[8 * h + 4 * q + 1], o[8 * h + 4 * q + 2], o[8 * h + 4 * q + 3]);
                } else if constexpr (K != 0 && kQ8) {
                    // ggml's q8_0 of the row (quantize_row_q8_0, ARM form): per 32 values amax, d =
                    // amax / 127, q = round-to-nearest-even(x * (1 / d)), d kept as f16. Lane c's
                    // first half lies in block c / 4, its second half in block 2 + c / 4; the four
                    // lanes of a block reduce its amax.
                    float amax[2] = {0.f, 0.f};
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        amax[0] = fmaxf(amax[0], fabsf(o[i]));
                        amax[1] = fmaxf(amax[1], fabsf(o[8 + i]));
                    }
#pragma unroll
                    for (int hh = 0; hh < 2; hh++) {
                        amax[hh] = fmaxf(amax[hh], __shfl_xor_sync(0x000000ffu << (8 * sub), amax[hh], 1));
                        amax[hh] = fmaxf(amax[hh], __shfl_xor_sync(0x000000ffu << (8 * sub), amax[hh], 2));
                    }
                    const int64_t row_i = at - c * 8;  // element offset of the row: (cell * Hkv + head) * 128
                    int8_t *qs = (K == 1 ? p.k_qs : p.v_qs) + row_i;
                    __half *dp = (K == 1 ? p.k_d : p.v_d) + row_i / 32;
#pragma unroll
                    for (int hh = 0; hh < 2; hh++) {
                        const float dd = __fdiv_rn(amax[hh], 127.0f);
                        const float id = dd != 0.f ? __frcp_rn(dd) : 0.f;
                        uint32_t w[2];
#pragma unroll
                        for (int k = 0; k < 2; k++) {
                            uint32_t v = 0;
#pragma unroll
                            for (int e = 0; e < 4; e++)
                                v |= (uint32_t) (__float2int_rn(__fmul_rn(o[8 * hh + 4 * k + e], id)) & 0xff) << (8 * e);
                            w[k] = v;
                        }
                        *reinterpret_cast<uint2 *>(qs + hh * 64 + c * 8) = make_uint2(w[0], w[1]);
                        if ((c & 3) == 0) dp[2 * hh + (c >> 2)] = __float2half_rn(dd);
                    }
                } else {
                    __half *d = (K == 0 ? reinterpret_cast<__half *>(p.q_out) : K == 1 ? p.k_cache : p.v_cache) + at;
#pragma unroll
                    for (int h = 0; h < 2; h++)
                        *reinterpret_cast<uint4 *>(d + h * 64) =
                            make_uint4(f16x2_bits(o[8 * h], o[8 * h + 1]), f16x2_bits(o[8 * h + 2], o[8 * h + 3]),
                                       f16x2_bits(o[8 * h + 4], o[8 * h + 5]), f16x2_bits(o[8 * h + 6], o[8 * h + 7]));
                }
            }
        };
        // group rows [0, nq) are Q rows, [nq, nqk) K rows, [nqk, nr) V rows
        const int nq = max(0, min(p.n_head - cur.j0, cur.nr));
        const int nqk = max(0, min(n_qk - cur.j0, cur.nr));
        const int64_t kv_row0 = (cur.cell * p.n_head_kv + cur.j0) * kD;  // + (j - Hq or j - Hq - Hkv) rows
        if (pos_ok) {
            write_rows(std::integral_constant<int, 0>(), 0, nq, ((int64_t) cur.t * p.n_head + cur.j0) * kD);
            if (cell_ok) write_rows(std::integral_constant<int, 1>(), nq, nqk, kv_row0 - (int64_t) p.n_head * kD);
        }
        if (cell_ok) write_rows(std::integral_constant<int, 2>(), nqk, cur.nr, kv_row0 - (int64_t) n_qk * kD);
        __syncwarp();  // buffer b is free for the group two steps ahead
        cur = nxt;
        nxt = nxt2;
    }
}

}  // namespace append
}  // namespace lstk
