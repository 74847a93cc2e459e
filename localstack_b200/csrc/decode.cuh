// decode.cuh - paged split-K flash-decoding (one new token per sequence) and the LSE combine.
//
// Replaces flash_attn_ext for the decode step (src/qwen3.cpp:155-167, n_tokens = 1). HBM-bound:
// per sequence it must stream len * n_head_kv * 128 * 2 bytes of K plus the same of V once.
//
// Data layout. K and V caches keep the reference layout [n_cells][n_head_kv][128] f16. A page
// is 32 consecutive cells; one KV head's share of a page is 32 rows of 256 bytes at a stride of
// n_head_kv * 256 bytes. A TMA tensor map over (d, head, cell) with box (64, 1, 32) and 128-byte
// swizzle loads half of one head's page (32 rows x 128 bytes) per instruction.
//
// Work decomposition (split-K over "page-groups"). A segment is (sequence b, head group hg) where
// a head group is up to 4 KV heads; it has ceil(len_b / 32) page-groups, each = one page of those
// 4 heads' K and V (64 KiB, read contiguously from HBM). All segments are concatenated into one
// index space of P page-groups and cut into gridDim.x equal contiguous ranges, one per CTA, so
// every CTA streams the same number of bytes whatever the mix of context lengths. Where a range
// boundary falls inside a segment, the pieces on either side are merged later by log-sum-exp
// (decode_combine_kernel); a segment inside one CTA is written out directly.
//
// CTA roles. Warp 4 (one lane) issues TMA loads into a 3-stage ring of 64 KiB stages; warps 0..3
// each own one KV head of the group and run the attention for it with mma.sync m16n8k16
// (f16 x f16 -> f32): S^T[16 tokens x 8 q-heads] = K[16 x 128] . Q^T, online softmax down the
// token axis, P^T re-packed in registers with movmatrix, then O^T[128 x 8] += V^T . P^T. The
// 8-wide N side holds the GQA group (n_head / n_head_kv <= 8 query heads share one K/V head), so
// every K/V byte brought in is used by all its query heads. The tensor cores only matter here
// because they take the FLOPs off the issue slots; the kernel is bound by HBM bytes.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "exchange.cuh"

namespace lstk {
namespace decode {

constexpr int kD = 128;
constexpr int kPage = 32;
constexpr int kHeadsPerGroup = 4;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 3;
constexpr int kSubTile = kPage * 128;                                // 4 KiB: 32 rows x 128 B
constexpr int kHeadPage = 2 * kSubTile;                              // 8 KiB: one head's K page
constexpr int kStageBytes = 2 * kHeadsPerGroup * kHeadPage;          // 64 KiB: K and V, 4 heads
constexpr int kMaxCtas = 512;
constexpr int kMaxGroup = 8;
constexpr int kMaxSeqs = 4096;
constexpr int kPartRows = kHeadsPerGroup * kMaxGroup;                // partial rows per piece

struct Params {
    const void *q;
    int q_f16;
    const int32_t *block_tables;
    int max_blocks;
    const int32_t *seq_lens;
    int kv_page0;  // key range of every sequence: [kv_page0 * 32, kv_end) (whole sequence: 0, INT_MAX)
    int kv_end;
    int n_seqs, n_head, n_head_kv, group, n_hg;
    int64_t n_pages;
    float scale_log2;  // softmax scale * log2(e)
    float *out;
    float *lse_out;
    float *part_o;    // [kMaxCtas][2][kPartRows][128]
    float *part_lse;  // [kMaxCtas][2][kPartRows], log2 units
    int32_t *prefix;  // [n_seqs + 1] pages before each sequence
    DeviceStatus *status;
    int q8_dpitch;              // q8_0 cache: bytes per cell row of a stage's scale tile (16 or 32)
    uint64_t wait_ns;           // limit of each pipeline wait (drains keep kWaitLimitNs)
    const int32_t *start_flag;  // optional: the producer waits for it to be non-zero before loading
};

// First page-group of CTA c's range: floor(c P / G). Computed in double precision, which is
// exact here: c P < 2^53 is represented exactly, the quotient is correctly rounded, and a
// non-integer quotient lies at least 1/G below the next integer - more than half an ulp of any
// value below 2^42 while G < 4096 (G <= kMaxCtas, P below 2^31 page-groups) - so the floor of
// the rounded quotient is the floor of the exact one. (A 64-bit integer division costs several
// times the instructions.)
__host__ __device__ inline int64_t range_lo(int c, int64_t P, int G) {
    return (int64_t) ((double) c * (double) P / (double) G);
}

// Keys of sequence b inside the call's range, counted from the range's first page.
__device__ __forceinline__ int range_len(const Params &p, int32_t len) {
    len = len < 0 ? 0 : min(len, p.max_blocks * kPage);
    return max(0, min(len, p.kv_end) - p.kv_page0 * kPage);
}

// Index of the CTA whose range [lo_c, lo_{c+1}) contains page-group x.
__device__ inline int cta_of(int64_t x, int64_t P, int G) {
    int c = (int) ((double) x * (double) G / (double) P);
    while (c + 1 < G && range_lo(c + 1, P, G) <= x) c++;
    while (c > 0 && range_lo(c, P, G) > x) c--;
    return c;
}

// Walks page-groups in index order: sequence b, head group hg, page p.
struct Cursor {
    int b, hg, p;
    __device__ void locate(int64_t x, const int32_t *pfx, int n_seqs, int n_hg) {
        int lo = 0, hi = n_seqs;  // largest b with n_hg * pfx[b] <= x
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if ((int64_t) n_hg * pfx[mid] <= x) lo = mid; else hi = mid - 1;
        }
        b = lo;
        const int np = pfx[b + 1] - pfx[b];
        const int64_t r = x - (int64_t) n_hg * pfx[b];
        hg = (int) (r / np);
        p = (int) (r % np);
    }
    __device__ void advance(const int32_t *pfx, int n_seqs, int n_hg) {
        const int np = pfx[b + 1] - pfx[b];
        if (++p < np) return;
        p = 0;
        if (++hg < n_hg) return;
        hg = 0;
        do { ++b; } while (b < n_seqs && pfx[b + 1] == pfx[b]);
    }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t r[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t r[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ void mma_16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Address of 16-byte chunk `chunk` (0..15 across the 128 dims) of token row `tok` (0..31) in one
// head's page buffer: two 4 KiB swizzled sub-tiles, dims 0..63 then 64..127.
__device__ __forceinline__ uint32_t page_addr(uint32_t base, int tok, int chunk) {
    return base + (uint32_t) (chunk >> 3) * kSubTile + sw128_offset((uint32_t) tok, (uint32_t) (chunk & 7));
}

// Per-warp running state for one (segment piece, KV head): 8 query-head columns, 128 dims.
struct HeadState {
    float o[8][4];   // O^T fragments: m-tile mt covers dims 16mt..16mt+15
    float m[2];      // running max (log2 units) for query heads 2t, 2t+1
    float l[2];      // this lane's partial softmax sums for heads 2t, 2t+1
    uint32_t qb[8][2];
    __device__ void reset() {
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) o[i][j] = 0.f;
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.f;
    }
};

// Loads the B fragments of Q^T (k = dims, n = query heads) for one KV head's query group.
__device__ __forceinline__ void load_q(HeadState &st, const Params &p, int b, int kvh, int lane) {
    const int g = lane >> 2, t = lane & 3;
    const bool live = g < p.group;
    const int64_t row = ((int64_t) b * p.n_head + (int64_t) kvh * p.group + (live ? g : 0)) * kD;
#pragma unroll
    for (int kk = 0; kk < 8; kk++) {
        const int d0 = kk * 16 + 2 * t;
        if (!live) {
            st.qb[kk][0] = st.qb[kk][1] = 0u;
        } else if (p.q_f16) {
            const __half *q = reinterpret_cast<const __half *>(p.q) + row;
            st.qb[kk][0] = *reinterpret_cast<const uint32_t *>(q + d0);
            st.qb[kk][1] = *reinterpret_cast<const uint32_t *>(q + d0 + 8);
        } else {
            const float *q = reinterpret_cast<const float *>(p.q) + row;
            const float2 a = *reinterpret_cast<const float2 *>(q + d0);
            const float2 c = *reinterpret_cast<const float2 *>(q + d0 + 8);
            st.qb[kk][0] = pack_half2(a.x, a.y);
            st.qb[kk][1] = pack_half2(c.x, c.y);
        }
    }
}

// One page (32 tokens, `valid` of them visible) of one KV head.
__device__ __forceinline__ void process_page(HeadState &st, uint32_t kbase, uint32_t vbase, int valid,
                                             float scale_log2, int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int li = lane >> 3, lr = lane & 7;
#pragma unroll
    for (int slab = 0; slab < 2; slab++) {
        if (slab * 16 >= valid) break;
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {
            uint32_t a[4];
            ldsm_x4(page_addr(kbase, slab * 16 + lr + 8 * (li & 1), 2 * kk + (li >> 1)), a);
            mma_16816(s, a, st.qb[kk][0], st.qb[kk][1]);
        }
        // s[0],s[1]: token slab*16+g, heads 2t,2t+1; s[2],s[3]: token +8.
        const int tok0 = slab * 16 + g;
        const bool v0 = tok0 < valid, v1 = tok0 + 8 < valid;
        float x[4];
        x[0] = v0 ? s[0] * scale_log2 : -INFINITY;
        x[1] = v0 ? s[1] * scale_log2 : -INFINITY;
        x[2] = v1 ? s[2] * scale_log2 : -INFINITY;
        x[3] = v1 ? s[3] * scale_log2 : -INFINITY;
        float alpha[2], mu[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float tm = fmaxf(x[h], x[h + 2]);
            tm = warp_max_xor(tm, 4);
            const float mn = fmaxf(st.m[h], tm);
            mu[h] = mn == -INFINITY ? 0.f : mn;
            alpha[h] = fast_exp2(st.m[h] - mu[h]);
            st.m[h] = mn;
        }
        const float p0 = fast_exp2(x[0] - mu[0]);
        const float p1 = fast_exp2(x[1] - mu[1]);
        const float p2 = fast_exp2(x[2] - mu[0]);
        const float p3 = fast_exp2(x[3] - mu[1]);
        st.l[0] = st.l[0] * alpha[0] + (p0 + p2);
        st.l[1] = st.l[1] * alpha[1] + (p1 + p3);
#pragma unroll
        for (int mt = 0; mt < 8; mt++) {
            st.o[mt][0] *= alpha[0];
            st.o[mt][1] *= alpha[1];
            st.o[mt][2] *= alpha[0];
            st.o[mt][3] *= alpha[1];
        }
        const uint32_t pb0 = movmatrix_trans(pack_half2(p0, p1));
        const uint32_t pb1 = movmatrix_trans(pack_half2(p2, p3));
        const bool tail = (slab + 1) * 16 > valid;
#pragma unroll
        for (int mt = 0; mt < 8; mt++) {
            uint32_t a[4];
            ldsm_x4_trans(page_addr(vbase, slab * 16 + lr + 8 * (li >> 1), 2 * mt + (li & 1)), a);
            if (tail) {
                // Zero V where the token is not visible, so stale non-finite cells cannot leak
                // through a zero probability. a0,a1: tokens 2t,2t+1; a2,a3: tokens 2t+8,2t+9.
                const int tb = slab * 16 + 2 * t;
                const uint32_t lo_keep = (tb < valid ? 0x0000ffffu : 0u) | (tb + 1 < valid ? 0xffff0000u : 0u);
                const uint32_t hi_keep = (tb + 8 < valid ? 0x0000ffffu : 0u) | (tb + 9 < valid ? 0xffff0000u : 0u);
                a[0] &= lo_keep;
                a[1] &= lo_keep;
                a[2] &= hi_keep;
                a[3] &= hi_keep;
            }
            mma_16816(st.o[mt], a, pb0, pb1);
        }
    }
}

// ---- q8_0 cache ------------------------------------------------------------------------------
// Planes: qs int8 [n_cells][n_head_kv][128] (a head's page: 32 rows of 128 bytes, loaded with the
// 128-byte swizzle like an f16 half-page) and d f16 [n_cells][n_head_kv][4] (one scale per 32
// values). Stage layout: K qs of the group's 4 heads (4 x 4 KiB), V qs (4 x 4 KiB), then the K and
// V scale tiles: 32 rows (cells) of the group's heads' scales, `dpitch` bytes per row.
constexpr int kQ8HeadPage = kPage * 128;                 // 4 KiB
constexpr int kQ8VOff = kHeadsPerGroup * kQ8HeadPage;    // 16 KiB
constexpr int kQ8KdOff = 2 * kHeadsPerGroup * kQ8HeadPage;
constexpr int kQ8VdOff = kQ8KdOff + kPage * 32;          // scale rows of up to 32 bytes

// Split-kernel shapes. f16: 4 consumer warps (one per KV head of the group, both 16-token slabs of
// a page), 3 stages of 64 KiB. q8_0: a page costs half the bytes and more instructions per byte,
// so 8 consumer warps - warp w takes KV head w % 4 and slab w / 4 of every page - and 2 stages of
// 35 KiB, with two CTAs per SM (the launch doubles the grid) so that 16 consumer warps per SM hide
// a slab's chain of dependent steps (one CTA of four stages streamed at ~0.73 of HBM, two CTAs of
// two stages at ~0.88); the two warps of a head merge their softmax states through shared memory
// at the end of each piece (kMergeBytes: per head, 32 lanes x (2 maxima, 2 sums, 32 accumulators)).
template <bool kQ8>
struct SplitCfg {
    static constexpr int kConsumers = kQ8 ? 8 : kConsumerWarps;
    static constexpr int kThreads = (kConsumers + 1) * 32;
    static constexpr int kStages = kQ8 ? 2 : decode::kStages;
    static constexpr int kStageBytes = kQ8 ? 35 * 1024 : decode::kStageBytes;
    static constexpr int kMergeBytes = kQ8 ? kHeadsPerGroup * 32 * 36 * 4 : 0;
    static constexpr int kBarriers = 2 * kStages + (kQ8 ? 2 * kHeadsPerGroup : 0);
};
// Dynamic shared memory of the split kernel for n_seqs sequences.
template <bool kQ8>
__host__ __device__ constexpr size_t split_smem_bytes(int n_seqs) {
    return 1024 + (size_t) SplitCfg<kQ8>::kStages * SplitCfg<kQ8>::kStageBytes + SplitCfg<kQ8>::kMergeBytes +
           sizeof(uint64_t) * SplitCfg<kQ8>::kBarriers + 16 + sizeof(int32_t) * ((size_t) n_seqs + 1);
}

__device__ __forceinline__ void mma_16832_s8(int c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Per-warp running state over a q8_0 cache: as HeadState, with the query quantised to q8_0.
struct HeadStateQ8 {
    float o[8][4];    // O^T fragments: m-tile mt covers dims 16mt + {2g, 2g + 1} (rows g, g + 8)
    float m[2];
    float l[2];
    uint32_t qq[4][2];  // B fragments of the quantised Q^T, one pair per 32-dim block
    float dq[2][4];     // f16-rounded Q block scales of query heads 2t, 2t + 1
    __device__ void reset() {
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) o[i][j] = 0.f;
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.f;
    }
};

// Quantises query head g's row to q8_0 as ggml does for a q8_0 K (quantize_row_q8_0 of the f32
// row: per 32 values d = amax / 127, q = round-to-nearest-even(x / d)), lane (g, t) keeping the
// bytes its B fragments need (dims 32b + 4t.. and 32b + 16 + 4t..) and the four lanes of a head
// reducing the block's amax; then gathers the scales of heads 2t, 2t + 1 (the S layout).
__device__ __forceinline__ void load_q_q8(HeadStateQ8 &st, const Params &p, int b, int kvh, int lane) {
    const int g = lane >> 2, t = lane & 3;
    const bool live = g < p.group;
    const int64_t row = ((int64_t) b * p.n_head + (int64_t) kvh * p.group + (live ? g : 0)) * kD;
    float dqb[4];
#pragma unroll
    for (int blk = 0; blk < 4; blk++) {
        float x[8];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int d0 = blk * 32 + h * 16 + 4 * t;
            if (!live) {
                x[4 * h] = x[4 * h + 1] = x[4 * h + 2] = x[4 * h + 3] = 0.f;
            } else if (p.q_f16) {
                const __half *q = reinterpret_cast<const __half *>(p.q) + row + d0;
                const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(q));
                const float2 c = __half22float2(*reinterpret_cast<const __half2 *>(q + 2));
                x[4 * h] = a.x, x[4 * h + 1] = a.y, x[4 * h + 2] = c.x, x[4 * h + 3] = c.y;
            } else {
                const float4 v = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(p.q) + row + d0);
                x[4 * h] = v.x, x[4 * h + 1] = v.y, x[4 * h + 2] = v.z, x[4 * h + 3] = v.w;
            }
        }
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(x[i]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.f ? __frcp_rn(d) : 0.f;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            uint32_t w = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) w |= (uint32_t) (__float2int_rn(__fmul_rn(x[4 * h + e], id)) & 0xff) << (8 * e);
            st.qq[blk][h] = w;
        }
        dqb[blk] = __half2float(__float2half_rn(d));
    }
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int blk = 0; blk < 4; blk++) st.dq[h][blk] = __shfl_sync(0xffffffffu, dqb[blk], (2 * t + h) * 4);
}

// Two f16 pairs from four int8 values r = (x0, x1, x2, x3): (x0, x2) and (x1, x3), exactly
// (bytes offset by 128 under the exponent of 1024, then 1152 subtracted).
__device__ __forceinline__ void i8x4_to_f16x2x2(uint32_t r, uint32_t &even, uint32_t &odd) {
    const uint32_t u = r ^ 0x80808080u;
    uint32_t lo, hi;
    asm("prmt.b32 %0, %1, %2, 0x4240;" : "=r"(lo) : "r"(u), "r"(0x64646464u));
    asm("prmt.b32 %0, %1, %2, 0x4341;" : "=r"(hi) : "r"(u), "r"(0x64646464u));
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const __half2 e = __hsub2(*reinterpret_cast<const __half2 *>(&lo), bias);
    const __half2 o = __hsub2(*reinterpret_cast<const __half2 *>(&hi), bias);
    even = *reinterpret_cast<const uint32_t *>(&e);
    odd = *reinterpret_cast<const uint32_t *>(&o);
}

// One page (32 tokens, `valid` visible) of one KV head over the q8_0 planes. S: per 32-dim block
// an int8 MMA (m16n8k32) gives the exact integer dot of the K and Q blocks; the score is
// sum_b (d_k,b * d_q,b) * dot_b in block order, as ggml's q8_0 x q8_0 dot. PV: V's int8 values
// become f16 exactly and each block's scale d_v multiplies P instead (P' = P * d_v per key and
// block, rounded to f16 like P itself), so O^T += V^T . P'^T per 16-dim m-tile; the tile's rows
// are dims 2g, 2g + 1 of its 16 (the pairs ldmatrix.trans delivers).
__device__ __forceinline__ void process_page_q8(HeadStateQ8 &st, uint32_t kbase, uint32_t vbase, const uint8_t *kd,
                                                const uint8_t *vd, int dpitch, int valid, float scale_log2, int lane,
                                                int slab_lo, int slab_hi) {
    const int g = lane >> 2, t = lane & 3;
    const int li = lane >> 3, lr = lane & 7;
    for (int slab = slab_lo; slab < slab_hi; slab++) {
        if (slab * 16 >= valid) break;
        const int tok0 = slab * 16 + g;
        int sb[4][4];
#pragma unroll
        for (int blk = 0; blk < 4; blk++) {
            uint32_t a[4];
            ldsm_x4(kbase + sw128_offset((uint32_t) (slab * 16 + lr + 8 * (li & 1)), (uint32_t) (2 * blk + (li >> 1))),
                    a);
            sb[blk][0] = sb[blk][1] = sb[blk][2] = sb[blk][3] = 0;
            mma_16832_s8(sb[blk], a, st.qq[blk][0], st.qq[blk][1]);
        }
        // scales of tokens tok0 and tok0 + 8 (4 f16 each)
        const uint2 k0 = *reinterpret_cast<const uint2 *>(kd + tok0 * dpitch);
        const uint2 k1 = *reinterpret_cast<const uint2 *>(kd + (tok0 + 8) * dpitch);
        float dk[2][4];
        {
            const float2 a0 = __half22float2(*reinterpret_cast<const __half2 *>(&k0.x));
            const float2 a1 = __half22float2(*reinterpret_cast<const __half2 *>(&k0.y));
            const float2 c0 = __half22float2(*reinterpret_cast<const __half2 *>(&k1.x));
            const float2 c1 = __half22float2(*reinterpret_cast<const __half2 *>(&k1.y));
            dk[0][0] = a0.x, dk[0][1] = a0.y, dk[0][2] = a1.x, dk[0][3] = a1.y;
            dk[1][0] = c0.x, dk[1][1] = c0.y, dk[1][2] = c1.x, dk[1][3] = c1.y;
        }
        // i: (token tok0 + 8 (i >> 1), head 2t + (i & 1)); fused multiply-adds (the result is held to
        // the attention tolerance, not to ggml's exact rounding order)
        float s[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float acc = 0.f;
#pragma unroll
            for (int blk = 0; blk < 4; blk++)
                acc = fmaf((float) sb[blk][i], dk[i >> 1][blk] * st.dq[i & 1][blk], acc);
            s[i] = acc;
        }
        const bool v0 = tok0 < valid, v1 = tok0 + 8 < valid;
        float x[4];
        x[0] = v0 ? s[0] * scale_log2 : -INFINITY;
        x[1] = v0 ? s[1] * scale_log2 : -INFINITY;
        x[2] = v1 ? s[2] * scale_log2 : -INFINITY;
        x[3] = v1 ? s[3] * scale_log2 : -INFINITY;
        float alpha[2], mu[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            float tm = fmaxf(x[h], x[h + 2]);
            tm = warp_max_xor(tm, 4);
            const float mn = fmaxf(st.m[h], tm);
            mu[h] = mn == -INFINITY ? 0.f : mn;
            alpha[h] = fast_exp2(st.m[h] - mu[h]);
            st.m[h] = mn;
        }
        const float p0 = fast_exp2(x[0] - mu[0]);
        const float p1 = fast_exp2(x[1] - mu[1]);
        const float p2 = fast_exp2(x[2] - mu[0]);
        const float p3 = fast_exp2(x[3] - mu[1]);
        st.l[0] = st.l[0] * alpha[0] + (p0 + p2);
        st.l[1] = st.l[1] * alpha[1] + (p1 + p3);
        if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {  // only when a maximum moved
#pragma unroll
            for (int mt = 0; mt < 8; mt++) {
                st.o[mt][0] *= alpha[0];
                st.o[mt][1] *= alpha[1];
                st.o[mt][2] *= alpha[0];
                st.o[mt][3] *= alpha[1];
            }
        }
        // V scales of tokens tok0, tok0 + 8; a key that is not visible gets P' = 0 outright (its
        // stale scale could be non-finite; its P is already 0)
        const uint2 w0 = *reinterpret_cast<const uint2 *>(vd + tok0 * dpitch);
        const uint2 w1 = *reinterpret_cast<const uint2 *>(vd + (tok0 + 8) * dpitch);
        float dv[2][4];
        {
            const float2 a0 = __half22float2(*reinterpret_cast<const __half2 *>(&w0.x));
            const float2 a1 = __half22float2(*reinterpret_cast<const __half2 *>(&w0.y));
            const float2 c0 = __half22float2(*reinterpret_cast<const __half2 *>(&w1.x));
            const float2 c1 = __half22float2(*reinterpret_cast<const __half2 *>(&w1.y));
            dv[0][0] = a0.x, dv[0][1] = a0.y, dv[0][2] = a1.x, dv[0][3] = a1.y;
            dv[1][0] = c0.x, dv[1][1] = c0.y, dv[1][2] = c1.x, dv[1][3] = c1.y;
        }
#pragma unroll
        for (int blk = 0; blk < 4; blk++) {
            const float s0 = v0 ? dv[0][blk] : 0.f, s1 = v1 ? dv[1][blk] : 0.f;
            const uint32_t pb0 = movmatrix_trans(pack_half2(p0 * s0, p1 * s0));
            const uint32_t pb1 = movmatrix_trans(pack_half2(p2 * s1, p3 * s1));
            uint32_t r[4];
            ldsm_x4_trans(vbase + sw128_offset((uint32_t) (slab * 16 + lr + 8 * (li & 1)), (uint32_t) (2 * blk + (li >> 1))),
                          r);
            // r[0] / r[1]: chunk 2 blk, tokens 0-7 / 8-15 of the slab; r[2] / r[3]: chunk 2 blk + 1
#pragma unroll
            for (int hc = 0; hc < 2; hc++) {
                uint32_t a[4];
                i8x4_to_f16x2x2(r[2 * hc], a[0], a[1]);
                i8x4_to_f16x2x2(r[2 * hc + 1], a[2], a[3]);
                mma_16816(st.o[2 * blk + hc], a, pb0, pb1);
            }
        }
    }
}

extern __shared__ __align__(1024) uint8_t dyn_smem[];

// kQ8: the cache is q8_0 planes (kmap / vmap over the qs planes, kdmap / vdmap over the scale
// planes); else f16 rows (kmap / vmap; the scale maps are unused).
template <bool kQ8>
__global__ void __launch_bounds__(SplitCfg<kQ8>::kThreads, kQ8 ? 2 : 1) decode_split_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                    const __grid_constant__ CUtensorMap vmap,
                                                                    const __grid_constant__ CUtensorMap kdmap,
                                                                    const __grid_constant__ CUtensorMap vdmap,
                                                                    const Params p) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;

    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
    constexpr int kConsumers = SplitCfg<kQ8>::kConsumers;
    constexpr int kNThreads = SplitCfg<kQ8>::kThreads;
    constexpr int kNStages = SplitCfg<kQ8>::kStages;
    constexpr int kSBytes = SplitCfg<kQ8>::kStageBytes;
    uint8_t *stages = base;
    float *merge_buf = reinterpret_cast<float *>(base + kNStages * kSBytes);  // q8_0: the second warps' states
    uint64_t *full = reinterpret_cast<uint64_t *>(base + kNStages * kSBytes + SplitCfg<kQ8>::kMergeBytes);
    uint64_t *empty = full + kNStages;
    uint64_t *merge_ready = empty + kNStages;  // q8_0, per head: the slab-1 warp's state is in merge_buf
    uint64_t *merge_taken = merge_ready + kHeadsPerGroup;  // q8_0, per head: the slab-0 warp has read it
    volatile int *abort_flag = reinterpret_cast<volatile int *>(full + SplitCfg<kQ8>::kBarriers);
    int32_t *pfx = reinterpret_cast<int32_t *>(full + SplitCfg<kQ8>::kBarriers) + 4;

    __shared__ int32_t stage_pid[kNStages];  // page id of each stage's page-group (producer -> consumers)
    // Before waiting for the previous kernel (whose work it may overlap): barrier set-up, the
    // tensor-map prefetch, and L2 prefetches of what the prologue and the producer read first -
    // seq_lens, and for a single sequence the block-table entries of this CTA's range as it would
    // be if the sequence filled the call's range (a guess; wrong guesses only cost the prefetch).
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kNStages; s++) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), kConsumers);
        }
        if constexpr (kQ8)
            for (int h = 0; h < kHeadsPerGroup; h++) {
                mbar_init(smem_u32(&merge_ready[h]), 1);
                mbar_init(smem_u32(&merge_taken[h]), 1);
            }
        fence_barrier_init();
    } else if (threadIdx.x == kConsumers * 32) {
        prefetch_tensormap(&kmap);
        prefetch_tensormap(&vmap);
        if constexpr (kQ8) {
            prefetch_tensormap(&kdmap);
            prefetch_tensormap(&vdmap);
        }
    }
    // (Warps 1-3 issue the prefetches, so thread 0's barrier set-up stays short; float arithmetic
    // is plenty for a guess.)
    if (warp >= 1 && warp < kConsumers) {
        const int t = threadIdx.x - 32;
        if (t * 32 < p.n_seqs) prefetch_l2(p.seq_lens + t * 32);
        if (p.n_seqs == 1) {
            const int64_t span =
                min((int64_t) p.max_blocks, ((int64_t) p.kv_end + kPage - 1) / kPage) - (int64_t) p.kv_page0;
            if (span > 0) {
                const float per = (float) span * (float) p.n_hg / (float) gridDim.x;  // page-groups per CTA
                const int64_t x0 = (int64_t) (per * (float) blockIdx.x);
                const int64_t x1 = min((int64_t) (per * (float) (blockIdx.x + 1)) + 1, span * p.n_hg);
                for (int64_t x = x0 + 32 * t; x < x1 + 31; x += 32 * (kConsumers - 1) * 32) {
                    int64_t xe = x < x1 ? x : x1 - 1;  // the range's last entry closes the loop
                    if (xe < x0) continue;
                    while (xe >= span) xe -= span;  // the entry of head group xe / span's page
                    prefetch_l2(p.block_tables + p.kv_page0 + xe);
                }
            }
        }
    }
    // Inputs (q, seq_lens, tables, pages) may come from the previous kernel in the stream; the
    // combine grid may be scheduled right away (it waits for this grid to complete).
    pdl_wait();
    pdl_launch_dependents();
    // Prefix over sequences of page counts (every CTA computes it; CTA 0 publishes it): thread t
    // sums the pages of its run of sequences, a block-wide scan (warp shuffles, then the warps'
    // totals) gives each run's start.
    __shared__ int32_t warp_tot[kNThreads / 32];
    {
        const int per = (p.n_seqs + kNThreads - 1) / kNThreads;
        const int b0 = threadIdx.x * per;
        int32_t local = 0;
        for (int b = b0; b < min(b0 + per, p.n_seqs); b++) {
            const int32_t len = p.seq_lens[b];
            if (len < 0 || len > p.max_blocks * kPage) report(p.status, kStatusBadIndex, kSiteDecodeLen, b);
            local += (range_len(p, len) + kPage - 1) / kPage;
        }
        int32_t incl = local;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int32_t y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        int32_t acc = incl - local;
        for (int w = 0; w < warp; w++) acc += warp_tot[w];
        for (int b = b0; b < min(b0 + per, p.n_seqs); b++) {
            pfx[b] = acc;
            acc += (range_len(p, p.seq_lens[b]) + kPage - 1) / kPage;
        }
        if (threadIdx.x == kNThreads - 1) pfx[p.n_seqs] = acc;
        __syncthreads();
        if (blockIdx.x == 0)
            for (int b = threadIdx.x; b <= p.n_seqs; b += kNThreads) p.prefix[b] = pfx[b];
    }

    const int64_t P = (int64_t) p.n_hg * pfx[p.n_seqs];
    const int64_t lo = range_lo(blockIdx.x, P, gridDim.x);
    const int64_t hi = range_lo(blockIdx.x + 1, P, gridDim.x);

    if (lo < hi && warp == kConsumers) {
        // Producer warp: the whole warp reads the block-table entries of the CTA's page-groups, 32
        // at a time and one batch ahead (lane i: page-group xb + i), so no copy waits on a table
        // read; lane 0 streams the page-groups through the stage ring, handing each stage's page id
        // to the consumers in shared memory.
        __shared__ int32_t batch_pid[2][32];
        __shared__ int32_t batch_hg[2][32];
        uint64_t policy = 0;
        bool ok = true;
        if (lane == 0) {
            policy = l2_policy_evict_first();
            if (p.start_flag != nullptr && !flag_wait_bounded(p.start_flag, abort_flag, p.wait_ns)) {
                report(p.status, kStatusTimeout, kSiteDecodeWaitStart, blockIdx.x);
                *abort_flag = 1;
                ok = false;
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        auto fetch = [&](int64_t xb, int32_t &pid, int &hg) {
            const int64_t x = xb + lane;
            pid = -1;
            hg = 0;
            if (x < hi) {
                Cursor c;
                c.locate(x, pfx, p.n_seqs, p.n_hg);
                hg = c.hg;
                pid = p.block_tables[(int64_t) c.b * p.max_blocks + p.kv_page0 + c.p];
            }
        };
        int32_t pid_next;
        int hg_next;
        fetch(lo, pid_next, hg_next);
        int64_t i = 0;  // page-groups issued (lane 0)
        for (int64_t xb = lo; ok && xb < hi; xb += 32) {
            const int bb = (int) ((xb - lo) >> 5) & 1;
            batch_pid[bb][lane] = pid_next;
            batch_hg[bb][lane] = hg_next;
            __syncwarp();
            if (xb + 32 < hi) fetch(xb + 32, pid_next, hg_next);  // in flight while lane 0 issues
            if (lane == 0) {
                const int cnt = (int) (hi - xb < 32 ? hi - xb : 32);
                for (int e = 0; e < cnt; e++, i++) {
                    const int s = (int) (i % kNStages);
                    const uint32_t k_use = (uint32_t) (i / kNStages);
                    if (k_use > 0 &&
                        !mbar_wait_bounded(smem_u32(&empty[s]), (k_use - 1) & 1, abort_flag, p.wait_ns)) {
                        report(p.status, kStatusTimeout, kSiteDecodeWaitEmpty, s);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const int32_t pid = batch_pid[bb][e];
                    const int hg = batch_hg[bb][e];
                    stage_pid[s] = pid;  // published to the consumers by the arrival below
                    const int nh = min(kHeadsPerGroup, p.n_head_kv - hg * kHeadsPerGroup);
                    const uint32_t fb = smem_u32(&full[s]);
                    if (pid < 0 || pid >= p.n_pages) {
                        report(p.status, kStatusBadIndex, kSiteDecodePage, pid);
                        mbar_arrive(fb);
                    } else if constexpr (kQ8) {
                        mbar_arrive_expect_tx(fb, (uint32_t) (2 * nh * kQ8HeadPage + 2 * kPage * p.q8_dpitch));
                        const uint32_t sb = smem_u32(stages + (size_t) s * kSBytes);
                        for (int h = 0; h < nh; h++) {
                            const int kvh = hg * kHeadsPerGroup + h;
                            tma_load_3d_hint(sb + h * kQ8HeadPage, &kmap, fb, 0, kvh, pid * kPage, policy);
                            tma_load_3d_hint(sb + kQ8VOff + h * kQ8HeadPage, &vmap, fb, 0, kvh, pid * kPage, policy);
                        }
                        // scale rows of the group's heads: x = 16 halves (32 bytes) per group
                        tma_load_2d(sb + kQ8KdOff, &kdmap, fb, hg * 16, pid * kPage);
                        tma_load_2d(sb + kQ8VdOff, &vdmap, fb, hg * 16, pid * kPage);
                    } else {
                        mbar_arrive_expect_tx(fb, (uint32_t) (2 * nh * kHeadPage));
                        const uint32_t sb = smem_u32(stages + (size_t) s * kSBytes);
                        for (int h = 0; h < nh; h++) {
                            const int kvh = hg * kHeadsPerGroup + h;
                            for (int half = 0; half < 2; half++) {
                                const uint32_t off = (uint32_t) (h * kHeadPage + half * kSubTile);
                                tma_load_3d_hint(sb + off, &kmap, fb, half * 64, kvh, pid * kPage, policy);
                                tma_load_3d_hint(sb + kHeadsPerGroup * kHeadPage + off, &vmap, fb, half * 64, kvh,
                                                 pid * kPage, policy);
                            }
                        }
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        if (lane == 0 && (!ok || *abort_flag)) {
            // Let every copy already issued land before the CTA's shared memory goes away.
            const int64_t n_issued = i;
            for (int64_t j = n_issued > kNStages ? n_issued - kNStages : 0; j < n_issued; j++)
                mbar_wait_bounded(smem_u32(&full[j % kNStages]), (uint32_t) (j / kNStages) & 1, nullptr);
        }
    } else if (lo < hi) {
        // Consumers: warp w owns KV head hg*4 + w % 4 of every page-group (q8_0: slab w / 4 of it).
        const int hw = warp % kHeadsPerGroup;
        const int half = warp / kHeadsPerGroup;  // 0, or 1 for the second warp of a head (q8_0)
        int64_t n_pieces = 0;                    // pieces finished (phases of the merge barriers)
        typename std::conditional<kQ8, HeadStateQ8, HeadState>::type st;
        Cursor cur;
        cur.locate(lo, pfx, p.n_seqs, p.n_hg);
        int64_t piece_start = lo;
        int64_t i = 0;
        int len = 0;  // keys of the current segment's sequence inside the call's range
        for (int64_t x = lo; x < hi; x++, i++) {
            const int np = pfx[cur.b + 1] - pfx[cur.b];
            const int kvh = cur.hg * kHeadsPerGroup + hw;
            const bool active = kvh < p.n_head_kv;
            if (x == lo || cur.p == 0) {
                piece_start = x;
                st.reset();
                if (active) {
                    if constexpr (kQ8) load_q_q8(st, p, cur.b, kvh, lane);
                    else load_q(st, p, cur.b, kvh, lane);
                }
                len = range_len(p, p.seq_lens[cur.b]);
            }
            const int s = (int) (i % kNStages);
            // Warp-uniform outcome: ldmatrix / mma.sync below are warp-collective.
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&full[s]), (uint32_t) (i / kNStages) & 1,
                                                             abort_flag, p.wait_ns))) {
                if (lane == 0) {
                    report(p.status, kStatusTimeout, kSiteDecodeWaitFull, s);
                    *abort_flag = 1;
                }
                break;
            }
            const int32_t pid = stage_pid[s];
            if (active && pid >= 0 && pid < p.n_pages) {
                const int valid = min(kPage, len - cur.p * kPage);
                const uint32_t sb = smem_u32(stages + (size_t) s * kSBytes);
                if constexpr (kQ8) {
                    const uint8_t *st_base = stages + (size_t) s * kSBytes;
                    process_page_q8(st, sb + hw * kQ8HeadPage, sb + kQ8VOff + hw * kQ8HeadPage,
                                    st_base + kQ8KdOff + hw * 8, st_base + kQ8VdOff + hw * 8, p.q8_dpitch, valid,
                                    p.scale_log2, lane, half, half + 1);
                } else {
                    process_page(st, sb + warp * kHeadPage, sb + kHeadsPerGroup * kHeadPage + warp * kHeadPage,
                                 valid, p.scale_log2, lane);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty[s]));

            if (cur.p == np - 1 || x == hi - 1) {
                // Piece ends: finish the softmax sums and write the (partial) result.
                if constexpr (kQ8) {
                    // The slab-1 warp hands its state to the slab-0 warp of its head, which merges:
                    // M = max(m_a, m_b), O = O_a 2^(m_a - M) + O_b 2^(m_b - M), the same for the sums.
                    float *mb = merge_buf + (hw * 32 + lane) * 36;
                    const uint32_t par = (uint32_t) (n_pieces & 1);
                    bool ok = true;
                    if (half == 1) {
                        if (n_pieces > 0)
                            ok = mbar_wait_bounded(smem_u32(&merge_taken[hw]), par ^ 1u, abort_flag, p.wait_ns);
                        ok = __all_sync(0xffffffffu, ok);  // warp-uniform: __syncwarp below
                        if (ok) {
                            mb[0] = st.m[0], mb[1] = st.m[1], mb[2] = st.l[0], mb[3] = st.l[1];
#pragma unroll
                            for (int mt = 0; mt < 8; mt++)
#pragma unroll
                                for (int j = 0; j < 4; j++) mb[4 + mt * 4 + j] = st.o[mt][j];
                            __syncwarp();
                            if (lane == 0) mbar_arrive(smem_u32(&merge_ready[hw]));
                        }
                    } else {
                        ok = __all_sync(0xffffffffu,
                                        mbar_wait_bounded(smem_u32(&merge_ready[hw]), par, abort_flag, p.wait_ns));
                        if (ok) {
#pragma unroll
                            for (int h = 0; h < 2; h++) {
                                const float mo = mb[h], M = fmaxf(st.m[h], mo);
                                const float fa = M == -INFINITY ? 0.f : fast_exp2(st.m[h] - M);
                                const float fb = M == -INFINITY ? 0.f : fast_exp2(mo - M);
                                st.l[h] = st.l[h] * fa + mb[2 + h] * fb;
                                st.m[h] = M;
#pragma unroll
                                for (int mt = 0; mt < 8; mt++) {
                                    st.o[mt][h] = st.o[mt][h] * fa + mb[4 + mt * 4 + h] * fb;
                                    st.o[mt][h + 2] = st.o[mt][h + 2] * fa + mb[4 + mt * 4 + h + 2] * fb;
                                }
                            }
                            __syncwarp();
                            if (lane == 0) mbar_arrive(smem_u32(&merge_taken[hw]));
                        }
                    }
                    n_pieces++;
                    if (!__all_sync(0xffffffffu, ok)) {
                        if (lane == 0) {
                            report(p.status, kStatusTimeout, kSiteDecodeWaitMerge, hw);
                            *abort_flag = 1;
                        }
                        break;
                    }
                    if (half == 1) {
                        cur.advance(pfx, p.n_seqs, p.n_hg);
                        continue;
                    }
                }
                const int g = lane >> 2, t = lane & 3;
                float l[2];
                l[0] = warp_sum_xor(st.l[0], 4);
                l[1] = warp_sum_xor(st.l[1], 4);
                const bool whole = piece_start == x - cur.p && cur.p == np - 1;
                if (active) {
                    const int slot = piece_start == lo ? 0 : 1;
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int n = 2 * t + h;
                        if (n >= p.group) continue;
                        const float inv = l[h] > 0.f ? 1.f / l[h] : 0.f;
                        const float lse2 = l[h] > 0.f ? st.m[h] + __log2f(l[h]) : -INFINITY;
                        float *dst;
                        if (whole) {
                            dst = p.out + ((int64_t) cur.b * p.n_head + (int64_t) kvh * p.group + n) * kD;
                            if (g == 0 && p.lse_out != nullptr)
                                p.lse_out[(int64_t) cur.b * p.n_head + (int64_t) kvh * p.group + n] =
                                    lse2 * 0.69314718055994531f;
                        } else {
                            const int64_t prow = ((int64_t) blockIdx.x * 2 + slot) * kPartRows +
                                                 (int64_t) hw * kMaxGroup + n;
                            dst = p.part_o + prow * kD;
                            if (g == 0) p.part_lse[prow] = lse2;
                        }
#pragma unroll
                        for (int mt = 0; mt < 8; mt++) {
                            if constexpr (kQ8) {  // m-tile rows g, g + 8 are dims 2g, 2g + 1
                                *reinterpret_cast<float2 *>(dst + mt * 16 + 2 * g) =
                                    make_float2(st.o[mt][h] * inv, st.o[mt][h + 2] * inv);
                            } else {
                                dst[mt * 16 + g] = st.o[mt][h] * inv;
                                dst[mt * 16 + g + 8] = st.o[mt][h + 2] * inv;
                            }
                        }
                    }
                }
            }
            cur.advance(pfx, p.n_seqs, p.n_hg);
        }
    }
    __syncthreads();
}

constexpr int kCombineThreads = 256;
constexpr int kCombineWarps = kCombineThreads / 32;

struct CombineParams {
    int n_seqs, n_head, n_head_kv, group, n_hg, grid;
    int dsplit;  // CTAs per output row (1, 2 or 4), each owning 128 / dsplit consecutive dims
    const int32_t *prefix;
    const float *part_o;
    const float *part_lse;
    float *out;
    float *lse_out;
    // Exchange across ranks (decode_combine_kernel<true>): the mailboxes of the exchange-merge
    // protocol (exchange.cuh) for n_seqs * n_head rows, this rank, the rank count, the flag-wait
    // bound and the device status.
    uint8_t *const *mailboxes;
    int rank, n_ranks;
    uint64_t wait_ns;
    DeviceStatus *status;
};

// CTAs per output row of decode_combine_kernel (1, 2 or 4): rows over many pieces (8 or more per
// segment) are split while the grid stays within one CTA per SM - one long sequence (32 rows)
// goes over 128 CTAs, each reading a quarter of every piece - and no further, since a CTA's fixed
// cost (launch, plan, barriers) is paid once per CTA. Fused exchange: every combine CTA owns an
// epoch counter in the mailbox header, so the grid must fit it.
__host__ __device__ inline int combine_dsplit(int n_seqs, int n_hg, int grid, bool exchange, int max_ctas, int n_sms) {
    const int64_t segs = (int64_t) n_seqs * n_hg;
    const int64_t per = segs > 0 ? grid / segs : 0;  // pieces per segment, about
    int d = 1;
    if (per >= 8)
        while (d < 4 && segs * kPartRows * d * 2 <= n_sms) d *= 2;
    while (exchange && d > 1 && segs * kPartRows * d > max_ctas) d >>= 1;
    return d;
}

// Batches whose segments average fewer than 16 pieces (more than a few sequences per grid) merge
// a row per warp (decode_combine_rows_kernel: one round trip for up to 16 pieces); longer rows
// spread over CTAs.
__host__ __device__ inline bool combine_by_rows(int n_seqs, int n_hg, int grid) {
    const int64_t segs = (int64_t) n_seqs * n_hg;
    return segs > 0 && grid / segs < 16;
}

// The slow path of a poll: spins on word w until it carries `epoch` (bounded: after wait_ns from
// t_start it reports the timeout once and returns 0). Out of line, so the inlined fast path (the
// word had already landed) stays small: after a launch every stretch of code is fetched anew.
__device__ __noinline__ float exchange_spin(const uint64_t *w, uint32_t epoch, uint64_t t_start, uint64_t wait_ns,
                                            DeviceStatus *status, int src, bool &timed_out) {
    for (uint32_t i = 1;; i++) {
        const uint64_t x = exchange::ld_relaxed_sys_u64(w);
        if ((uint32_t) (x >> 32) == epoch) return __uint_as_float((uint32_t) x);
        if ((i & 63u) == 0 && global_timer_ns() - t_start > wait_ns) {
            if (!timed_out) report(status, kStatusTimeout, kSiteExchangeWait, src);
            timed_out = true;
            return 0.f;
        }
    }
}

// A combine CTA's exchange state, read at the kernel's start (off the critical path): its own
// mailbox, its epoch for this call, and (in shared memory) every rank's mailbox address.
struct ExchangeState {
    uint8_t *own;
    uint32_t epoch;
    uint8_t *const *mb;  // shared memory [n_ranks]
};

// The end of a combine CTA's share of a row: dims [d0, d0 + nd), thread t < nd holding dim
// d0 + t in o, and the row's lse (natural log; every CTA of the row has the same). Without an
// exchange, out (and, from the row's first CTA, lse_out) get the local values. With one, the
// share goes to every peer (exchange.cuh's mailboxes) and out / lse_out get the log-sum-exp merge
// of the R ranks' rows. A share travels as words of 8 bytes - a value's f32 bits and the call's
// epoch - stored straight into slot `rank` of every peer's mailbox (plain peer stores; the lse
// word by the row's first CTA); a reader polls the words of its own mailbox until each carries
// the epoch, and an 8-byte word is written and read whole, so no flag and no system-scope fence
// is needed. Waits are bounded by wait_ns (on timeout the status records it and the share is
// zeros). The epoch is the mailbox header counter of the CTA's linear index, advanced once per
// call by every CTA of the grid (see advance_epoch), so calls replay from a CUDA graph and the
// CTAs of one row always agree on it; words alternate between two banks by epoch parity (a rank
// is at most one call ahead of a peer: it needs the peer's row of the current call to finish it).
template <bool kExchange>
__device__ __forceinline__ void finish_row(const CombineParams &p, int64_t row, int d0, int nd, float o, float lse,
                                           const ExchangeState &xs) {
    const int tid = threadIdx.x;
    const bool first = d0 == 0;
    if constexpr (!kExchange) {
        if (tid < nd) p.out[row * kD + d0 + tid] = o;
        if (tid == 0 && first && p.lse_out != nullptr) p.lse_out[row] = lse;
    } else {
        // Thread t < nd sends its dim's word to every peer and polls the same dim's word of every
        // peer in its own mailbox (thread 0 also the lse words), then merges the R sources in rank
        // order - the same order on every rank - online in chunks of 8 with all of a chunk's loads
        // issued before any is checked: no shared memory and no block barrier, so a share costs
        // one memory round trip once the peers' words have landed. On a timeout (a word still
        // without this call's epoch after wait_ns) the thread reports it and writes zero.
        if (tid >= nd) return;
        const int R = p.n_ranks;
        const int64_t n_rows = (int64_t) p.n_seqs * p.n_head;
        const uint32_t epoch = xs.epoch;
        const int bank = (int) (epoch & 1u);
        const size_t w_off = exchange::words_offset(R, n_rows);
        const int64_t slot = n_rows * (kD + 1);  // words per (bank, source)
        const uint64_t tag = (uint64_t) epoch << 32;
        const uint64_t t_start = global_timer_ns();  // the waits below are bounded from here
        const int64_t w_row = ((int64_t) bank * R + p.rank) * slot + row * (kD + 1);
        for (int r = 0; r < R; r++) {
            if (r == p.rank) continue;
            uint64_t *w = reinterpret_cast<uint64_t *>(xs.mb[r] + w_off) + w_row;
            exchange::st_relaxed_sys_u64(w + d0 + tid, tag | __float_as_uint(o));
            if (tid == 0 && first) exchange::st_relaxed_sys_u64(w + kD, tag | __float_as_uint(lse));
        }
        const uint64_t *base = reinterpret_cast<const uint64_t *>(xs.own + w_off) + (int64_t) bank * R * slot + row * (kD + 1);
        bool timed_out = false;
        auto value = [&](uint64_t x, const uint64_t *w, int src) -> float {
            if ((uint32_t) (x >> 32) == epoch) return __uint_as_float((uint32_t) x);
            return exchange_spin(w, epoch, t_start, p.wait_ns, p.status, src, timed_out);
        };
        constexpr int kChunk = 8;
        float M = -INFINITY, den = 0.f, acc = 0.f;
        for (int r0 = 0; r0 < R; r0 += kChunk) {
            uint64_t lw[kChunk], xw[kChunk];
#pragma unroll
            for (int k = 0; k < kChunk; k++) {
                const int r = r0 + k;
                if (r < R && r != p.rank) {
                    lw[k] = exchange::ld_relaxed_sys_u64(base + (int64_t) r * slot + kD);
                    xw[k] = exchange::ld_relaxed_sys_u64(base + (int64_t) r * slot + d0 + tid);
                }
            }
            float lv[kChunk], xv[kChunk];
#pragma unroll
            for (int k = 0; k < kChunk; k++) {
                const int r = r0 + k;
                lv[k] = -INFINITY, xv[k] = 0.f;
                if (r == p.rank) {
                    lv[k] = lse, xv[k] = o;
                } else if (r < R) {
                    lv[k] = value(lw[k], base + (int64_t) r * slot + kD, r);
                    xv[k] = value(xw[k], base + (int64_t) r * slot + d0 + tid, r);
                }
            }
            float cm = M;
#pragma unroll
            for (int k = 0; k < kChunk; k++) cm = fmaxf(cm, lv[k]);
            if (cm != -INFINITY) {
                const float f = __expf(M - cm);
                den *= f;
                acc *= f;
#pragma unroll
                for (int k = 0; k < kChunk; k++) {
                    const float wt = __expf(lv[k] - cm);
                    den += wt;
                    acc += wt * xv[k];
                }
                M = cm;
            }
        }
        const bool ok = M != -INFINITY && !timed_out;
        p.out[row * kD + d0 + tid] = ok ? acc / den : 0.f;
        if (tid == 0 && first && p.lse_out != nullptr) p.lse_out[row] = ok ? M + __logf(den) : -INFINITY;
    }
}

// Every CTA of an exchanging combine grid, whatever it does, advances its epoch counter once per
// call (after its last read of it), so CTAs that share a row in one call have the same history.
template <bool kExchange>
__device__ __forceinline__ void advance_epoch(const CombineParams &p, const ExchangeState &xs) {
    if constexpr (kExchange) {
        if (threadIdx.x == 0)
            reinterpret_cast<uint32_t *>(xs.own)[(blockIdx.x * gridDim.y + blockIdx.y) * gridDim.z + blockIdx.z] =
                xs.epoch;
    }
}

// Merges (m, den, acc) running states: M = max, weights 2^(m - M).
__device__ __forceinline__ void merge_state(float &m, float &den, float4 &acc, float m2, float den2, float4 acc2) {
    const float M = fmaxf(m, m2);
    if (M == -INFINITY) return;
    const float f1 = exp2f(m - M), f2 = exp2f(m2 - M);
    den = den * f1 + den2 * f2;
    acc.x = acc.x * f1 + acc2.x * f2;
    acc.y = acc.y * f1 + acc2.y * f2;
    acc.z = acc.z * f1 + acc2.z * f2;
    acc.w = acc.w * f1 + acc2.w * f2;
    m = M;
}

// Grid (sequence b, head group hg, 32 x dsplit): CTA z owns query row z / dsplit of the group's
// 4 x 8 partial rows (KV head w, query head n) and dims [d0, d0 + nd) of it, nd = 128 / dsplit.
// The row's pieces - one per split CTA whose range touched the segment, up to the split grid for
// a single long sequence - are read in one pass: lane group j of a warp (nd / 4 lanes, a float4
// each) takes pieces j, j + stride, ... and loads each piece's lse together with its slice of O,
// so the whole row costs one memory round trip after the prefix; each lane keeps an online
// (max, sum, accumulator) state, merged across lane groups by shuffles and across warps in shared
// memory. Piece i is split CTA c0 + i; its record is slot 0 of that CTA's pair, except for the
// first piece when the CTA's range began in an earlier segment (slot 1).
template <bool kExchange>
__global__ void __launch_bounds__(kCombineThreads, 2) decode_combine_kernel(const CombineParams p) {
    pdl_wait();  // the split grid's partials and prefix are complete and visible
    const int S = p.dsplit;
    const int b = blockIdx.x, hg = blockIdx.y;
    const int zr = blockIdx.z / S, q = blockIdx.z - zr * S;
    const int w = zr / kMaxGroup, n = zr % kMaxGroup;
    const int kvh = hg * kHeadsPerGroup + w;
    const int nd = kD / S, d0 = q * nd;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ uint8_t *mb_s[kExchange ? kCombineThreads : 1];
    ExchangeState xs{nullptr, 0u, mb_s};
    if constexpr (kExchange) {
        xs.own = p.mailboxes[p.rank];
        xs.epoch = reinterpret_cast<const uint32_t *>(xs.own)[(blockIdx.x * gridDim.y + blockIdx.y) * gridDim.z +
                                                              blockIdx.z] + 1u;
        if (tid < p.n_ranks) mb_s[tid] = p.mailboxes[tid];  // published by the plan's barrier below
    }
    if (kvh >= p.n_head_kv || n >= p.group) {
        __syncthreads();  // every thread has read the epoch counter before it is advanced
        advance_epoch<kExchange>(p, xs);
        return;
    }
    const int64_t out_row = (int64_t) b * p.n_head + (int64_t) kvh * p.group + n;
    const int part_row = w * kMaxGroup + n;
    const int lp = nd / 4;  // lanes per piece
    const int pw = 32 / lp;  // pieces per warp load
    const int sub = warp * pw + lane / lp, li = lane % lp;
    const int stride = kCombineWarps * pw;
    constexpr int kBatch = 8;  // one batch covers the pieces of a lane group in every dsplit case
    float lv[kBatch];
    float4 v[kBatch];
    // Loads one batch: pieces i0, i0 + stride, ... of the CTA range [c0, c0 + n_pc).
    auto load = [&](int i0, int c0, int n_pc, int first_slot, bool may_be_empty, int64_t P) {
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int i = i0 + k * stride;
            lv[k] = -INFINITY;
            v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < n_pc) {
                const int c = c0 + i;
                bool ok = true;
                if (may_be_empty) ok = range_lo(c + 1, P, p.grid) > range_lo(c, P, p.grid);
                if (ok) {
                    const int64_t prow = (int64_t) (c * 2 + (i == 0 ? first_slot : 0)) * kPartRows + part_row;
                    lv[k] = p.part_lse[prow];
                    v[k] = reinterpret_cast<const float4 *>(p.part_o + prow * kD + d0)[li];
                }
            }
        }
    };
    float m = -INFINITY, den = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    auto accumulate = [&]() {
        float bm = m;
#pragma unroll
        for (int k = 0; k < kBatch; k++) bm = fmaxf(bm, lv[k]);
        if (bm != -INFINITY) {
            const float f = exp2f(m - bm);
            den *= f;
            acc.x *= f, acc.y *= f, acc.z *= f, acc.w *= f;
#pragma unroll
            for (int k = 0; k < kBatch; k++) {
                const float wt = exp2f(lv[k] - bm);  // 0 for an absent piece
                den += wt;
                acc.x += wt * v[k].x, acc.y += wt * v[k].y, acc.z += wt * v[k].z, acc.w += wt * v[k].w;
            }
            m = bm;
        }
    };
    // One sequence whose head groups divide the split grid evenly (a single context over the
    // whole grid): the row's pieces are loaded in the same round trip as the prefix, on the
    // assumption that head group hg's segment is exactly CTAs [hg g, (hg + 1) g), g = grid / n_hg.
    // That holds when the sequence has at least g pages (P >= grid: CTA hg g's range then starts
    // at the segment's first page-group and no range is empty, so every piece is its CTA's
    // first, slot 0); otherwise the pieces are loaded again below.
    const int per_hg = p.grid / p.n_hg;
    const bool guess = p.n_seqs == 1 && per_hg * p.n_hg == p.grid && per_hg >= 2 && per_hg <= stride * kBatch;
    if (guess) load(sub, hg * per_hg, per_hg, 0, false, 0);
    // The row's plan, worked out by one thread (the range arithmetic is the costly part of a
    // short row) and shared: 0 = the guess holds, 1 = no keys, 2 = written by one split CTA,
    // 3 = pieces c0 .. c0 + n_pc - 1.
    __shared__ int plan_s[4];
    __shared__ long long plan_P;
    if (tid == 0) {
        const int32_t pb = p.prefix[b];
        const int np = p.prefix[b + 1] - pb;
        const int64_t P = (int64_t) p.n_hg * p.prefix[p.n_seqs];
        int mode = 0, c0 = 0, n_pc = 0, first_slot = 0;
        if (!(guess && P >= p.grid)) {
            if (np == 0) {
                mode = 1;
            } else {
                const int64_t x0 = (int64_t) p.n_hg * pb + (int64_t) hg * np;
                c0 = cta_of(x0, P, p.grid);
                const int c1 = cta_of(x0 + np - 1, P, p.grid);
                mode = c0 == c1 ? 2 : 3;
                n_pc = c1 - c0 + 1;  // <= p.grid <= kMaxCtas
                first_slot = range_lo(c0, P, p.grid) < x0 ? 1 : 0;
            }
        }
        plan_s[0] = mode, plan_s[1] = c0, plan_s[2] = n_pc, plan_s[3] = first_slot;
        plan_P = P;
    }
    __syncthreads();
    // Every path below ends in the one call of finish_row (one copy of its code: after a cold
    // start each new stretch of code is fetched from memory).
    const int mode = plan_s[0];
    if (mode == 2 && !kExchange) return;  // the split kernel wrote this row directly
    if (mode == 3) {
        const int c0 = plan_s[1], n_pc = plan_s[2], first_slot = plan_s[3];
        const int64_t P = plan_P;
        const bool may_be_empty = P < p.grid;  // only then can a split CTA's range be empty
        for (int i0 = sub; i0 < n_pc; i0 += stride * kBatch) {
            load(i0, c0, n_pc, first_slot, may_be_empty, P);
            accumulate();
        }
    } else if (mode == 0) {
        accumulate();
    }
    float o = 0.f, row_lse = -INFINITY;
    if (mode == 2) {  // with an exchange: the local row the split kernel wrote
        if (tid < nd) o = p.out[out_row * kD + d0 + tid];
        row_lse = p.lse_out[out_row];
    } else if (mode != 1) {
        // Lane groups of a warp hold the same dims: merge them (offsets lp, 2 lp, ...).
        for (int off = lp; off < 32; off <<= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
            const float den2 = __shfl_xor_sync(0xffffffffu, den, off);
            float4 a2;
            a2.x = __shfl_xor_sync(0xffffffffu, acc.x, off);
            a2.y = __shfl_xor_sync(0xffffffffu, acc.y, off);
            a2.z = __shfl_xor_sync(0xffffffffu, acc.z, off);
            a2.w = __shfl_xor_sync(0xffffffffu, acc.w, off);
            merge_state(m, den, acc, m2, den2, a2);
        }
        __shared__ float m_s[kCombineWarps], den_s[kCombineWarps];
        __shared__ __align__(16) float acc_s[kCombineWarps][kD];  // written as float4
        if (lane < lp) reinterpret_cast<float4 *>(acc_s[warp])[lane] = acc;
        if (lane == 0) m_s[warp] = m, den_s[warp] = den;
        __syncthreads();
        float M = -INFINITY;
        for (int k = 0; k < kCombineWarps; k++) M = fmaxf(M, m_s[k]);
        float total = 0.f;  // on every thread: the exchange needs the row's lse in all of them
        if (M != -INFINITY) {
            for (int k = 0; k < kCombineWarps; k++) {
                const float f = exp2f(m_s[k] - M);
                total += den_s[k] * f;
                if (tid < nd) o += acc_s[k][tid] * f;
            }
        }
        o = total > 0.f ? o / total : 0.f;
        row_lse = total > 0.f ? (M + __log2f(total)) * 0.69314718055994531f : -INFINITY;
    }
    finish_row<kExchange>(p, out_row, d0, nd, o, row_lse, xs);
    advance_epoch<kExchange>(p, xs);
}

// The combine for a batch of short rows (no exchange): grid (sequence b, head group hg, KV head
// w of the group), warp n merging query row n's pieces on its own - lane l the float4 of dims
// 4l .. 4l + 3 of each piece, 16 pieces in flight, an online (max, sum, accumulator) state -
// and writing the row, so nothing crosses warps after the segment's plan, which thread 0 works
// out once for the CTA's eight rows. Chosen where segments have few pieces (many sequences per
// grid); a long row over many pieces takes decode_combine_kernel, which spreads it over CTAs.
__global__ void __launch_bounds__(kCombineThreads, 2) decode_combine_rows_kernel(const CombineParams p) {
    pdl_wait();  // the split grid's partials and prefix are complete and visible
    const int b = blockIdx.x, hg = blockIdx.y, w = blockIdx.z;
    const int kvh = hg * kHeadsPerGroup + w;
    if (kvh >= p.n_head_kv) return;
    const int tid = threadIdx.x, lane = tid & 31, n = tid >> 5;
    __shared__ int plan_s[4];  // mode (1 no keys, 2 written by one split CTA, 3 pieces), c0, n_pc, first slot
    __shared__ long long plan_P;
    if (tid == 0) {
        const int32_t pb = p.prefix[b];
        const int np = p.prefix[b + 1] - pb;
        const int64_t P = (int64_t) p.n_hg * p.prefix[p.n_seqs];
        int mode = 1, c0 = 0, n_pc = 0, first_slot = 0;
        if (np > 0) {
            const int64_t x0 = (int64_t) p.n_hg * pb + (int64_t) hg * np;
            c0 = cta_of(x0, P, p.grid);
            const int c1 = cta_of(x0 + np - 1, P, p.grid);
            mode = c0 == c1 ? 2 : 3;
            n_pc = c1 - c0 + 1;
            first_slot = range_lo(c0, P, p.grid) < x0 ? 1 : 0;
        }
        plan_s[0] = mode, plan_s[1] = c0, plan_s[2] = n_pc, plan_s[3] = first_slot;
        plan_P = P;
    }
    __syncthreads();
    const int mode = plan_s[0];
    if (n >= p.group || mode == 2) return;
    const int64_t out_row = (int64_t) b * p.n_head + (int64_t) kvh * p.group + n;
    float4 *dst = reinterpret_cast<float4 *>(p.out + out_row * kD) + lane;
    if (mode == 1) {
        *dst = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane == 0 && p.lse_out != nullptr) p.lse_out[out_row] = -INFINITY;
        return;
    }
    const int c0 = plan_s[1], n_pc = plan_s[2], first_slot = plan_s[3];
    const int64_t P = plan_P;
    const bool may_be_empty = P < p.grid;
    const int part_row = w * kMaxGroup + n;
    constexpr int kBatch = 16;
    float m = -INFINITY, den = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i0 = 0; i0 < n_pc; i0 += kBatch) {
        float lv[kBatch];
        float4 v[kBatch];
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int i = i0 + k, c = c0 + i;
            lv[k] = -INFINITY;
            v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < n_pc && (!may_be_empty || range_lo(c + 1, P, p.grid) > range_lo(c, P, p.grid))) {
                const int64_t prow = (int64_t) (c * 2 + (i == 0 ? first_slot : 0)) * kPartRows + part_row;
                lv[k] = p.part_lse[prow];
                v[k] = reinterpret_cast<const float4 *>(p.part_o + prow * kD)[lane];
            }
        }
        float bm = m;
#pragma unroll
        for (int k = 0; k < kBatch; k++) bm = fmaxf(bm, lv[k]);
        if (bm != -INFINITY) {
            const float f = exp2f(m - bm);
            den *= f;
            acc.x *= f, acc.y *= f, acc.z *= f, acc.w *= f;
#pragma unroll
            for (int k = 0; k < kBatch; k++) {
                const float wt = exp2f(lv[k] - bm);  // 0 for an absent piece
                den += wt;
                acc.x += wt * v[k].x, acc.y += wt * v[k].y, acc.z += wt * v[k].z, acc.w += wt * v[k].w;
            }
            m = bm;
        }
    }
    // Divided as decode_combine_kernel divides: a row of up to 8 pieces then gets the same bits
    // from both kernels (the same weights, summed in piece order).
    *dst = den > 0.f ? make_float4(acc.x / den, acc.y / den, acc.z / den, acc.w / den) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (lane == 0 && p.lse_out != nullptr)
        p.lse_out[out_row] = den > 0.f ? (m + __log2f(den)) * 0.69314718055994531f : -INFINITY;
}

// LSE merge of n_parts partial results (natural-log lse), one warp per output row.
__global__ void __launch_bounds__(256) lse_merge_kernel(const float *o_parts, const float *lse_parts, int n_parts,
                                                        int64_t n_rows, int head_dim, int64_t o_stride,
                                                        int64_t lse_stride, float *out, float *lse_out) {
    const int64_t row = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= n_rows) return;
    float M = -INFINITY;
    for (int r = 0; r < n_parts; r++) M = fmaxf(M, lse_parts[(int64_t) r * lse_stride + row]);
    float den = 0.f;
    for (int d = lane; d < head_dim; d += 32) out[row * head_dim + d] = 0.f;
    if (M == -INFINITY) {
        if (lane == 0 && lse_out) lse_out[row] = -INFINITY;
        return;
    }
    for (int d = lane; d < head_dim; d += 32) {
        float acc = 0.f;
        float dn = 0.f;
        for (int r = 0; r < n_parts; r++) {
            const float wt = __expf(lse_parts[(int64_t) r * lse_stride + row] - M);
            dn += wt;
            acc += wt * o_parts[(int64_t) r * o_stride + row * head_dim + d];
        }
        out[row * head_dim + d] = acc / dn;
        den = dn;
    }
    den = __shfl_sync(0xffffffffu, den, 0);
    if (lane == 0 && lse_out) lse_out[row] = M + __logf(den);
}

}  // namespace decode
}  // namespace lstk
