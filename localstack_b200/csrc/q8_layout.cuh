// q8_layout.cuh - conversion between ggml's block_q8_0 rows and the q8_0 planes of the cache, and
// the dequantising page gather that lets the f16 prefill read a q8_0 cache.
//
// ggml stores a q8_0 row of 128 values as 4 blocks of 34 bytes: the f16 scale d, then 32 int8
// values (block_q8_0). The cache keeps the same bytes as two planes, qs int8 [rows][128] and d f16
// [rows][4], so its rows stay 16-byte aligned for TMA. These kernels move the bytes between the
// two layouts (no arithmetic), in units of 16-bit words: word w of block i is its scale (w = 0)
// or values 2(w - 1), 2(w - 1) + 1.
#pragma once

#include "common.cuh"

namespace lstk {
namespace q8 {

constexpr int kBlockWords = 17;  // 34 bytes

__global__ void __launch_bounds__(256) from_blocks_kernel(const uint16_t *blocks, int64_t n_blocks, uint16_t *qs,
                                                          uint16_t *d) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t total = n_blocks * kBlockWords;
    for (int64_t k = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; k < total; k += (int64_t) gridDim.x * blockDim.x) {
        const int64_t i = k / kBlockWords;
        const int w = (int) (k - i * kBlockWords);
        const uint16_t v = blocks[k];
        if (w == 0) d[i] = v;
        else qs[i * 16 + (w - 1)] = v;
    }
}

__global__ void __launch_bounds__(256) to_blocks_kernel(const uint16_t *qs, const uint16_t *d, int64_t n_blocks,
                                                        uint16_t *blocks) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t total = n_blocks * kBlockWords;
    for (int64_t k = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; k < total; k += (int64_t) gridDim.x * blockDim.x) {
        const int64_t i = k / kBlockWords;
        const int w = (int) (k - i * kBlockWords);
        blocks[k] = w == 0 ? d[i] : qs[i * 16 + (w - 1)];
    }
}

// Prefill over a q8_0 cache: the pages a call reads, dequantised into a compact f16 cache with
// dense block tables (sequence b's page p -> scratch page b * max_blocks + p), which the f16
// prefill then reads. CTA (p, b) converts one page of K and V (its keys below kv_lens[b]): 16
// values per thread from one 16-byte load, each d * q rounded once to f16.
__global__ void __launch_bounds__(256) gather_dequant_kernel(const int8_t *k_qs, const __half *k_d, const int8_t *v_qs,
                                                             const __half *v_d, int hkv, int64_t n_pages_src,
                                                             const int32_t *block_tables, int max_blocks,
                                                             const int32_t *kv_lens, __half *k_out, __half *v_out,
                                                             int32_t *bt_out, DeviceStatus *status) {
    pdl_wait();
    pdl_launch_dependents();
    const int p = blockIdx.x, b = blockIdx.y;
    const int64_t dst_page = (int64_t) b * max_blocks + p;
    if (threadIdx.x == 0) bt_out[dst_page] = (int32_t) dst_page;
    const int len = kv_lens[b];
    const int32_t src_page = p * 32 < len ? block_tables[dst_page] : -1;
    const int64_t vals = (int64_t) 32 * hkv * 128;  // one page of one cache
    const int64_t dst0 = dst_page * vals;
    if (src_page < 0 || src_page >= n_pages_src) {
        // a page past the sequence's keys (or a bad page id, reported) becomes zeros: the prefill
        // reads whole 128-key tiles, and masked keys must hold finite values
        if (p * 32 < len && threadIdx.x == 0) report(status, kStatusBadIndex, kSitePrefillPage, src_page);
        for (int64_t i = (int64_t) threadIdx.x * 8; i < vals; i += (int64_t) blockDim.x * 8) {
            *reinterpret_cast<uint4 *>(k_out + dst0 + i) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(v_out + dst0 + i) = make_uint4(0, 0, 0, 0);
        }
        return;
    }
    const int64_t src0 = (int64_t) src_page * vals;
    for (int64_t i = (int64_t) threadIdx.x * 16; i < vals; i += (int64_t) blockDim.x * 16) {
#pragma unroll
        for (int kv = 0; kv < 2; kv++) {
            const int8_t *qs = (kv ? v_qs : k_qs) + src0 + i;
            const float d = __half2float((kv ? v_d : k_d)[(src0 + i) / 32]);
            const int4 w = *reinterpret_cast<const int4 *>(qs);
            const uint32_t ws[4] = {(uint32_t) w.x, (uint32_t) w.y, (uint32_t) w.z, (uint32_t) w.w};
            uint32_t h[8];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int8_t *bytes = reinterpret_cast<const int8_t *>(&ws[e]);
                const __half2 lo = __floats2half2_rn(d * (float) bytes[0], d * (float) bytes[1]);
                const __half2 hi = __floats2half2_rn(d * (float) bytes[2], d * (float) bytes[3]);
                h[2 * e] = *reinterpret_cast<const uint32_t *>(&lo);
                h[2 * e + 1] = *reinterpret_cast<const uint32_t *>(&hi);
            }
            __half *out = (kv ? v_out : k_out) + dst0 + i;
            *reinterpret_cast<uint4 *>(out) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4 *>(out + 8) = make_uint4(h[4], h[5], h[6], h[7]);
        }
    }
}

}  // namespace q8
}  // namespace lstk
