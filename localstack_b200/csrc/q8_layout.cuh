// q8_layout.cuh - conversion between ggml's block_q8_0 rows and the q8_0 planes of the cache.
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

}  // namespace q8
}  // namespace lstk
