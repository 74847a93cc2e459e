// kv_cache_host.cpp - host-side page/cell bookkeeping for the paged KV cache.
//
// The reference keeps this state in KvCache (src/kv_cache.h:24-62, src/kv_cache.cpp:59-150) and
// its interface stays unchanged when this backend is plugged in. This file restates the same
// rules in a ggml-free class so the backend can run standalone (benchmarks, tests) and so that
// the one thing the kernels need from it - a sequence's block table - has a home:
//   - cells are handed out in blocks of `block_size`; free blocks form a stack and `alloc` pops
//     from the back (KvCache::alloc, src/kv_cache.cpp:59-83);
//   - position p of a sequence lives in cell blocks[p / bs] * bs + p % bs;
//   - remove_seq / truncate_seq return whole blocks to the stack and recompute the high-water
//     mark (src/kv_cache.cpp:85-132);
//   - fill_mask gives the dense 0/-inf view the reference's attention scans
//     (src/kv_cache.cpp:140-150); the kernels use the block table + causal rule instead, and the
//     tests check the two agree.
#include "lstk_cuda_attn.h"
#include "lstk_kv_cache.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <unordered_map>
#include <vector>

struct lstk_kv_cache {
    uint32_t size = 0;
    uint32_t block_size = 32;
    std::vector<int32_t> cell_seq;
    std::vector<int32_t> cell_pos;
    std::vector<uint32_t> free_blocks;
    std::unordered_map<int32_t, std::vector<uint32_t>> seq_blocks;
    std::unordered_map<int32_t, int32_t> seq_len;
    uint32_t used_hwm = 0;

    void recompute_hwm() {
        used_hwm = 0;
        for (uint32_t c = size; c > 0; c--)
            if (cell_seq[c - 1] >= 0) {
                used_hwm = c;
                break;
            }
    }
};

namespace {

uint16_t f16_bits(float x) {
    // 0 and -inf, the only values fill_mask writes.
    if (x == 0.0f) return 0x0000;
    return 0xFC00;
}

}  // namespace

extern "C" {

lstk_kv_cache *lstk_kv_cache_create(uint32_t size, uint32_t block_size) {
    if (size == 0 || block_size == 0 || size % block_size != 0) return nullptr;
    lstk_kv_cache *kv = new lstk_kv_cache();
    kv->size = size;
    kv->block_size = block_size;
    kv->cell_seq.assign(size, -1);
    kv->cell_pos.assign(size, -1);
    // Reverse order so the first pop hands out block 0 (low blocks first, small high-water mark).
    for (uint32_t b = size / block_size; b > 0; b--) kv->free_blocks.push_back(b - 1);
    return kv;
}

void lstk_kv_cache_destroy(lstk_kv_cache *kv) { delete kv; }

int lstk_kv_cache_set_free_blocks(lstk_kv_cache *kv, const uint32_t *blocks, int32_t n) {
    if (kv == nullptr || (n > 0 && blocks == nullptr) || n < 0) return LSTK_ERR_INVALID_ARG;
    for (int32_t i = 0; i < n; i++)
        if (blocks[i] >= kv->size / kv->block_size) return LSTK_ERR_INVALID_ARG;
    kv->free_blocks.assign(blocks, blocks + n);
    return LSTK_OK;
}

int lstk_kv_cache_alloc(lstk_kv_cache *kv, int32_t seq, int32_t n_tokens, int64_t *cells, int32_t *positions) {
    if (kv == nullptr || n_tokens < 0 || (n_tokens > 0 && (cells == nullptr || positions == nullptr)))
        return LSTK_ERR_INVALID_ARG;
    int32_t &len = kv->seq_len[seq];
    std::vector<uint32_t> &blocks = kv->seq_blocks[seq];
    const uint32_t bs = kv->block_size;
    const uint32_t have = (uint32_t) blocks.size() * bs;
    const uint32_t need = (uint32_t) len + (uint32_t) n_tokens;
    const uint32_t extra = need > have ? (need - have + bs - 1) / bs : 0;
    if (extra > kv->free_blocks.size()) return LSTK_ERR_CAPACITY;
    for (uint32_t i = 0; i < extra; i++) {
        blocks.push_back(kv->free_blocks.back());
        kv->free_blocks.pop_back();
    }
    for (int32_t i = 0; i < n_tokens; i++) {
        const uint32_t p = (uint32_t) len;
        const uint32_t cell = blocks[p / bs] * bs + p % bs;
        kv->cell_seq[cell] = seq;
        kv->cell_pos[cell] = len;
        cells[i] = cell;
        positions[i] = len;
        kv->used_hwm = std::max(kv->used_hwm, cell + 1);
        len++;
    }
    return LSTK_OK;
}

void lstk_kv_cache_remove_seq(lstk_kv_cache *kv, int32_t seq) {
    if (kv == nullptr) return;
    auto it = kv->seq_blocks.find(seq);
    if (it == kv->seq_blocks.end()) return;
    const uint32_t bs = kv->block_size;
    for (uint32_t b : it->second) {
        std::fill(kv->cell_seq.begin() + (size_t) b * bs, kv->cell_seq.begin() + (size_t) (b + 1) * bs, -1);
        std::fill(kv->cell_pos.begin() + (size_t) b * bs, kv->cell_pos.begin() + (size_t) (b + 1) * bs, -1);
        kv->free_blocks.push_back(b);
    }
    kv->seq_blocks.erase(it);
    kv->seq_len.erase(seq);
    kv->recompute_hwm();
}

void lstk_kv_cache_truncate_seq(lstk_kv_cache *kv, int32_t seq, int32_t keep) {
    if (kv == nullptr) return;
    auto it = kv->seq_blocks.find(seq);
    if (it == kv->seq_blocks.end()) return;
    if (keep <= 0) {
        lstk_kv_cache_remove_seq(kv, seq);
        return;
    }
    std::vector<uint32_t> &blocks = it->second;
    int32_t &len = kv->seq_len[seq];
    if (keep >= len) return;
    const uint32_t bs = kv->block_size;
    for (int32_t p = keep; p < len; p++) {
        const uint32_t cell = blocks[(uint32_t) p / bs] * bs + (uint32_t) p % bs;
        kv->cell_seq[cell] = -1;
        kv->cell_pos[cell] = -1;
    }
    const size_t keep_blocks = ((size_t) keep + bs - 1) / bs;
    while (blocks.size() > keep_blocks) {
        kv->free_blocks.push_back(blocks.back());
        blocks.pop_back();
    }
    len = keep;
    kv->recompute_hwm();
}

int32_t lstk_kv_cache_length(const lstk_kv_cache *kv, int32_t seq) {
    if (kv == nullptr) return 0;
    auto it = kv->seq_len.find(seq);
    return it == kv->seq_len.end() ? 0 : it->second;
}

uint32_t lstk_kv_cache_used_hwm(const lstk_kv_cache *kv) { return kv ? kv->used_hwm : 0; }

uint32_t lstk_kv_cache_n_free_cells(const lstk_kv_cache *kv) {
    return kv ? (uint32_t) kv->free_blocks.size() * kv->block_size : 0;
}

int32_t lstk_kv_cache_free_blocks(const lstk_kv_cache *kv, uint32_t *out, int32_t cap) {
    if (kv == nullptr) return 0;
    const int32_t n = (int32_t) kv->free_blocks.size();
    for (int32_t i = 0; i < n && i < cap; i++) out[i] = kv->free_blocks[i];
    return n;
}

int32_t lstk_kv_cache_seq_blocks(const lstk_kv_cache *kv, int32_t seq, uint32_t *out, int32_t cap) {
    if (kv == nullptr) return 0;
    auto it = kv->seq_blocks.find(seq);
    if (it == kv->seq_blocks.end()) return 0;
    const int32_t n = (int32_t) it->second.size();
    for (int32_t i = 0; i < n && i < cap; i++) out[i] = it->second[i];
    return n;
}

void lstk_kv_cache_cells(const lstk_kv_cache *kv, int32_t *cell_seq, int32_t *cell_pos) {
    if (kv == nullptr) return;
    std::memcpy(cell_seq, kv->cell_seq.data(), sizeof(int32_t) * kv->size);
    std::memcpy(cell_pos, kv->cell_pos.data(), sizeof(int32_t) * kv->size);
}

int lstk_kv_cache_block_tables(const lstk_kv_cache *kv, const int32_t *seqs, int32_t n_seqs, int32_t max_blocks,
                               int32_t *block_tables, int32_t *seq_lens) {
    if (kv == nullptr || n_seqs < 0 || max_blocks <= 0 || (n_seqs > 0 && (!seqs || !block_tables || !seq_lens)))
        return LSTK_ERR_INVALID_ARG;
    for (int32_t i = 0; i < n_seqs; i++) {
        int32_t *row = block_tables + (size_t) i * max_blocks;
        auto it = kv->seq_blocks.find(seqs[i]);
        const int32_t len = lstk_kv_cache_length(kv, seqs[i]);
        const int32_t nb = it == kv->seq_blocks.end() ? 0 : (int32_t) it->second.size();
        const int32_t used = (len + (int32_t) kv->block_size - 1) / (int32_t) kv->block_size;
        if (used > max_blocks) return LSTK_ERR_CAPACITY;
        for (int32_t j = 0; j < max_blocks; j++) row[j] = j < nb ? (int32_t) it->second[j] : 0;
        seq_lens[i] = len;
    }
    return LSTK_OK;
}

void lstk_kv_cache_fill_mask(const lstk_kv_cache *kv, int32_t seq, const int32_t *pos, int32_t n_tokens,
                             int32_t n_kv, uint16_t *mask) {
    if (kv == nullptr) return;
    const uint16_t zero = f16_bits(0.0f), neg_inf = f16_bits(-INFINITY);
    for (int32_t i = 0; i < n_tokens; i++) {
        uint16_t *row = mask + (size_t) i * n_kv;
        for (int32_t j = 0; j < n_kv; j++) {
            const bool visible = (uint32_t) j < kv->size && kv->cell_seq[j] == seq && kv->cell_pos[j] <= pos[i];
            row[j] = visible ? zero : neg_inf;
        }
    }
}

int32_t lstk_n_kv_for(uint32_t cache_size, int32_t n_total) {
    const int32_t padded = (n_total + 255) / 256 * 256;
    return std::min<int32_t>((int32_t) cache_size, std::max<int32_t>(256, padded));
}

}  // extern "C"
