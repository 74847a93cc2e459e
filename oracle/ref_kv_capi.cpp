// C entry points over the reference's own KvCache (src/kv_cache.h:24-62), compiled unchanged
// from the reference sources against the ggml stand-in in ref_shim/. Test infrastructure only:
// it exists so tests can drive the reference bookkeeping (alloc, remove_seq, truncate_seq,
// fill_mask, src/kv_cache.cpp:59-150) through ctypes and compare the product's page tables
// and masks with it. Built into oracle/_ref/ by oracle/Makefile; never shipped.
#include "kv_cache.h"

#include <cstring>
#include <string>

extern "C" {

void *refkv_create(uint32_t n_layer, uint32_t n_embd_gqa, uint32_t size) {
    KvCache *kv = new KvCache();
    std::string err;
    if (!kv->init(nullptr, n_layer, n_embd_gqa, n_embd_gqa, size, GGML_TYPE_F16, err)) {
        delete kv;
        return nullptr;
    }
    return kv;
}

void refkv_destroy(void *h) { delete (KvCache *) h; }

// Seeds the free-block stack in a caller-given order (pop_back hands out the last entry first),
// the way a permuted page placement is realised through the reference's own allocator.
void refkv_set_free_blocks(void *h, const uint32_t *blocks, int n) {
    KvCache *kv = (KvCache *) h;
    kv->free_blocks.assign(blocks, blocks + n);
}

int refkv_alloc(void *h, int32_t seq, int n_tokens, int64_t *cells, int32_t *positions) {
    KvCache *kv = (KvCache *) h;
    std::vector<int64_t> c;
    std::vector<int32_t> p;
    if (!kv->alloc(seq, n_tokens, c, p)) return 0;
    std::memcpy(cells, c.data(), sizeof(int64_t) * n_tokens);
    std::memcpy(positions, p.data(), sizeof(int32_t) * n_tokens);
    return 1;
}

void refkv_remove_seq(void *h, int32_t seq) { ((KvCache *) h)->remove_seq(seq); }
void refkv_truncate_seq(void *h, int32_t seq, int32_t keep) { ((KvCache *) h)->truncate_seq(seq, keep); }
int32_t refkv_length(void *h, int32_t seq) { return ((KvCache *) h)->length(seq); }
uint32_t refkv_used_hwm(void *h) { return ((KvCache *) h)->used_hwm; }
uint32_t refkv_n_free_cells(void *h) { return ((KvCache *) h)->n_free_cells(); }

void refkv_cells(void *h, int32_t *cell_seq, int32_t *cell_pos) {
    KvCache *kv = (KvCache *) h;
    std::memcpy(cell_seq, kv->cell_seq.data(), sizeof(int32_t) * kv->size);
    std::memcpy(cell_pos, kv->cell_pos.data(), sizeof(int32_t) * kv->size);
}

int refkv_free_blocks(void *h, uint32_t *out, int cap) {
    KvCache *kv = (KvCache *) h;
    const int n = (int) kv->free_blocks.size();
    for (int i = 0; i < n && i < cap; i++) out[i] = kv->free_blocks[i];
    return n;
}

int refkv_seq_blocks(void *h, int32_t seq, uint32_t *out, int cap) {
    KvCache *kv = (KvCache *) h;
    auto it = kv->seq_blocks.find(seq);
    if (it == kv->seq_blocks.end()) return 0;
    const int n = (int) it->second.size();
    for (int i = 0; i < n && i < cap; i++) out[i] = it->second[i];
    return n;
}

void refkv_fill_mask(void *h, int32_t seq, const int32_t *pos, int n_tokens, int n_kv, uint16_t *mask) {
    ((KvCache *) h)->fill_mask(seq, pos, n_tokens, n_kv, mask);
}

}  // extern "C"
