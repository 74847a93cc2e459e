/*
 * lstk_kv_cache.h - host-side page/cell bookkeeping of the paged KV cache, with the semantics of
 * the reference's KvCache (src/kv_cache.h:24-62, src/kv_cache.cpp:59-150), plus the export the
 * device kernels consume: per-sequence block tables.
 *
 * In a drop-in deployment the reference keeps its own KvCache unchanged and only converts
 * KvCache::seq_blocks / seq_len into the int32 tables of lstk_kv_cache_block_tables' format.
 * This C ABI lets the backend run standalone with identical bookkeeping.
 * Not thread-safe, like the reference's Engine (src/engine.h:65).
 */
#ifndef LSTK_KV_CACHE_H
#define LSTK_KV_CACHE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lstk_kv_cache lstk_kv_cache;

/* KvCache::init (src/kv_cache.cpp:11-42), bookkeeping part: `size` cells in blocks of
 * `block_size`, all free, stack ordered so block 0 is handed out first. NULL on bad sizes. */
lstk_kv_cache *lstk_kv_cache_create(uint32_t size, uint32_t block_size);
void lstk_kv_cache_destroy(lstk_kv_cache *kv);

/* Replaces the free-block stack (KvCache::free_blocks, src/kv_cache.h:39); the last entry is
 * handed out first. Used to realise a seeded page permutation through the normal allocator. */
int lstk_kv_cache_set_free_blocks(lstk_kv_cache *kv, const uint32_t *blocks, int32_t n);

/* KvCache::alloc (src/kv_cache.cpp:59-83): reserves cells for the next n_tokens positions of
 * `seq`. LSTK_OK, or LSTK_ERR_CAPACITY (nothing allocated) when free blocks run out. */
int lstk_kv_cache_alloc(lstk_kv_cache *kv, int32_t seq, int32_t n_tokens, int64_t *cells, int32_t *positions);

/* KvCache::remove_seq (src/kv_cache.cpp:85-103). */
void lstk_kv_cache_remove_seq(lstk_kv_cache *kv, int32_t seq);
/* KvCache::truncate_seq (src/kv_cache.cpp:105-132). */
void lstk_kv_cache_truncate_seq(lstk_kv_cache *kv, int32_t seq, int32_t keep);
/* KvCache::length (src/kv_cache.cpp:134-137). */
int32_t lstk_kv_cache_length(const lstk_kv_cache *kv, int32_t seq);
/* KvCache::used_hwm (src/kv_cache.h:44). */
uint32_t lstk_kv_cache_used_hwm(const lstk_kv_cache *kv);
/* KvCache::n_free_cells (src/kv_cache.h:58). */
uint32_t lstk_kv_cache_n_free_cells(const lstk_kv_cache *kv);
/* Copies of KvCache::free_blocks / seq_blocks[seq] (src/kv_cache.h:39-41); return the counts. */
int32_t lstk_kv_cache_free_blocks(const lstk_kv_cache *kv, uint32_t *out, int32_t cap);
int32_t lstk_kv_cache_seq_blocks(const lstk_kv_cache *kv, int32_t seq, uint32_t *out, int32_t cap);
/* Copies of KvCache::cell_seq / cell_pos (src/kv_cache.h:36-37), `size` entries each. */
void lstk_kv_cache_cells(const lstk_kv_cache *kv, int32_t *cell_seq, int32_t *cell_pos);

/* The device view: block_tables[i][:] = seq_blocks[seqs[i]] (zero-padded to max_blocks) and
 * seq_lens[i] = length(seqs[i]). This is what replaces fill_mask + the dense n_kv scan: the
 * kernels read positions [0, seq_len) through the table. LSTK_ERR_CAPACITY if a sequence has
 * more than max_blocks blocks in use. */
int lstk_kv_cache_block_tables(const lstk_kv_cache *kv, const int32_t *seqs, int32_t n_seqs, int32_t max_blocks,
                               int32_t *block_tables, int32_t *seq_lens);

/* KvCache::fill_mask (src/kv_cache.cpp:140-150): mask[i][j] = 0 (f16) when cell j belongs to
 * `seq` at a position <= pos[i], else -inf. Kept for equivalence checks against the tables. */
void lstk_kv_cache_fill_mask(const lstk_kv_cache *kv, int32_t seq, const int32_t *pos, int32_t n_tokens,
                             int32_t n_kv, uint16_t *mask);

/* Engine::n_kv_for (src/engine.cpp:193-196): the reference's dense scan length, the cache
 * high-water mark plus new tokens padded to 256, at least 256, at most the cache size. */
int32_t lstk_n_kv_for(uint32_t cache_size, int32_t n_total);

#ifdef __cplusplus
}
#endif

#endif /* LSTK_KV_CACHE_H */
