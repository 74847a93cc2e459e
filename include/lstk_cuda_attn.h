/*
 * lstk_cuda_attn.h - C ABI of the B200 (sm_100a) backend for the Qwen3 attention node of
 * ludehsar/localstack (`attn_block`, src/qwen3.cpp:128-171).
 *
 * The reference records these ggml ops per layer and lets ggml's scheduler run them
 * (src/engine.cpp:282-298):
 *     q/k = ggml_mul(ggml_rms_norm(.., eps), q_norm/k_norm)        src/qwen3.cpp:112-114, 139-140
 *     q/k = ggml_rope_ext(.., GGML_ROPE_TYPE_NEOX, base, 1, 0, 1) src/qwen3.cpp:143-146
 *     ggml_set_rows(kv.k[l] / kv.v[l], rows, kv_idxs)            src/qwen3.cpp:150-153
 *     ggml_flash_attn_ext(Q, K, V, mask, 1/sqrt(hd), 0, 0)       src/qwen3.cpp:155-167
 * Each entry point below replaces one group of those nodes. Everything is plain C: device
 * pointers and sizes, no allocation, no host synchronisation, stream-ordered on `stream`
 * (a cudaStream_t passed as void*; NULL = legacy default stream). Errors come back as a
 * negative status with a message in lstk_cuda_last_error(), mirroring the reference's
 * `bool + std::string &err` convention (src/kv_cache.h:47-48, src/engine.h:70-73).
 *
 * Cache layout (unchanged from the reference's KvCache, src/kv_cache.h:30-33 and
 * src/kv_cache.cpp:20-26): one f16 tensor per layer for K and one for V, each
 * [n_cells][n_head_kv][head_dim] (ggml [n_embd_gqa, size], ne0 innermost). Cell c holds one
 * token; cells are handed out in blocks (pages) of block_size = 32 consecutive cells, and a
 * sequence's block table lists its pages in position order (KvCache::seq_blocks,
 * src/kv_cache.h:41): position p lives in cell table[p / 32] * 32 + p % 32
 * (KvCache::alloc, src/kv_cache.cpp:59-83).
 */
#ifndef LSTK_CUDA_ATTN_H
#define LSTK_CUDA_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define LSTK_OK 0
#define LSTK_ERR_INVALID_ARG (-1)  /* null pointer, bad size or shape */
#define LSTK_ERR_CAPACITY (-2)     /* workspace too small, more work than a launch can hold */
#define LSTK_ERR_TIMEOUT (-3)      /* a kernel's bounded wait ran out (device status) */
#define LSTK_ERR_CUDA (-4)         /* a CUDA runtime/driver call failed */
#define LSTK_ERR_UNSUPPORTED (-5)  /* shape outside what the kernels implement */
#define LSTK_ERR_DEVICE_INDEX (-6) /* a kernel met an out-of-range cell, page or position */

/* Element types. */
#define LSTK_DTYPE_F32 0
#define LSTK_DTYPE_F16 1
#define LSTK_DTYPE_BF16 2

/* Geometry of one layer's K (or V) cache tensor. */
typedef struct lstk_kv_layout {
    int64_t n_cells;    /* KvCache::size; a multiple of block_size */
    int32_t n_head_kv;  /* Qwen3HParams::n_head_kv (src/qwen3.h:30) */
    int32_t head_dim;   /* Qwen3HParams::head_dim; the kernels implement 128 */
    int32_t block_size; /* KvCache::block_size (src/kv_cache.h:27); the kernels implement 32 */
} lstk_kv_layout;

/* Message for the last failed call on this host thread ("" if none). */
const char *lstk_cuda_last_error(void);

/* Synchronises `stream`, then reads and clears the device status word that kernels set when a
 * bounded wait times out or an index is out of range. Returns LSTK_OK, LSTK_ERR_TIMEOUT,
 * LSTK_ERR_DEVICE_INDEX or LSTK_ERR_CUDA. Status is per device and sticky until read. */
int lstk_cuda_status(void *stream);

/* ---- Bounded waits ----------------------------------------------------------------------------
 * (no counterpart in the reference, whose ggml ops never wait on other work). Every wait inside
 * the decode and prefill kernels is bounded: when one runs out, the kernel records LSTK_ERR_TIMEOUT
 * in the device status, lets its in-flight copies and tensor-core work finish, frees its tensor
 * memory and returns, so the context stays usable. This sets, for later decode / prefill launches
 * from the calling host thread (lstk_cuda_attn_decode, _decode_partial, _decode_static,
 * _prefill):
 *   pipeline_wait_ns  limit of each wait between the kernels' own warps (0 = the default, 4 s);
 *                     the waits that drain in-flight work before a kernel exits keep 4 s;
 *   start_flag        optional device int32: the kernels' loaders wait (bounded by
 *                     pipeline_wait_ns) until it is non-zero before their first load, to hold a
 *                     launched kernel until a producer outside its stream (another process or GPU
 *                     writing the pages) has published its inputs; NULL = no gate.
 * A CUDA graph captures the policy in force when it is captured. */
int lstk_cuda_set_wait_policy(uint64_t pipeline_wait_ns, const int32_t *start_flag);

/* ---- RoPE table -----------------------------------------------------------------------------
 * ggml builds the NEOX rotation per step (ggml_rope_cache_init for each position); the backend
 * reads the same values from a persistent table instead. Entry [p][i] = (cosf(t), sinf(t)) with
 * t = freq_scale * theta_i, theta_0 = p and theta_{i+1} = theta_i * powf(freq_base, -2/head_dim)
 * (repeated float multiplication), i < head_dim/2 - what ggml computes for the attn_block call
 * (freq_factors null, ext_factor 0, attn_factor 1; src/qwen3.cpp:141-146).
 * Host-side fill into a caller buffer of lstk_rope_table_bytes() bytes (float pairs). */
size_t lstk_rope_table_bytes(int32_t n_pos, int32_t head_dim);
int lstk_rope_table_fill(float *host_table, int32_t n_pos, int32_t head_dim, float freq_base, float freq_scale);

/* ---- K/V append: replaces rms_norm+mul (Q,K), rope_ext (Q,K) and the two set_rows -----------
 * (src/qwen3.cpp:139-153). For each of n_tokens tokens t:
 *   Q head rows: RMSNorm (sum of squares in double, as ggml's CPU rms_norm) * q_gamma, NEOX RoPE
 *                at positions[t] -> q_out[t][h][:] (f32 or f16);
 *   K head rows: the same with k_gamma -> f16 (round-to-nearest-even) into k_cache at cells[t];
 *   V head rows: -> f16 into v_cache at cells[t].
 * Inputs are token-major rows [T][H][D] (f32 or bf16) with a per-token stride in elements, so a
 * fused QKV projection output can be passed as three views; strides are whole 16-byte units
 * (multiples of 4 f32 / 8 bf16 elements) and all pointers 16-byte aligned. q_gamma / k_gamma may be NULL
 * (no QK-norm, as for Qwen2, src/qwen3.cpp:139-140). positions must be < rope_n_pos and cells
 * < n_cells; offending tokens are skipped and set LSTK_ERR_DEVICE_INDEX in the device status.
 * Every f32 operation is separately rounded, so the written f16 pages are bit-identical to a
 * CPU evaluation of the ggml op sequence with the same RoPE table. */
int lstk_cuda_kv_append(const lstk_kv_layout *layout, void *k_cache, void *v_cache, const void *q_in,
                        const void *k_in, const void *v_in, int32_t in_dtype, int64_t q_row_stride,
                        int64_t k_row_stride, int64_t v_row_stride, int32_t n_tokens, int32_t n_head,
                        const int32_t *positions, const int64_t *cells, const float *q_gamma, const float *k_gamma,
                        float eps, const float *rope_table, int32_t rope_n_pos, void *q_out, int32_t q_out_dtype,
                        void *stream);

/* ---- Paged decode: replaces flash_attn_ext for one new token per sequence --------------------
 * (src/qwen3.cpp:155-167 with n_tokens = 1 per sequence). Query b attends to positions
 * [0, seq_lens[b]) of its own sequence through block_tables[b][:] - the cells KvCache::fill_mask
 * leaves visible to the sequence's last token (src/kv_cache.cpp:140-150) - with
 * softmax(scale * q k^T) v, f16 K/V, f16-rounded Q for the dot (as ggml's CPU kernel rounds Q to
 * the K type) and f32 accumulation (GGML_PREC_F32, src/qwen3.cpp:167).
 *   q            [n_seqs][n_head][head_dim], f32 or f16
 *   block_tables [n_seqs][max_blocks_per_seq] int32 page ids (< n_cells / block_size)
 *   seq_lens     [n_seqs] int32, 0 <= len <= max_blocks_per_seq * block_size
 *   max_seq_len  host upper bound of seq_lens (sizes the launch; 0 = max_blocks * block_size)
 *   out          [n_seqs][n_head][head_dim] f32; a sequence with no keys gets zeros
 *   lse_out      optional [n_seqs][n_head] f32: natural-log sum of exp(scale * q k), -inf if empty
 *   n_ctas       0 = one CTA per SM; otherwise the split-K grid size (results agree within
 *                rounding for any value; identical for identical values)
 * Split-K: the page-groups of all sequences are cut into n_ctas equal contiguous ranges, each
 * CTA streams its range with TMA and emits per-piece (O, lse); a second kernel merges pieces by
 * log-sum-exp. n_head / n_head_kv must be 1..8. */
size_t lstk_cuda_attn_decode_workspace_size(int32_t n_seqs, int32_t n_head, int32_t n_head_kv, int32_t head_dim);
int lstk_cuda_attn_decode(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache, const void *q,
                          int32_t q_dtype, int32_t n_seqs, int32_t n_head, const int32_t *block_tables,
                          int32_t max_blocks_per_seq, const int32_t *seq_lens, int32_t max_seq_len, float scale,
                          float *out, float *lse_out, void *workspace, size_t workspace_bytes, int32_t n_ctas,
                          void *stream);

/* Decode over a key range only (one context split across GPUs, or any partial pass): every
 * sequence attends to its keys [kv_begin, min(kv_end, seq_lens[b])) - kv_begin a multiple of
 * block_size - with the same arguments and results as lstk_cuda_attn_decode otherwise; lse_out
 * gives the weights lstk_cuda_attn_merge needs to combine ranges. A sequence with no key in the
 * range gets zeros and lse -inf. */
int lstk_cuda_attn_decode_partial(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache,
                                  const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                                  const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *seq_lens,
                                  int32_t max_seq_len, int32_t kv_begin, int32_t kv_end, float scale, float *out,
                                  float *lse_out, void *workspace, size_t workspace_bytes, int32_t n_ctas,
                                  void *stream);

/* ---- Paged decode with no caller workspace (no counterpart in the reference) ----------------
 * Same computation, arguments and results as lstk_cuda_attn_decode, minus the workspace: the
 * split-K scratch is a fixed array compiled into this library (about 5.3 MiB, held on every
 * device that loads the library until the process exits). It is for callers that cannot
 * allocate device memory at the point where they decode - an engine whose memory is all handed
 * to its own pool up front, code running where cudaMalloc is not allowed or would stall the
 * pipeline, or a plain C/FFI host that only owns the tensors it passes in. This call allocates
 * nothing. Limits: n_seqs <= 1024 and n_ctas <= 160 (0 = one CTA per SM); larger requests fail
 * with LSTK_ERR_CAPACITY. The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture. All calls on a device
 * share the one array and it keeps the previous call's contents (nothing in it needs to start at
 * zero), so calls whose kernels overlap on the GPU - different streams without ordering between
 * them - race and give wrong results; order them on one stream. */
int lstk_cuda_attn_decode_static(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache,
                                 const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                                 const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *seq_lens,
                                 int32_t max_seq_len, float scale, float *out, float *lse_out, int32_t n_ctas,
                                 void *stream);

/* ---- Log-sum-exp merge of partial results over disjoint key ranges --------------------------
 * Used when one long context is split across GPUs (each GPU runs lstk_cuda_attn_decode over its
 * contiguous chunk of pages with lse_out). o_parts [n_parts][n_rows][head_dim] f32 (each
 * normalised by its own softmax sum), lse_parts [n_parts][n_rows] (natural log, -inf = empty).
 * Part r starts at o_parts + r * o_part_stride and lse_parts + r * lse_part_stride (elements;
 * 0 = densely packed, n_rows * head_dim and n_rows), so the parts can sit in one gathered buffer
 * of per-rank records [O | lse]. out [n_rows][head_dim]; lse_out optional [n_rows]. */
int lstk_cuda_attn_merge(const float *o_parts, const float *lse_parts, int32_t n_parts, int64_t n_rows,
                         int32_t head_dim, int64_t o_part_stride, int64_t lse_part_stride, float *out,
                         float *lse_out, void *stream);

/* ---- Device-side KV bookkeeping for serving steps ------------------------------------------
 * The state of KvCache (src/kv_cache.h:24-62) in caller-owned device memory: the LIFO stack of
 * free 32-cell blocks, and per sequence slot its block table (position order) and length; plus
 * the high-water mark. lstk_cuda_kv_alloc gives each listed slot (distinct slots, at most 2048)
 * counts[i] new tokens (counts NULL: one each), in list order, exactly as sequential
 * KvCache::alloc(slot, counts[i]) calls (src/kv_cache.cpp:59-83) would: new blocks are popped from
 * the stack's top in slot order; token t of slot i (position len + t) goes to cells / positions
 * [sum(counts[0..i)) + t] with cell = table[p / 32] * 32 + p % 32. A slot whose new blocks exceed
 * what the stack holds after the slots before it, or its table row, gets nothing: ok[i] = 0 and
 * its cells / positions are -1 (later slots may still fit, as with the reference). If the counts
 * add up to more than max_tokens, nothing is allocated, every ok is 0 and the device status
 * (lstk_cuda_status) reports LSTK_ERR_DEVICE_INDEX. lstk_cuda_kv_release is KvCache::truncate_seq
 * (keep > 0) / remove_seq (keep <= 0) (src/kv_cache.cpp:85-132): freed blocks go back on the
 * stack in the reference's order and the high-water mark is recomputed. The block_tables /
 * seq_lens arrays are the ones lstk_cuda_attn_decode and lstk_cuda_attn_prefill read, so a step
 * (allocate -> append -> attend) stays on the device and can be captured in a CUDA graph. Fill
 * free_blocks / free_top like KvCache::init (or a permuted free list) before use. */
typedef struct lstk_kv_pages {
    uint32_t *free_blocks;  /* [n_blocks] stack, top at free_blocks[*free_top - 1] */
    int32_t *free_top;      /* [1] */
    int32_t *block_tables;  /* [n_slots][max_blocks] */
    int32_t *seq_lens;      /* [n_slots] */
    int32_t *used_hwm;      /* [1] */
    int32_t n_slots;
    int32_t max_blocks;
    int32_t block_size;     /* 32 */
} lstk_kv_pages;
int lstk_cuda_kv_alloc(const lstk_kv_pages *state, const int32_t *slots, const int32_t *counts, int32_t n,
                       int32_t max_tokens, int64_t *cells, int32_t *positions, int32_t *ok, void *stream);
int lstk_cuda_kv_release(const lstk_kv_pages *state, int32_t slot, int32_t keep, void *stream);

/* ---- q8_0 KV cache (the reference's planned option, docs/plan.md:389-395; not built there) ----
 * The values of ggml's block_q8_0 (per 32 consecutive values of a row: d = amax / 127 kept as
 * f16, q = round-to-nearest-even(x / d) as int8 - quantize_row_q8_0's ARM form) in two planes per
 * cache, so every 128-byte row stays 16-byte aligned for TMA: qs int8 [n_cells][n_head_kv][128]
 * and d f16 [n_cells][n_head_kv][4]. layout describes the cache as for f16 (head_dim 128,
 * block_size 32); n_head_kv must be even for the decode (16-byte scale rows). Planes 16-byte
 * aligned.
 *
 * lstk_cuda_kv_append_q8: lstk_cuda_kv_append with the K and V rows quantised into the planes
 * (bit-identical to quantising the f16 path's f32 rows). lstk_cuda_attn_decode_q8:
 * lstk_cuda_attn_decode over q8_0 planes with ggml's CPU semantics for a q8_0 cache - the query
 * row quantised to q8_0, each score sum_b (d_k,b * d_q,b) * (integer dot of block b), f32
 * accumulation of the dequantised V (the softmax as in lstk_cuda_attn_decode). Same workspace
 * (lstk_cuda_attn_decode_workspace_size). */
int lstk_cuda_kv_append_q8(const lstk_kv_layout *layout, int8_t *k_qs, void *k_d, int8_t *v_qs, void *v_d,
                           const void *q_in, const void *k_in, const void *v_in, int32_t in_dtype,
                           int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride, int32_t n_tokens,
                           int32_t n_head, const int32_t *positions, const int64_t *cells, const float *q_gamma,
                           const float *k_gamma, float eps, const float *rope_table, int32_t rope_n_pos, void *q_out,
                           int32_t q_out_dtype, void *stream);
int lstk_cuda_attn_decode_q8(const lstk_kv_layout *layout, const int8_t *k_qs, const void *k_d, const int8_t *v_qs,
                             const void *v_d, const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                             const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *seq_lens,
                             int32_t max_seq_len, float scale, float *out, float *lse_out, void *workspace,
                             size_t workspace_bytes, int32_t n_ctas, void *stream);
/* Prefill over a q8_0 cache: the pages the call reads (kv_lens[b] keys of each sequence through
 * its block table) are dequantised (d * q rounded once to f16) into a compact f16 cache in
 * `scratch` with dense block tables, and lstk_cuda_attn_prefill runs on it (same arguments and
 * results; its `workspace` as for the f16 call). The scratch holds n_seqs * max_blocks_per_seq
 * pages of K and V: lstk_cuda_q8_prefill_scratch_size bytes, 256-byte aligned. */
size_t lstk_cuda_q8_prefill_scratch_size(int32_t n_seqs, int32_t max_blocks_per_seq, int32_t n_head_kv);
int lstk_cuda_attn_prefill_q8(const lstk_kv_layout *layout, const int8_t *k_qs, const void *k_d, const int8_t *v_qs,
                              const void *v_d, const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                              const int32_t *q_seq_start, int32_t max_q_len, int64_t total_tokens,
                              const int32_t *q_pos0, const int32_t *kv_lens, const int32_t *block_tables,
                              int32_t max_blocks_per_seq, float scale, float *out, void *workspace,
                              size_t workspace_bytes, void *scratch, size_t scratch_bytes, void *stream);
/* Byte moves between ggml's block_q8_0 rows (n_rows rows of 128 values = 4 blocks of 34 bytes:
 * f16 d, then 32 int8) and the planes (qs [n_rows][128], d [n_rows][4]); n_rows = n_cells *
 * n_head_kv for a whole cache. For a cache kept as a ggml q8_0 tensor. Pointers 2-byte aligned. */
int lstk_cuda_q8_from_ggml_blocks(const void *blocks, int64_t n_rows, int8_t *qs, void *d, void *stream);
int lstk_cuda_q8_to_ggml_blocks(const int8_t *qs, const void *d, int64_t n_rows, void *blocks, void *stream);

/* ---- One context over several processes / GPUs: peer-memory exchange and merge -------------
 * (no counterpart in the reference, which runs in one process). Rank r of R decodes its
 * contiguous chunk of a sequence's pages with lstk_cuda_attn_decode(..., lse_out) and then calls
 * lstk_cuda_attn_exchange_merge, which stores its rows (O, lse) straight into every rank's
 * mailbox over NVLink (CUDA IPC mappings, plain stores), raises per-row flags, waits for the
 * other ranks' flags (bounded by wait_ns, 0 = 1 s; on timeout LSTK_ERR_TIMEOUT in the device
 * status and zero rows) and merges the R records by log-sum-exp into out [n_rows][128] (and
 * lse_out, natural log, optional). Set-up per rank: lstk_cuda_mailbox_alloc (on the current
 * device; zeroed; 64-byte IPC handle out), share the handles through any host channel,
 * lstk_cuda_mailbox_open each peer's, and place the R pointers (own at [rank]) in a device
 * array `mailboxes`. At most 128 ranks (LSTK_ERR_UNSUPPORTED beyond). Every rank must make the
 * same sequence of calls with the same n_rows; the
 * calls advance an epoch kept in the mailbox, so they can be replayed from a CUDA graph. */
size_t lstk_cuda_mailbox_bytes(int32_t n_ranks, int64_t n_rows, int32_t head_dim);
/* The decode of this rank's chunk and the exchange-merge in one call, without the separate merge
 * launch: lstk_cuda_attn_decode's arguments, plus the mailboxes / rank / n_ranks / wait_ns of
 * lstk_cuda_attn_exchange_merge (mailboxes sized for n_seqs * n_head rows). The decode's own
 * combine kernel runs the exchange protocol on each output row as it finishes it, so out and
 * lse_out receive the rows merged over all ranks. lse_out is required (it also carries the
 * local lse of rows the split kernel finishes alone). Limits: n_seqs * ceil(n_head_kv / 4) <= 64
 * (one mailbox epoch counter per combine CTA; LSTK_ERR_CAPACITY beyond) and n_ranks <= 256. A
 * mailbox set serves either this call or lstk_cuda_attn_exchange_merge, not both (they map rows
 * to epoch counters differently). */
int lstk_cuda_attn_decode_exchange(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache,
                                   const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                                   const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *seq_lens,
                                   int32_t max_seq_len, float scale, float *out, float *lse_out, void *workspace,
                                   size_t workspace_bytes, int32_t n_ctas, void *const *mailboxes, int32_t rank,
                                   int32_t n_ranks, uint64_t wait_ns, void *stream);
int lstk_cuda_mailbox_alloc(size_t bytes, void **mailbox, void *ipc_handle);
int lstk_cuda_mailbox_free(void *mailbox);
int lstk_cuda_mailbox_open(const void *ipc_handle, void **peer_mailbox);
int lstk_cuda_mailbox_close(void *peer_mailbox);
int lstk_cuda_attn_exchange_merge(void *const *mailboxes, int32_t rank, int32_t n_ranks, const float *local_o,
                                  const float *local_lse, int64_t n_rows, int32_t head_dim, uint64_t wait_ns,
                                  float *out, float *lse_out, void *stream);

/* ---- Paged causal prefill: replaces flash_attn_ext for a chunk of prompt tokens -------------
 * (src/qwen3.cpp:155-167 with n_tokens > 1). Sequence b's query tokens are rows
 * [q_seq_start[b], q_seq_start[b+1]) of q, at positions q_pos0[b], q_pos0[b]+1, ...; query
 * token i attends to positions [0, min(pos_i + 1, kv_lens[b])) of its sequence (causal), read
 * through block_tables[b][:] - the visibility KvCache::fill_mask grants. K/V must already hold
 * the chunk (lstk_cuda_kv_append first, as attn_block writes set_rows before flash_attn_ext).
 *   q            [total_tokens][n_head][head_dim], f16 (the tensor-core operand type) or f32
 *                (converted into the workspace first)
 *   q_seq_start  [n_seqs + 1] int32 device; max_q_len = host upper bound of any sequence's rows.
 *                A sequence whose rows are not inside [0, total_tokens) (or whose start exceeds
 *                its end) is skipped - nothing is read or written for it - and lstk_cuda_status
 *                reports LSTK_ERR_DEVICE_INDEX (site 23, detail = the sequence index)
 *   out          [total_tokens][n_head][head_dim] f32
 * Computed with tcgen05 tensor-core MMAs (f16 x f16 -> f32 in tensor memory) on 128-row query
 * tiles and 128-key tiles fed by TMA from the scattered pages. The workspace is sized by
 * lstk_cuda_attn_prefill_workspace_size from the same shape arguments (today: the f16 copy of
 * f32 queries; 0 bytes for f16 queries). n_head / n_head_kv must be 1, 2, 4 or 8. */
size_t lstk_cuda_attn_prefill_workspace_size(int32_t n_seqs, int32_t n_head, int32_t n_head_kv, int32_t head_dim,
                                             int32_t max_q_len, int32_t max_blocks_per_seq, int64_t total_tokens,
                                             int32_t q_dtype);
int lstk_cuda_attn_prefill(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache, const void *q,
                           int32_t q_dtype, int32_t n_seqs, int32_t n_head, const int32_t *q_seq_start,
                           int32_t max_q_len, int64_t total_tokens, const int32_t *q_pos0, const int32_t *kv_lens,
                           const int32_t *block_tables, int32_t max_blocks_per_seq, float scale, float *out,
                           void *workspace, size_t workspace_bytes, void *stream);

/* ---- Projections: replace attn_block's mul_mat nodes and the input RMSNorm ------------------
 * (src/qwen3.cpp:117-120 proj(), called at :135-138 for Wq / Wk / Wv and at :169 for Wo; the
 * residual add of :170; rms(x, attn_norm) of :112-114 / :134).
 * lstk_cuda_proj: out[m][n] = sum_k x[m][k] * w[n][k] (+ residual[m][n]) on the tcgen05 tensor
 *   cores. x [m][ldx] bf16 activations; w [n][ldw] bf16, a weight in ggml's mul_mat layout (ne0 = k
 *   contiguous, one output row per row of w: a fused Wq|Wk|Wv is the three weights stacked);
 *   residual optional [m][ldr] bf16; out [m][ldo] bf16 or f32 (out_dtype). f32 accumulation; the
 *   residual is added in f32 and the sum rounded once. Row strides are whole 16-byte units and
 *   pointers 16-byte aligned; k > 0. out must not overlap x or w (it may be the residual itself).
 * lstk_cuda_rms_norm: y[r][:] = x[r][:] / sqrt(mean(x[r][:]^2) + eps) * gamma (gamma NULL = 1),
 *   x bf16 or f32, y bf16; f32 sums. cols a multiple of 8 (bf16) or 4 (f32).
 * lstk_cuda_to_bf16: y = bf16(x) for a [rows][cols] f32 block (the f32 attention output entering the
 *   bf16 Wo projection). */
int lstk_cuda_proj(const void *x, int64_t ldx, const void *w, int64_t ldw, int32_t m, int32_t n, int32_t k,
                   const void *residual, int64_t ldr, void *out, int32_t out_dtype, int64_t ldo, void *stream);
/* lstk_cuda_proj with a caller workspace: when the 128 x 256 output tiles would leave most SMs
 * idle (small m: the per-GPU shapes of a sharded batch), K is split over the idle SMs into f32
 * slices of the workspace and summed in slice order (plus the residual, rounded once) by a second
 * kernel. lstk_cuda_proj_workspace_size gives the bytes that split needs on the current device (0:
 * no split for this shape; a smaller workspace, or NULL, runs unsplit). Same results up to f32
 * summation order. */
size_t lstk_cuda_proj_workspace_size(int32_t m, int32_t n, int32_t k);
int lstk_cuda_proj_ws(const void *x, int64_t ldx, const void *w, int64_t ldw, int32_t m, int32_t n, int32_t k,
                      const void *residual, int64_t ldr, void *out, int32_t out_dtype, int64_t ldo, void *workspace,
                      size_t workspace_bytes, void *stream);
int lstk_cuda_rms_norm(const void *x, int32_t x_dtype, int64_t ldx, const float *gamma, float eps, void *y,
                       int64_t ldy, int32_t rows, int32_t cols, void *stream);
int lstk_cuda_to_bf16(const float *x, int64_t ldx, void *y, int64_t ldy, int32_t rows, int32_t cols, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LSTK_CUDA_ATTN_H */
