// kv_pages.cuh - device-side KV-cache bookkeeping for decode steps.
//
// The reference keeps the paged cache's bookkeeping on the host (KvCache, src/kv_cache.cpp:59-132):
// a LIFO stack of free 32-cell blocks, each sequence's block list in position order and its
// length. A decode step calls KvCache::alloc(seq, 1) for every running sequence, then uploads
// the cells, positions and tables. These kernels keep the same state in device memory and apply
// the same rules on the device, so a decode step (allocate, append, attend) needs no host round
// trip:
//   alloc_kernel       - counts[i] new tokens for each listed slot, in list order, exactly as
//                        sequential KvCache::alloc(slot, count) calls: new blocks are popped from
//                        the stack's top in slot order, and a slot whose blocks do not fit gets
//                        nothing (ok = 0) while later slots may still fit;
//   release_kernel     - KvCache::truncate_seq / remove_seq: blocks beyond the kept length go
//                        back to the stack (truncate pushes the last block first, remove pushes
//                        the list in order), and the high-water mark is recomputed.
#pragma once

#include "common.cuh"

namespace lstk {
namespace pages {

constexpr int kThreads = 1024;
constexpr int kBlock = 32;

struct State {
    uint32_t *free_blocks;  // stack of free block ids, [n_blocks]
    int32_t *free_top;      // [1] entries on the stack
    int32_t *block_tables;  // [n_slots][max_blocks]
    int32_t *seq_lens;      // [n_slots]
    int32_t *used_hwm;      // [1] one past the highest occupied cell
    int n_slots, max_blocks;
};

constexpr int kMaxSlots = 2048;  // slots per call (2 per thread)
constexpr int kPerThread = kMaxSlots / kThreads;

__device__ __forceinline__ int n_blocks_for(int len) { return (len + kBlock - 1) / kBlock; }

// Exclusive scan of v over the CTA (warp shuffles + one shared row of warp totals); *total gets the sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int *warp_sums, int *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = warp_sums[lane];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, off);
            if (lane >= off) w += y;
        }
        warp_sums[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
    *total = warp_sums[31];
    __syncthreads();  // warp_sums is reused by the next scan
    return before;
}

// KvCache::alloc(slots[i], counts[i]) for i = 0..n-1 in order (counts == nullptr: one token each).
// One CTA; slots distinct; n <= kMaxSlots. Slot i's tokens go to cells / positions at
// [sum(counts[0..i)), + counts[i]) in position order. A slot gets all its tokens or none: it fails
// (ok 0, its cells / positions -1, nothing taken) when the blocks it needs exceed what the stack
// holds after the slots before it, as KvCache::alloc does, or exceed its table row. When the
// tokens add up to more than max_tokens (the outputs' length) nothing is allocated, every ok is 0
// and the device status records it.
__global__ void __launch_bounds__(kThreads) alloc_kernel(State st, const int32_t *slots, const int32_t *counts, int n,
                                                         int max_tokens, int64_t *cells, int32_t *positions,
                                                         int32_t *ok, DeviceStatus *status) {
    __shared__ int s_len[kMaxSlots], s_tok[kMaxSlots], s_pop[kMaxSlots];
    __shared__ int warp_sums[32];
    __shared__ int s_serial;
    const int avail = *st.free_top;
    int slot[kPerThread], len[kPerThread], cnt[kPerThread], extra[kPerThread];
    int cnt_sum = 0, extra_sum = 0, bad = 0;
#pragma unroll
    for (int k = 0; k < kPerThread; k++) {
        const int i = threadIdx.x * kPerThread + k;  // consecutive items per thread keep list order
        slot[k] = -1, len[k] = 0, cnt[k] = 0, extra[k] = 0;
        if (i < n) {
            const int s = slots[i];
            const int c = counts ? counts[i] : 1;
            const bool valid = s >= 0 && s < st.n_slots && c >= 0;
            if (!valid) report(status, kStatusBadIndex, kSitePagesSlot, s);
            slot[k] = valid ? s : -1;
            len[k] = valid ? st.seq_lens[s] : 0;
            cnt[k] = valid ? c : 0;
            const int need = n_blocks_for(len[k] + cnt[k]);
            extra[k] = valid && need <= st.max_blocks ? need - n_blocks_for(len[k]) : -1;  // -1: cannot succeed
        }
        cnt_sum += cnt[k];
        extra_sum += max(extra[k], 0);
        bad |= extra[k] < 0;
    }
    int total_tokens, total_extra, n_bad;
    const int tok0 = block_exclusive_scan(cnt_sum, warp_sums, &total_tokens);
    const int pop0 = block_exclusive_scan(extra_sum, warp_sums, &total_extra);
    block_exclusive_scan(bad, warp_sums, &n_bad);
    if (total_tokens > max_tokens) {  // the outputs cannot hold the tokens: nothing is allocated
        if (threadIdx.x == 0) report(status, kStatusBadIndex, kSitePagesTokens, total_tokens);
        for (int i = threadIdx.x; i < n; i += kThreads) ok[i] = 0;
        return;
    }
    {
        int t = tok0, p = pop0;
#pragma unroll
        for (int k = 0; k < kPerThread; k++) {
            const int i = threadIdx.x * kPerThread + k;
            if (i < n) {
                s_len[i] = len[k];
                s_tok[i] = t;
                s_pop[i] = extra[k] >= 0 ? p : -1;
            }
            t += cnt[k];
            p += max(extra[k], 0);
        }
    }
    const bool serial = n_bad > 0 || total_extra > avail;
    __syncthreads();
    if (serial && threadIdx.x == 0) {
        // some slot fails: the decisions depend on one another, as in the sequential loop
        int taken = 0;
        // recompute each slot's extra from its length and count (s_pop only holds prefix sums)
        for (int i = 0; i < n; i++) {
            const int c = counts ? counts[i] : 1;
            const int s = slots[i];
            const bool valid = s >= 0 && s < st.n_slots && c >= 0;
            const int need = valid ? n_blocks_for(s_len[i] + c) : 0;
            const int e = valid && need <= st.max_blocks ? need - n_blocks_for(s_len[i]) : -1;
            if (e >= 0 && e <= avail - taken) {
                s_pop[i] = taken;
                taken += e;
            } else {
                s_pop[i] = -1;
            }
        }
        s_serial = taken;
    }
    __syncthreads();
    const int popped = serial ? s_serial : total_extra;
    // block tables: slot i's j-th new block is the (s_pop[i] + j)-th entry from the stack's top
#pragma unroll
    for (int k = 0; k < kPerThread; k++) {
        const int i = threadIdx.x * kPerThread + k;
        if (i < n && s_pop[i] >= 0) {
            int32_t *bt = st.block_tables + (int64_t) slot[k] * st.max_blocks;
            const int b0 = n_blocks_for(len[k]);
            for (int j = 0; j < extra[k]; j++) bt[b0 + j] = (int32_t) st.free_blocks[avail - 1 - s_pop[i] - j];
        }
    }
    __syncthreads();
    // cells and positions: one warp per slot, lanes over its tokens
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int hwm = 0;
    for (int i = warp; i < n; i += kThreads / 32) {
        const int s = slots[i];
        const int c_raw = counts ? counts[i] : 1;
        // An invalid item (slot out of range, negative count) reserved no output entries in the
        // token scan above, so it writes none: its s_tok is the next item's start.
        const int c = (s >= 0 && s < st.n_slots && c_raw >= 0) ? c_raw : 0;
        const bool got = s_pop[i] >= 0;
        const int l0 = s_len[i];
        const int64_t t0 = s_tok[i];
        if (c > 0) {
            const int32_t *bt = got ? st.block_tables + (int64_t) s * st.max_blocks : nullptr;
            for (int t = lane; t < c; t += 32) {
                const int p = l0 + t;
                const int64_t cell = got ? (int64_t) bt[p / kBlock] * kBlock + p % kBlock : -1;
                cells[t0 + t] = cell;
                positions[t0 + t] = got ? p : -1;
                hwm = max(hwm, (int) (cell + 1));
            }
        }
        if (lane == 0) {
            ok[i] = got ? 1 : 0;
            if (got) st.seq_lens[s] = l0 + c;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) hwm = max(hwm, __shfl_xor_sync(0xffffffffu, hwm, off));
    if (lane == 0 && hwm > 0) atomicMax(st.used_hwm, hwm);
    if (threadIdx.x == 0) *st.free_top = avail - popped;
}

// Keeps positions [0, keep) of `slot` (keep <= 0 removes the sequence). One CTA.
__global__ void __launch_bounds__(kThreads) release_kernel(State st, int slot, int keep) {
    __shared__ int hwm_s;
    if (threadIdx.x == 0) {
        int32_t *bt = st.block_tables + (int64_t) slot * st.max_blocks;
        const int len = st.seq_lens[slot];
        const int n_blocks = (len + kBlock - 1) / kBlock;
        int top = *st.free_top;
        if (keep <= 0) {
            for (int b = 0; b < n_blocks; b++) st.free_blocks[top++] = (uint32_t) bt[b];
            st.seq_lens[slot] = 0;
        } else if (keep < len) {
            const int keep_blocks = (keep + kBlock - 1) / kBlock;
            for (int b = n_blocks - 1; b >= keep_blocks; b--) st.free_blocks[top++] = (uint32_t) bt[b];
            st.seq_lens[slot] = keep;
        }
        *st.free_top = top;
        hwm_s = 0;
    }
    __syncthreads();
    // high-water mark: one past the highest occupied cell over every slot
    int hwm = 0;
    for (int s = threadIdx.x; s < st.n_slots; s += kThreads) {
        const int len = st.seq_lens[s];
        const int32_t *bt = st.block_tables + (int64_t) s * st.max_blocks;
        for (int b = 0; b * kBlock < len; b++) {
            const int last = min(kBlock, len - b * kBlock) - 1;
            hwm = max(hwm, bt[b] * kBlock + last + 1);
        }
    }
    atomicMax(&hwm_s, hwm);
    __syncthreads();
    if (threadIdx.x == 0) *st.used_hwm = hwm_s;
}

}  // namespace pages
}  // namespace lstk
