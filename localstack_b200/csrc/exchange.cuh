// exchange.cuh - exchange-and-merge of KV-split decode partials across GPUs over peer memory.
//
// One long context can be split across R processes (one GPU each): rank r decodes a contiguous
// chunk of the sequence's pages and gets, per output row (query head), O_r (normalised) and
// lse_r (natural log). The merged row is sum_r e^(lse_r - M) O_r / sum_r e^(lse_r - M).
//
// Instead of a library all-gather followed by a merge launch, one kernel per rank does both:
// every rank owns a "mailbox" in its own HBM that the other ranks can write through CUDA IPC
// mappings (plain peer stores over NVLink; no multicast). On rank s, the CTA owning a row
//   1. stores the row (O_s, lse_s) into slot s of every rank's mailbox (its own included),
//      release-stores the row's flag = epoch in every mailbox;
//   2. waits until the flags of all R sources for that row in its own mailbox equal the epoch
//      (acquire loads, bounded by wait_ns; on timeout it records LSTK_ERR_TIMEOUT in the device
//      status and writes zeros);
//   3. merges the R records of its own mailbox into out / lse_out.
// Epochs come from per-CTA counters in the mailbox header (CTA b of every call owns the same rows
// and advances its own counter), so the kernel can be replayed from a CUDA graph. Records and flags are double-banked by epoch
// parity: a rank can be at most one call ahead of a peer (it waits for that peer's record of the
// current call before returning), so it never overwrites a bank the peer is still reading.
#pragma once

#include "common.cuh"

namespace lstk {
namespace exchange {

constexpr int kThreads = 128;  // thread = one of the 128 dims of a row
constexpr int kD = 128;
constexpr int kMaxCtas = 2048;
constexpr int kHeaderBytes = kMaxCtas * 4;

// Mailbox layout (bytes from the base):
//   header        uint32 [kMaxCtas]: epoch counter of each CTA
//   flags         uint32 [2 banks][R sources][n_rows]
//   records       float  [2 banks][R sources][n_rows][kD + 1]   (O row, then lse)
__host__ __device__ inline size_t flags_offset() { return kHeaderBytes; }
__host__ __device__ inline size_t records_offset(int n_ranks, int64_t n_rows) {
    return (flags_offset() + sizeof(uint32_t) * 2 * (size_t) n_ranks * (size_t) n_rows + 255) / 256 * 256;
}
// Words of the fused decode exchange (decode_combine_kernel<true>): uint64 [2 banks][R sources]
// [n_rows][kD + 1], each the f32 bits of one value (low half) and the epoch that wrote it (high
// half), so a reader that sees its epoch in a word has the word's value - no flag, no fence.
__host__ __device__ inline size_t words_offset(int n_ranks, int64_t n_rows) {
    return (records_offset(n_ranks, n_rows) + sizeof(float) * 2 * (size_t) n_ranks * (size_t) n_rows * (kD + 1) + 255) /
           256 * 256;
}
__host__ __device__ inline size_t mailbox_bytes(int n_ranks, int64_t n_rows) {
    return words_offset(n_ranks, n_rows) + sizeof(uint64_t) * 2 * (size_t) n_ranks * (size_t) n_rows * (kD + 1);
}

struct Params {
    uint8_t *const *mailboxes;  // [n_ranks] device pointers: peers' mailboxes (mapped), own at [rank]
    int rank, n_ranks;
    int64_t n_rows;
    const float *local_o;    // [n_rows][kD]
    const float *local_lse;  // [n_rows], natural log, -inf for an empty chunk
    uint64_t wait_ns;
    float *out;      // [n_rows][kD]
    float *lse_out;  // [n_rows] or null
    DeviceStatus *status;
};

// Flags: a release store at system scope (cumulative: it publishes the CTA's record stores that
// precede it through the CTA barrier) and acquire loads at system scope (the CTA barrier after
// them orders the record loads of the other threads).
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Single 8-byte accesses (naturally aligned: single-copy atomic) for the value+epoch words.
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid: at most as many CTAs as can be resident at once (the host caps it), each taking rows
// blockIdx.x, blockIdx.x + gridDim.x, ... Every CTA pushes all its rows before it waits on any
// flag, so no rank's wait depends on a CTA of another rank that has not started.
__global__ void __launch_bounds__(kThreads) exchange_merge_kernel(const Params p) {
    pdl_wait();  // the local partials come from the decode launched before
    const int d = threadIdx.x;
    const int R = p.n_ranks;
    uint8_t *own = p.mailboxes[p.rank];
    uint32_t *my_epoch = reinterpret_cast<uint32_t *>(own) + blockIdx.x;
    const uint32_t epoch = *my_epoch + 1u;
    const int bank = (int) (epoch & 1u);
    const size_t rec_off = records_offset(R, p.n_rows);
    const int64_t slot_stride = p.n_rows * (kD + 1);  // floats per (bank, source)

    // 1. push this rank's rows to every mailbox, then raise the rows' flags there.
    for (int64_t row = blockIdx.x; row < p.n_rows; row += gridDim.x) {
        const float v = p.local_o[row * kD + d];
        const float l = p.local_lse[row];
        for (int r = 0; r < R; r++) {
            float *rec = reinterpret_cast<float *>(p.mailboxes[r] + rec_off) +
                         ((int64_t) bank * R + p.rank) * slot_stride + row * (kD + 1);
            rec[d] = v;
            if (d == 0) rec[kD] = l;
        }
    }
    __syncthreads();
    if (d < R)
        for (int64_t row = blockIdx.x; row < p.n_rows; row += gridDim.x)
            st_release_sys(reinterpret_cast<uint32_t *>(p.mailboxes[d] + flags_offset()) +
                               ((int64_t) bank * R + p.rank) * p.n_rows + row,
                           epoch);

    __shared__ int timed_out;
    for (int64_t row = blockIdx.x; row < p.n_rows; row += gridDim.x) {
        // 2. wait for every source's flag of this row in the own mailbox (bounded).
        if (d == 0) timed_out = 0;
        __syncthreads();
        if (d < R) {
            const uint32_t *flag =
                reinterpret_cast<const uint32_t *>(own + flags_offset()) + ((int64_t) bank * R + d) * p.n_rows + row;
            bool ok = ld_acquire_sys(flag) == epoch;
            if (!ok) {
                const uint64_t t0 = global_timer_ns();
                for (uint32_t i = 1; i < (1u << 30); i++) {
                    if (ld_acquire_sys(flag) == epoch) {
                        ok = true;
                        break;
                    }
                    if ((i & 63u) == 0 && global_timer_ns() - t0 > p.wait_ns) break;
                }
            }
            if (!ok) {
                timed_out = 1;
                report(p.status, kStatusTimeout, kSiteExchangeWait, d);
            }
        }
        __syncthreads();

        // 3. merge the R records of this row from the own mailbox.
        float o = 0.f, lse = -INFINITY;
        if (!timed_out) {
            const float *base =
                reinterpret_cast<const float *>(own + rec_off) + (int64_t) bank * R * slot_stride + row * (kD + 1);
            float M = -INFINITY;
            for (int r = 0; r < R; r++) M = fmaxf(M, __ldcv(base + r * slot_stride + kD));
            if (M != -INFINITY) {
                float den = 0.f, acc = 0.f;
                for (int r = 0; r < R; r++) {
                    const float wt = __expf(__ldcv(base + r * slot_stride + kD) - M);
                    den += wt;
                    acc += wt * __ldcv(base + r * slot_stride + d);
                }
                o = acc / den;
                lse = M + __logf(den);
            }
        }
        p.out[row * kD + d] = o;
        if (d == 0 && p.lse_out != nullptr) p.lse_out[row] = lse;
        __syncthreads();  // timed_out is reset for the next row only after every thread read it
    }

    if (d == 0) *my_epoch = epoch;  // read by this CTA's successor in the next call
}

}  // namespace exchange
}  // namespace lstk
