// prefill.cuh - paged causal flash-attention for prompt chunks on the tcgen05 tensor cores.
//
// Replaces flash_attn_ext for n_tokens > 1 (src/qwen3.cpp:155-167), where QK^T and PV are real
// dense contractions: per 128x128 tile pair, 2 x 128x128x128 MACs on f16 operands.
//
// Tiling. A work item is (sequence b, query tile qt, KV head kvh). Its 128 query rows are
// 128/G consecutive tokens x the G = n_head/n_head_kv query heads that share KV head kvh,
// row r = token (r / G), head kvh*G + r % G. Packing the GQA group into the M dimension lets
// one K/V tile feed all G heads in the same MMA. A TMA map over q [T][n_head][128] with box
// (64, G, 128/G) loads exactly that row order. K/V tiles are 128 keys = 4 pages, each page
// fetched by TMA through the block table (box (64, 1, 32), 128-byte swizzle).
//
// Persistent: one CTA per SM (226 KiB of shared memory, 512 TMEM columns) walks its share of the
// items, rounds of gridDim.x items in snake order over the heaviest-first numbering, so that per-CTA
// set-up is paid once and the next item's loads and first scores overlap the current item's
// epilogue. Pipeline:
//   warps 8, 10  TMA producers: Q (per item, once the item's last QK has read the previous one)
//           and K_j (warp 8), V_j (warp 10), each into a double buffer, running ahead into the next
//           item; the block table is read a warp at a time, one chunk of 32 pages ahead.
//   warp 9  S issuer (one lane): S_j = Q K_j^T into TMEM buffer j%2 once K_j has landed and PV_{j-2}
//           (which read P_{j-2} from the same columns) has completed, so it runs up to two tiles
//           ahead of the softmax, into the next item while the current one ends.
//   warp 11 PV issuer (one lane): O_h += P_j V_j per key half with P_j read from tensor memory
//           (TS form), as soon as that half's softmax warps have written it; an item's first PV
//           waits until the previous epilogue has read O out. Two issuing threads keep the
//           tensor core's shallow queue fed while either of them waits on a barrier.
//   warps 0-7  softmax: warp w owns the 32 rows of TMEM quadrant w%4 and key half w/4 of every
//           tile (its 64 score columns), so two warps on each SM sub-partition share the tile's
//           exp work. Each key half keeps its own running max, row sum and O accumulator (O_0,
//           O_1), so the halves never wait for each other inside the loop. Per tile: tcgen05.ld
//           of its 64 scores, causal mask, row max, P = 2^(s*scale - m) as f16 pairs, their sum
//           by mixed-precision adds, P written back over the first 32 of its 64 score columns.
//           The running max only moves (and O_h is rescaled in TMEM) when a tile's max exceeds
//           it by more than 2^8, so the softmax rarely waits for the previous PV. Epilogue: the
//           halves swap (m, l) per row through shared memory and merge O = (O_0 2^(m_0-M) +
//           O_1 2^(m_1-M)) / (l_0 2^(m_0-M) + l_1 2^(m_1-M)); a full tile is staged in its own
//           buffer and leaves through TMA stores that complete while the next item runs (their source reads are awaited before the buffer
//           is written again). All softmax warps run every item's named barriers and agree on
//           failure with a barrier reduction, so they stop at the same item.
// The kernel is launched with programmatic stream serialization: barrier and TMEM set-up overlap
// the previous kernel, and griddepcontrol.wait precedes every read of earlier work.
// TMEM: S0 cols [0,128), S1 [128,256), O_0 [256,384), O_1 [384,512) (f32, 128 lanes = 128 rows).
// P_j occupies S_j's columns [0,32) (keys 0..63) and [64,96) (keys 64..127); QK_{j+2}
// overwrites them only after PV_j has completed (o_done).
// Every mbarrier wait is on a parity at most one phase from the arrivals: per-buffer barriers
// (K, V, S, P, o_done) indexed by a running tile count across items, and one q_full / q_empty /
// o_free / o_final phase per item.
// Measured limit: per 128-key tile the tensor core runs 8 SS MMAs (S) and 8 TS MMAs (PV) of
// 128x128x16, 64 cycles each when fed back to back. Its instruction queue is shallow, so stalls
// of the issuing threads (barrier checks, issue slots lost to the busy softmax warps) leave it
// idle; with one tile of lookahead (two S buffers) the round trip S_j -> softmax -> PV_j ->
// S_{j+2} bounds the kernel at about 2.1 k cycles per tile.
//
// Operand layouts (UMMA shared-memory descriptors, 128-byte swizzle, atoms of 8 rows x 128 B):
//   Q, K: K-major (contraction dim contiguous), two 16 KiB sub-tiles of 64 columns.
//   V: the B operand of PV with N = head dim contiguous ("MN-major"): sub-tile h holds dims
//      64h..64h+63 of all 128 keys; LBO = 16 KiB between the two dim halves, SBO = 1 KiB
//      between groups of 8 keys.
#pragma once

#include "common.cuh"
#include "tcgen05.cuh"

namespace lstk {
namespace prefill {

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kD = 128;
constexpr int kPage = 32;
constexpr int kTile = kBM * kD * 2;  // 32 KiB
constexpr int kSub = kTile / 2;      // 16 KiB: 128 rows x 128 B
constexpr int kSoftmaxWarps = 8;
constexpr int kWarpTmaK = 8;   // Q and K producer
constexpr int kWarpMma = 9;     // S (QK) MMA issuer; allocates TMEM
constexpr int kWarpTmaV = 10;  // V producer
constexpr int kWarpMmaPv = 11; // PV MMA issuer
constexpr int kThreads = 384;
constexpr int kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO0 = 256, kColO1 = 384;

// Shared memory carve-up (offsets from the 1024-aligned dynamic shared memory base).
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTile;       // 2 buffers
constexpr int kOffV = kOffK + 2 * kTile;   // 2 buffers
constexpr int kOffO = kOffV + 2 * kTile;   // output staging: 128 rows x 128 f32 (64 KiB)
constexpr int kOffBar = kOffO + 2 * kTile;
constexpr int kSmemBytes = kOffBar + 2304;  // + barriers and row statistics

struct Params {
    int n_seqs, n_head, n_head_kv, group, n_qt, n_items;
    int total_tokens;  // rows of q and out: every sequence's [q_seq_start[b], q_seq_start[b+1]) must lie inside
    const int32_t *q_seq_start;
    const int32_t *q_pos0;
    const int32_t *kv_lens;
    const int32_t *block_tables;
    int max_blocks;
    int64_t n_pages;
    int64_t n_cells;
    float scale_log2;
    float *out;
    DeviceStatus *status;
    uint64_t wait_ns;           // limit of each pipeline wait (drains keep kWaitLimitNs)
    const int32_t *start_flag;  // optional: the producers wait for it to be non-zero before loading
};

struct Barriers {
    uint64_t q_full;
    uint64_t q_empty;  // the item's last S MMA has read Q: the next item's Q may load
    uint64_t o_free;   // the softmax warps have read O out: the next item's first PV may write it
    uint64_t k_full[2], v_full[2];  // K_j / V_j landed; their buffers are freed by s_full / o_done
    uint64_t s_full[2];
    // P_j of key half h: one arrival per softmax warp of that half, on p_full[h][j % 2]. A barrier
    // per S buffer keeps every wait within one phase of the arrivals: P_{j+2} needs S_{j+2},
    // which the S issuer creates only after PV_j (which needed P_j) has completed.
    uint64_t p_full[2][2];
    // PV_j done, on o_done[j % 2]: V_j's buffer and P_j's TMEM columns are free, and O may be
    // rescaled by a softmax warp.
    uint64_t o_done[2];
    // One completion per item, after its last PV: the epilogue's wait. The next item's PVs need
    // the epilogue's o_free first, so this barrier is never two phases ahead of a waiter.
    uint64_t o_final;
    uint64_t mma_drain[2];  // per MMA-issuing thread
    uint32_t tmem_base;
    int abort;
    float row_m[2][kBM], row_l[2][kBM];  // per key half: running max (log2 domain) and sum per row
};
static_assert(sizeof(Barriers) <= 2304, "barrier block over its reserved bytes");
static_assert(kSmemBytes <= 232448, "shared memory over the 227 KiB limit");

// Instruction descriptor for kind::f16: f32 accumulator, f16 A and B, M = 128, N = 128.
constexpr uint32_t idesc_f16(bool b_mn_major) {
    return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t) (kBN >> 3) << 17) | ((uint32_t) (kBM >> 4) << 24);
}

// Three-input max (one instruction on sm_100a).
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Softmax numerator for two adjacent scores with packed instructions: x = s * scale_log2 - mu
// for both (fma.f32x2), rounded to an f16 pair, 2^x for both (ex2.approx.f16x2; P is consumed
// as f16 by the PV MMA anyway), and the two f16 results added to two f32 row sums by
// mixed-precision adds (add.f32.f16), so the normaliser sums exactly the P the tensor core
// multiplies. Returns the f16 pair (lower half = first score).
__device__ __forceinline__ uint32_t softmax_pair(float s0, float s1, uint64_t scale2, uint64_t neg_mu2, float &sum_lo,
                                                 float &sum_hi) {
    uint32_t p;
    asm("{\n\t"
        ".reg .b64 x, y;\n\t"
        ".reg .f32 a, b;\n\t"
        ".reg .b16 lo, hi;\n\t"
        "mov.b64 x, {%3, %4};\n\t"
        "fma.rn.f32x2 y, x, %5, %6;\n\t"
        "mov.b64 {a, b}, y;\n\t"
        "cvt.rn.f16x2.f32 %0, b, a;\n\t"
        "ex2.approx.f16x2 %0, %0;\n\t"
        "mov.b32 {lo, hi}, %0;\n\t"
        "add.f32.f16 %1, lo, %1;\n\t"
        "add.f32.f16 %2, hi, %2;\n\t"
        "}"
        : "=r"(p), "+f"(sum_lo), "+f"(sum_hi)
        : "f"(s0), "f"(s1), "l"(scale2), "l"(neg_mu2));
    return p;
}

__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
    return ((uint64_t) __float_as_uint(hi) << 32) | __float_as_uint(lo);
}

// The running max is only moved (and O rescaled) when a tile's max exceeds it by more than this
// many powers of two; otherwise P uses the stale max, so its entries stay below 2^8.
constexpr float kRescaleThreshold = 8.f;

extern __shared__ __align__(1024) uint8_t dyn_smem[];

// One work item: (sequence b, query tile, KV head kvh). Items are numbered heaviest first (latest
// query positions first); an item past its sequence's end has no keys and no live rows.
struct Item {
    int b, kvh, tok0, q_begin, n_q, kv_len, pos0, n_keys, n_tiles;
    bool bad_rows;  // the sequence's query rows are not inside [0, total_tokens): no rows, reported
};

// An item's sequence metadata as loaded; item_finish derives the rest, so a loop can issue the
// next item's loads early and use them one item later.
struct ItemRaw {
    int b, kvh, tok0, q0, q1, kv_len_raw, pos0;
};

__device__ __forceinline__ ItemRaw item_load(const Params &p, int x) {
    ItemRaw r;
    r.kvh = x % p.n_head_kv;
    const int rest = x / p.n_head_kv;
    r.b = rest % p.n_seqs;
    r.tok0 = (p.n_qt - 1 - rest / p.n_seqs) * (kBM / p.group);
    r.q0 = p.q_seq_start[r.b];
    r.q1 = p.q_seq_start[r.b + 1];
    r.kv_len_raw = p.kv_lens[r.b];
    r.pos0 = p.q_pos0[r.b];
    return r;
}

__device__ __forceinline__ Item item_finish(const Params &p, const ItemRaw &r) {
    Item it;
    it.b = r.b;
    it.kvh = r.kvh;
    it.tok0 = r.tok0;
    it.q_begin = r.q0;
    // Rows come from device memory: a range outside q / out or a decreasing start gives the
    // sequence no rows (nothing is read or written for it) and is reported once.
    it.bad_rows = r.q0 < 0 || r.q1 < r.q0 || r.q1 > p.total_tokens;
    it.n_q = it.bad_rows ? 0 : r.q1 - r.q0;
    it.kv_len = max(0, min(r.kv_len_raw, p.max_blocks * kPage));
    it.pos0 = r.pos0;
    const int last_tok = min(it.tok0 + kBM / p.group, it.n_q) - 1;
    it.n_keys = it.tok0 < it.n_q ? max(0, min(it.kv_len, it.pos0 + last_tok + 1)) : 0;
    it.n_tiles = (it.n_keys + kBN - 1) / kBN;
    return it;
}

__device__ __forceinline__ Item item_at(const Params &p, int x) { return item_finish(p, item_load(p, x)); }

// The r-th item of this CTA (-1 past the end): rounds of gridDim.x items in "snake" order, forward
// in even rounds and backward in odd ones, so the CTA that took one of the lightest items of a
// round takes the heaviest of the next.
__device__ __forceinline__ int item_index(const Params &p, int r) {
    const int64_t g = gridDim.x;
    const int64_t idx = (int64_t) r * g + ((r & 1) ? g - 1 - (int64_t) blockIdx.x : (int64_t) blockIdx.x);
    return idx < p.n_items ? (int) idx : -1;
}

__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                                                              const __grid_constant__ CUtensorMap kmap,
                                                              const __grid_constant__ CUtensorMap vmap,
                                                              const __grid_constant__ CUtensorMap omap,
                                                              const Params p) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;

    uint8_t *base = dyn_smem;
    if ((smem_u32(base) & 1023u) != 0) {  // the 128-byte swizzle needs 1024-byte aligned tiles
        if (threadIdx.x == 0) report(p.status, kStatusBadIndex, kSitePrefillSmem, (int) (smem_u32(base) & 1023u));
        return;
    }
    Barriers *bars = reinterpret_cast<Barriers *>(base + kOffBar);
    const uint32_t sQ = smem_u32(base + kOffQ);
    const uint32_t sK = smem_u32(base + kOffK);
    const uint32_t sV = smem_u32(base + kOffV);
    const uint32_t sO = smem_u32(base + kOffO);
    volatile int *abort_flag = &bars->abort;

    if (threadIdx.x == 0) {
        bars->abort = 0;
        mbar_init(smem_u32(&bars->q_full), 1);
        mbar_init(smem_u32(&bars->q_empty), 1);
        mbar_init(smem_u32(&bars->o_free), kSoftmaxWarps);
        for (int i = 0; i < 2; i++) {
            mbar_init(smem_u32(&bars->k_full[i]), 1);
            mbar_init(smem_u32(&bars->v_full[i]), 1);
            mbar_init(smem_u32(&bars->s_full[i]), 1);
            mbar_init(smem_u32(&bars->o_done[i]), 1);
            mbar_init(smem_u32(&bars->mma_drain[i]), 1);
        }
        for (int h = 0; h < 2; h++)
            for (int i = 0; i < 2; i++) mbar_init(smem_u32(&bars->p_full[h][i]), kSoftmaxWarps / 2);
        mbar_init(smem_u32(&bars->o_final), 1);
        fence_barrier_init();
    }
    if (warp == kWarpMma) {
        tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    // The set-up above overlaps the previous kernel in the stream (programmatic dependent
    // launch); everything below reads what earlier work produced.
    pdl_wait();
    pdl_launch_dependents();
    const int G = p.group;

    // Every role walks the same item sequence. Barrier phases come from running counters: g, the
    // global index of a K/V tile in this CTA (buffer g % 2, parity (g / 2) % 2 for the per-buffer
    // barriers; parity g % 2 for o_done, one completion per PV), and the count of items that have
    // tiles (q_full, q_empty, o_free, o_final: one completion per item).
    if (warp == kWarpTmaK || warp == kWarpTmaV) {
        // ---- TMA producers: warp 8 streams Q and the K tiles, warp 10 the V tiles, each into
        // its own double buffer, running ahead into the next item while the current one ends.
        // The block table is read a warp at a time (lane i: page 32c + i, one chunk ahead) and
        // lane 0 issues the copies. ----
        const bool is_k = warp == kWarpTmaK;
        if (lane == 0) {
            if (is_k) {
                prefetch_tensormap(&qmap);
                prefetch_tensormap(&kmap);
            } else {
                prefetch_tensormap(&vmap);
            }
        }
        const uint32_t dst0 = is_k ? sK : sV;
        const CUtensorMap *map = is_k ? &kmap : &vmap;
        int g = 0, n_items_t = 0;
        bool ok = true;
        if (p.start_flag != nullptr) {
            if (lane == 0 && !(ok = flag_wait_bounded(p.start_flag, abort_flag, p.wait_ns))) {
                report(p.status, kStatusTimeout, kSitePrefillWaitStart, warp);
                *abort_flag = 1;
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        for (int r = 0; ok; r++) {
            const int x = item_index(p, r);
            if (x < 0) break;
            const Item I = item_at(p, x);
            if (I.n_tiles == 0) continue;
            if (is_k && lane == 0) {
                if (n_items_t > 0)
                    ok = mbar_wait_bounded(smem_u32(&bars->q_empty), (uint32_t) (n_items_t - 1) & 1, abort_flag, p.wait_ns);
                if (ok) {
                    mbar_arrive_expect_tx(smem_u32(&bars->q_full), kTile);
                    for (int h = 0; h < 2; h++)
                        tma_load_3d(sQ + h * kSub, &qmap, smem_u32(&bars->q_full), h * 64, I.kvh * G,
                                    I.q_begin + I.tok0);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            n_items_t++;
            const int32_t *bt = p.block_tables + (int64_t) I.b * p.max_blocks;
            const int n_pg = (I.n_keys + kPage - 1) / kPage;  // pages holding visible keys
            auto load_chunk = [&](int chunk) -> int {
                const int pi = chunk * 32 + lane;
                int cell = (int) p.n_cells;  // out of bounds: TMA fills zeros
                if (pi < n_pg) {
                    const int32_t pid = bt[pi];
                    if (pid >= 0 && pid < p.n_pages) cell = pid * kPage;
                    else if (is_k) report(p.status, kStatusBadIndex, kSitePrefillPage, pid);
                }
                return cell;
            };
            int cur = load_chunk(0);
            int nxt = n_pg > 32 ? load_chunk(1) : (int) p.n_cells;
            for (int j = 0; j < I.n_tiles; j++) {
                if (j > 0 && (j & 7) == 0) {  // next 32 pages: 8 tiles
                    cur = nxt;
                    nxt = (j / 8 + 1) * 32 < n_pg ? load_chunk(j / 8 + 1) : (int) p.n_cells;
                }
                int cell0[4];
#pragma unroll
                for (int q = 0; q < 4; q++) cell0[q] = __shfl_sync(0xffffffffu, cur, (j & 7) * 4 + q);
                if (lane == 0) {
                    const int buf = g & 1;
                    const uint32_t use = (uint32_t) (g >> 1);
                    const uint32_t empty = smem_u32(is_k ? &bars->s_full[buf] : &bars->o_done[buf]);
                    const uint32_t full = smem_u32(is_k ? &bars->k_full[buf] : &bars->v_full[buf]);
                    if (use > 0) ok = mbar_wait_bounded(empty, (use - 1) & 1, abort_flag, p.wait_ns);
                    if (ok) {
                        mbar_arrive_expect_tx(full, kTile);
                        for (int q = 0; q < 4; q++)
                            for (int h = 0; h < 2; h++)
                                tma_load_3d(dst0 + buf * kTile + h * kSub + q * (kPage * 128), map, full, h * 64,
                                            I.kvh, cell0[q]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                g++;
            }
        }
        if (lane == 0) {
            if (!ok) {
                report(p.status, kStatusTimeout, kSitePrefillWait, warp);
                *abort_flag = 1;
            }
            if (*abort_flag) {
                // Drain: every load still in flight lands before shared memory is released.
                if (is_k && n_items_t > 0)
                    mbar_wait_bounded(smem_u32(&bars->q_full), (uint32_t) (n_items_t - 1) & 1, nullptr);
                for (int gg = max(0, g - 2); gg < g; gg++)
                    mbar_wait_bounded(smem_u32(is_k ? &bars->k_full[gg & 1] : &bars->v_full[gg & 1]),
                                      (uint32_t) (gg >> 1) & 1, nullptr);
            }
        }
    } else if (warp == kWarpMma) {
        // ---- S issuer: S_gg = Q K_gg^T into TMEM buffer gg % 2, once K_gg has landed and PV_{gg-2}
        // (same buffer: it read P_{gg-2} from these columns) has completed. Two issuing threads,
        // one for S and one for PV, keep the tensor core's shallow queue fed while either waits
        // on a barrier. A commit tracks only the committing thread's MMAs: s_full[gg % 2] also
        // frees K buffer gg % 2; after the item's last S, Q may be reloaded. ----
        if (lane == 0) {
            constexpr uint32_t idesc_qk = idesc_f16(false);
            // Shared-memory descriptors as (low, high) words, built once: the high word is fixed,
            // the low word holds address >> 4 (tiles stay below 256 KiB, so offsets never carry
            // out of it), so each MMA needs one add for its operand addresses.
            const uint64_t dq0 = sdesc_sw128(sQ, 16, 1024), dk0 = sdesc_sw128(sK, 16, 1024);
            const uint32_t lq = (uint32_t) dq0, lk = (uint32_t) dk0;
            const uint64_t hq = dq0 & 0xFFFFFFFF00000000ull, hk = dk0 & 0xFFFFFFFF00000000ull;
            int g = 0, n_items_t = 0;
            bool ok = true, issued = false;
            for (int r = 0; ok; r++) {
                const int x = item_index(p, r);
                if (x < 0) break;
                const int n = item_at(p, x).n_tiles;
                if (n == 0) continue;
                ok = mbar_wait_bounded(smem_u32(&bars->q_full), (uint32_t) n_items_t & 1, abort_flag, p.wait_ns);
                for (int j = 0; ok && j < n; j++) {
                    const int gg = g + j;
                    const int buf = gg & 1;
                    ok = mbar_wait_bounded(smem_u32(&bars->k_full[buf]), (uint32_t) (gg >> 1) & 1, abort_flag, p.wait_ns);
                    if (ok && gg >= 2)
                        ok = mbar_wait_bounded(smem_u32(&bars->o_done[buf]), (uint32_t) ((gg - 2) >> 1) & 1,
                                               abort_flag, p.wait_ns);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t d = tmem + (buf ? kColS1 : kColS0);
                    const uint32_t lkb = lk + (uint32_t) buf * (kTile >> 4);
                    mma_f16_ss_k<0>(d, hq | lq, hk | lkb, idesc_qk);
#pragma unroll
                    for (int kk = 1; kk < 8; kk++) {
                        const uint32_t off = (uint32_t) (((kk >> 2) * kSub + (kk & 3) * 32) >> 4);
                        mma_f16_ss_k<1>(d, hq | (lq + off), hk | (lkb + off), idesc_qk);
                    }
                    mma_commit(smem_u32(&bars->s_full[buf]));
                    if (j == n - 1) mma_commit(smem_u32(&bars->q_empty));
                    issued = true;
                }
                g += n;
                n_items_t++;
            }
            if (!ok) {
                report(p.status, kStatusTimeout, kSitePrefillWait, kWarpMma);
                *abort_flag = 1;
            }
            // Every MMA this thread issued completes before TMEM can be released.
            if (issued) {
                mma_commit(smem_u32(&bars->mma_drain[0]));
                mbar_wait_bounded(smem_u32(&bars->mma_drain[0]), 0, nullptr);
            }
        }
    } else if (warp == kWarpMmaPv) {
        // ---- PV issuer: O_h += P_gg V_gg for key half h, as soon as that half's four softmax
        // warps have written P_gg; its commits (o_done, o_final) track only the PV MMAs. ----
        if (lane == 0) {
            constexpr uint32_t idesc_pv = idesc_f16(true);
            const uint64_t dv0 = sdesc_sw128(sV, kSub, 1024);
            const uint32_t lv = (uint32_t) dv0;
            const uint64_t hv = dv0 & 0xFFFFFFFF00000000ull;
            int g = 0, n_items_t = 0;
            bool ok = true, issued = false;
            for (int r = 0; ok; r++) {
                const int x = item_index(p, r);
                if (x < 0) break;
                const int n = item_at(p, x).n_tiles;
                if (n == 0) continue;
                for (int j = 0; ok && j < n; j++) {
                    const int gg = g + j;
                    const int buf = gg & 1;
                    ok = mbar_wait_bounded(smem_u32(&bars->v_full[buf]), (uint32_t) (gg >> 1) & 1, abort_flag, p.wait_ns);
                    // The item's first PV overwrites O: the previous item's epilogue must have read it.
                    if (ok && j == 0 && n_items_t > 0)
                        ok = mbar_wait_bounded(smem_u32(&bars->o_free), (uint32_t) (n_items_t - 1) & 1, abort_flag, p.wait_ns);
                    // P_gg sits in TMEM over S_gg: keys 0..63 in columns [0, 32), keys 64..127 in
                    // [64, 96) of the S buffer, two f16 per 32-bit column (16 keys per MMA step).
                    const uint32_t pcol = tmem + (buf ? kColS1 : kColS0);
                    for (int h = 0; h < 2 && ok; h++) {
                        ok = mbar_wait_bounded(smem_u32(&bars->p_full[h][buf]), (uint32_t) (gg >> 1) & 1,
                                               abort_flag, p.wait_ns);
                        if (!ok) break;
                        tc_fence_after();
                        // V rows of K step kk: 16 keys x 128 B = 128 descriptor units from the tile start.
                        const uint32_t oc = tmem + (h ? kColO1 : kColO0), pc = pcol + (uint32_t) (h * 64);
                        const uint32_t lvb = lv + (uint32_t) buf * (kTile >> 4) + (uint32_t) (4 * h) * 128u;
                        mma_f16_ts(oc, pc, hv | lvb, idesc_pv, j > 0 ? 1u : 0u);
#pragma unroll
                        for (int kq = 1; kq < 4; kq++) mma_f16_ts_k<1>(oc, pc + kq * 8, hv | (lvb + kq * 128u), idesc_pv);
                        issued = true;
                    }
                    if (!ok) break;
                    mma_commit(smem_u32(&bars->o_done[buf]));
                    if (j == n - 1) mma_commit(smem_u32(&bars->o_final));
                }
                g += n;
                n_items_t++;
            }
            if (!ok) {
                report(p.status, kStatusTimeout, kSitePrefillWait, kWarpMmaPv);
                *abort_flag = 1;
            }
            if (issued) {
                mma_commit(smem_u32(&bars->mma_drain[1]));
                mbar_wait_bounded(smem_u32(&bars->mma_drain[1]), 0, nullptr);
            }
        }
    } else {
        // ---- softmax warps 0..7: warp w owns rows 32*(w%4).. and the key half w/4 of every
        // tile (score columns 64*(w/4)..); each half keeps its own running max, sum and O ----
        const int hf = warp >> 2;
        const int quad = warp & 3;
        const int r = quad * 32 + lane;  // row within the tile
        const uint32_t lane_base = tmem + ((uint32_t) (quad * 32) << 16);
        const uint32_t ocol = lane_base + (hf ? kColO1 : kColO0);
        const uint64_t scale2 = pack_f32x2(p.scale_log2, p.scale_log2);
        bool store_pending = false;  // warp 0 lane 0: a TMA store still reading the staging buffer
        int g = 0, n_items_t = 0;
        int x = item_index(p, 0);
        ItemRaw raw_next = x >= 0 ? item_load(p, x) : ItemRaw{};
        for (int it = 0; x >= 0; it++) {
            const Item I = item_finish(p, raw_next);
            if (I.bad_rows && warp == 0 && lane == 0) report(p.status, kStatusBadIndex, kSitePrefillRows, I.b);
            // The next item's metadata loads are issued now and used one item later.
            const int x_next = item_index(p, it + 1);
            if (x_next >= 0) raw_next = item_load(p, x_next);
            x = x_next;
            const int n_tiles = I.n_tiles;
            const int tq = I.tok0 + r / G;  // query token index within the sequence
            const int head = I.kvh * G + r % G;
            const int row_keys = min(I.kv_len, I.pos0 + tq + 1);  // keys [0, row_keys) are visible
            const bool live = tq < I.n_q;
            bool ok = true;
            float m = -INFINITY, l = 0.f;  // this key half's running max (log2 domain) and sum
            for (int j = 0; j < n_tiles; j++) {
                const int gg = g + j;
                const int buf = gg & 1;
                // Warp-uniform outcomes: tcgen05.ld / st below are warp-collective.
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&bars->s_full[buf]),
                                                                (uint32_t) (gg >> 1) & 1, abort_flag, p.wait_ns))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float sc[64];
                tmem_ld32(lane_base + (buf ? kColS1 : kColS0) + 64 * hf, sc);
                tmem_ld32(lane_base + (buf ? kColS1 : kColS0) + 64 * hf + 32, sc + 32);
                tmem_wait_ld();
                const int kbase = j * kBN + 64 * hf;  // key index of this warp's first column
                if (kbase + 64 > row_keys) {
#pragma unroll
                    for (int c = 0; c < 64; c++) sc[c] = (kbase + c < row_keys) ? sc[c] : -INFINITY;
                }
                // Row max of the raw scores (the scale is positive): 8 independent max3 chains.
                float mx[8];
#pragma unroll
                for (int i = 0; i < 8; i++) mx[i] = fmaxf(sc[i], sc[8 + i]);
#pragma unroll
                for (int c = 16; c < 64; c += 16)
#pragma unroll
                    for (int i = 0; i < 8; i++) mx[i] = max3(mx[i], sc[c + i], sc[c + 8 + i]);
                const float m_tile =
                    fmaxf(max3(mx[0], mx[1], mx[2]), fmaxf(max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]))) *
                    p.scale_log2;
                const bool move = m_tile > m + kRescaleThreshold;  // always true for the first visible tile
                const float m_new = move ? m_tile : m;
                const float alpha = move ? fast_exp2(m - m_new) : 1.f;
                const float mu = m_new == -INFINITY ? 0.f : m_new;
                const uint64_t neg_mu2 = pack_f32x2(-mu, -mu);
                float rsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // independent partial row sums
                uint32_t pk[32];
#pragma unroll
                for (int c = 0; c < 32; c++)
                    pk[c] = softmax_pair(sc[2 * c], sc[2 * c + 1], scale2, neg_mu2, rsum[2 * (c & 3)],
                                         rsum[2 * (c & 3) + 1]);
                // A moved max rescales O_hf, which PV_{gg-1} must have finished updating (PV_{gg-2}
                // has: S_gg ready implies it). P goes to buffer gg % 2, last read by PV_{gg-2}.
                if (j > 0 && __any_sync(0xffffffffu, move)) {
                    if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&bars->o_done[(gg - 1) & 1]),
                                                                    (uint32_t) ((gg - 1) >> 1) & 1, abort_flag, p.wait_ns))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        float o[32];
                        tmem_ld32(ocol + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] *= alpha;
                        tmem_st32(ocol + c * 32, o);
                    }
                }
                // P row r, keys 64*hf.., packed f16 pairs, over the first 32 of this warp's own
                // 64 score columns (already read), where the PV MMA reads its A operand.
                {
                    float pkf[32];
#pragma unroll
                    for (int c = 0; c < 32; c++) pkf[c] = __uint_as_float(pk[c]);
                    tmem_st32(lane_base + (buf ? kColS1 : kColS0) + 64 * hf, pkf);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bars->p_full[hf][buf]));
                const float rs = ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
                l = l * alpha + rs;
                m = m_new;
            }
            // Epilogue: every PV of the item has completed (o_final, one phase per item).
            if (n_tiles > 0) {
                if (ok)
                    ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&bars->o_final),
                                                                    (uint32_t) n_items_t & 1, abort_flag, p.wait_ns));
                // The halves swap (m, l) per row and merge O = (O_0 2^(m_0 - M) + O_1 2^(m_1 - M)) /
                // (l_0 2^(m_0 - M) + l_1 2^(m_1 - M)); warp w writes output columns 64*(w/4) .. +63.
                bars->row_m[hf][r] = m;
                bars->row_l[hf][r] = l;
                if (warp == 0 && lane == 0 && store_pending) {  // the staging buffer is free again
                    tma_store_wait_read();
                    store_pending = false;
                }
                tc_fence_before();
                asm volatile("bar.sync 1, %0;" ::"r"(kSoftmaxWarps * 32) : "memory");
                tc_fence_after();
                const float m_o = bars->row_m[hf ^ 1][r], l_o = bars->row_l[hf ^ 1][r];
                const float mm = fmaxf(m, m_o);
                const float a_me = l > 0.f ? fast_exp2(m - mm) : 0.f;
                const float a_ot = l_o > 0.f ? fast_exp2(m_o - mm) : 0.f;
                const float den = l * a_me + l_o * a_ot;
                const float inv = den > 0.f ? 1.f / den : 0.f;
                const float c0 = (hf == 0 ? a_me : a_ot) * inv;  // weight of O_0
                const float c1 = (hf == 0 ? a_ot : a_me) * inv;  // weight of O_1
                const bool use0 = c0 > 0.f, use1 = c1 > 0.f;      // an O that never saw a visible key is not read
                ok = __all_sync(0xffffffffu, ok);
                // This warp's 64 output columns, 32 at a time out of both accumulators: a full tile
                // is staged for TMA stores (four 32-column boxes of 128 rows x 128 B with the
                // 128-byte swizzle, whose row order (token, head) is the tile's), a ragged tile's
                // live rows are stored directly. Then O is released for the next item's PVs.
                const bool full = I.tok0 + kBM / G <= I.n_q;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    float a[32], b2[32];
                    tmem_ld32(lane_base + kColO0 + 64 * hf + 32 * c, a);
                    tmem_ld32(lane_base + kColO1 + 64 * hf + 32 * c, b2);
                    tmem_wait_ld();
                    float o[32];
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = (use0 ? a[i] * c0 : 0.f) + (use1 ? b2[i] * c1 : 0.f);
                    if (full && ok) {
                        const uint32_t box = sO + (uint32_t) (2 * hf + c) * kSub;
#pragma unroll
                        for (int ch = 0; ch < 8; ch++)
                            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(
                                             box + sw128_offset((uint32_t) r, (uint32_t) ch)),
                                         "f"(o[4 * ch]), "f"(o[4 * ch + 1]), "f"(o[4 * ch + 2]), "f"(o[4 * ch + 3])
                                         : "memory");
                    } else if (!full && live && ok) {
                        float *dst = p.out + ((int64_t) (I.q_begin + tq) * p.n_head + head) * kD + 64 * hf + 32 * c;
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            *reinterpret_cast<float4 *>(dst + i) = make_float4(o[i], o[i + 1], o[i + 2], o[i + 3]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&bars->o_free));
                if (full) {
                    if (ok) fence_proxy_async_smem();
                    asm volatile("bar.sync 1, %0;" ::"r"(kSoftmaxWarps * 32) : "memory");
                    if (warp == 0 && lane == 0 && ok && !*abort_flag) {  // completes while the next item runs
                        for (int bx = 0; bx < 4; bx++)
                            tma_store_3d(&omap, sO + (uint32_t) bx * kSub, 32 * bx, I.kvh * G, I.q_begin + I.tok0);
                        tma_store_commit();
                        store_pending = true;
                    }
                }
                g += n_tiles;
                n_items_t++;
            } else if (live) {
                // no visible keys: the row's output is zero
                float *dst = p.out + ((int64_t) (I.q_begin + tq) * p.n_head + head) * kD + 64 * hf;
#pragma unroll
                for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4 *>(dst + i) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            // All eight warps stop at the same item if any of them failed (every warp has run this
            // item's named barriers).
            int any_fail;
            asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.s32 p, %1, 0;\n\t"
                         "bar.red.or.pred p, 2, %2, p;\n\tselp.s32 %0, 1, 0, p;\n\t}"
                         : "=r"(any_fail)
                         : "r"(ok ? 0 : 1), "r"(kSoftmaxWarps * 32)
                         : "memory");
            if (any_fail) {
                if (threadIdx.x == 0) {
                    report(p.status, kStatusTimeout, kSitePrefillWait, warp);
                    *abort_flag = 1;
                }
                break;
            }
        }
        if (warp == 0 && lane == 0 && store_pending) tma_store_wait_read();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kWarpMma) tmem_dealloc(tmem, kTmemCols);
}

// f32 -> f16 copy of q for the tensor-core path (when the caller passes f32 queries).
__global__ void q_to_f16_kernel(const float *src, __half *dst, int64_t n) {
    for (int64_t i = ((int64_t) blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n;
         i += (int64_t) gridDim.x * blockDim.x * 4) {
        if (i + 3 < n) {
            const float4 v = *reinterpret_cast<const float4 *>(src + i);
            *reinterpret_cast<__half2 *>(dst + i) = __floats2half2_rn(v.x, v.y);
            *reinterpret_cast<__half2 *>(dst + i + 2) = __floats2half2_rn(v.z, v.w);
        } else {
            for (int64_t k = i; k < n; k++) dst[k] = __float2half_rn(src[k]);
        }
    }
}

}  // namespace prefill
}  // namespace lstk
