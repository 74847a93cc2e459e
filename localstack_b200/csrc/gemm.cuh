// gemm.cuh - the attention block's projections on the tcgen05 tensor cores, and the small
// row kernels around them.
//
// Replaces ggml_mul_mat for the Q/K/V and output projections of attn_block (proj() at
// src/qwen3.cpp:117-120, called at :135-138, and the Wo projection + residual add at :169-170),
// plus the input RMSNorm rms(x, attn_norm) (:112-114, :134):
//   out[m][n] = sum_k x[m][k] * w[n][k]  (+ residual[m][n])
// x: activations [tokens][k] bf16 (row-major, k contiguous); w: a weight in ggml's layout for
// mul_mat, [n][k] bf16 (ne0 = k contiguous); both operands are K-major, the UMMA's native form.
// f32 accumulation in tensor memory; the epilogue adds the residual in f32 and rounds once to the
// output type (bf16 or f32).
//
// Tiling. One CTA per SM (persistent) walks output tiles of 128 x 256 in rounds of gridDim.x,
// m-tile fastest, so the CTAs of a round share few weight tiles and the whole operand set stays in
// the 126 MB L2. Per 64-wide K block a stage holds the x tile (128 rows x 128 B) and the w tile
// (256 rows x 128 B), both written by TMA with the 128-byte swizzle; four stages (192 KiB).
// Roles (6 warps):
//   warp 0   TMA producer (one lane): the stage ring, across tiles;
//   warp 1   MMA issuer (one lane; allocates 512 tensor-memory columns): per stage four
//            tcgen05.mma.cta_group::1.kind::f16 of M 128 x N 256 x K 16 (bf16 x bf16 -> f32) into
//            accumulator buffer (tile % 2), then a commit that frees the stage; after the tile's
//            last stage a commit to acc_full;
//   warps 2-5 epilogue: warp w reads tensor-memory lanes 32 (w % 4) .. + 31 (its quadrant: one
//            output row per thread), 32 columns at a time, adds the residual, rounds, and writes
//            the 32 x 32 block into one of its two swizzled staging buffers, which a TMA bulk store
//            copies out while the warp goes on (coalesced, clipped at the matrix edges); the
//            accumulator buffer is released as soon as its last columns are read, and the MMA
//            issuer reuses it two tiles later.
// Two accumulator buffers (2 x 256 columns) let the epilogue of tile i run under the MMAs of
// tile i + 1. Every wait is bounded (the launch's wait limit); on timeout the kernel records it,
// drains its copies and MMAs, frees tensor memory and returns.
#pragma once

#include "common.cuh"
#include "tcgen05.cuh"

namespace lstk {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;  // 128 bytes of bf16: one swizzle row
constexpr int kStages = 4;
constexpr int kATile = kBM * kBK * 2;  // 16 KiB
constexpr int kBTile = kBN * kBK * 2;  // 32 KiB
constexpr int kStageBytes = kATile + kBTile;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kTmemCols = 2 * kBN;
// Output staging: 8 KiB per epilogue warp, a ring of 32 x 32 blocks in the swizzled TMA layout:
// two f32 blocks of 4 KiB (rows of 128 B) or four bf16 blocks of 2 KiB (rows of 64 B).
constexpr int kWarpStageBytes = 8192;
constexpr int kOffOut = kStages * kStageBytes;
constexpr int kOffBar = kOffOut + kEpiWarps * kWarpStageBytes;
constexpr int kSmemBytes = 1024 + kOffBar + 256;  // + alignment slack, barriers
static_assert(kSmemBytes <= 232448, "shared memory over the 227 KiB limit");

struct Params {
    int m, n, k;
    int m_tiles, n_tiles, k_blocks, n_work;
    // K split (small M): work item = (m-tile, n-tile, slice), slice s covering K blocks
    // [s * kb_per_split, (s + 1) * kb_per_split); each slice's f32 tile goes to slice s of a
    // [k_splits][m][n] workspace (omap is then a 3-D map) and split_reduce_kernel sums them.
    int k_splits, kb_per_split;
    void *out;
    int64_t ldo;
    int out_f32;
    const __nv_bfloat16 *res;  // optional residual [m][ldr] bf16
    int64_t ldr;
    DeviceStatus *status;
    uint64_t wait_ns;
};

struct Barriers {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t drain;
    uint64_t res_full[kEpiWarps][4];  // residual block landed in staging buffer b of epilogue warp w
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Barriers) <= 256, "barrier block over its reserved bytes");

// Instruction descriptor, kind::f16: f32 accumulator (bits 4-5 = 1), bf16 A and B (bits 7-9 and
// 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (kBN >> 3) << 17) |
                            ((uint32_t) (kBM >> 4) << 24);

extern __shared__ __align__(1024) uint8_t gemm_smem[];

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return (uint32_t) __bfloat16_as_ushort(h.x) | ((uint32_t) __bfloat16_as_ushort(h.y) << 16);
}

// The two bf16 of a 32-bit word as floats (exact).
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Adds the residual to 32 consecutive outputs of one row (ncol < 32 at the right edge).
__device__ __forceinline__ void add_residual32(const Params &p, int64_t gm, int gn, int ncol, float v[32]) {
    // (Tail loops are unrolled with a predicate so v stays in registers.)
    if (p.res != nullptr) {
        const __nv_bfloat16 *r = p.res + gm * p.ldr + gn;
        if (ncol == 32) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint4 u = *reinterpret_cast<const uint4 *>(r + 8 * i);
                v[8 * i + 0] += bf16_lo(u.x), v[8 * i + 1] += bf16_hi(u.x);
                v[8 * i + 2] += bf16_lo(u.y), v[8 * i + 3] += bf16_hi(u.y);
                v[8 * i + 4] += bf16_lo(u.z), v[8 * i + 5] += bf16_hi(u.z);
                v[8 * i + 6] += bf16_lo(u.w), v[8 * i + 7] += bf16_hi(u.w);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; i++)
                if (i < ncol) v[i] += __bfloat162float(r[i]);
        }
    }
}

// Row `row` (0..31) of a 32 x 32 staging block, rounded once to the output type and written as
// 16-byte chunks in the TMA swizzled layout: f32 rows of 128 B (128-byte swizzle: chunk ^ row % 8),
// bf16 rows of 64 B (64-byte swizzle: chunk ^ (row / 2) % 4). One row per lane is bank-conflict
// free in both.
__device__ __forceinline__ void stage_row32(uint32_t buf, int row, bool f32, const float v[32]) {
    if (f32) {
#pragma unroll
        for (int c = 0; c < 8; c++)
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(buf + (uint32_t) row * 128u +
                                                                           (uint32_t) ((c ^ (row & 7)) << 4)),
                         "f"(v[4 * c]), "f"(v[4 * c + 1]), "f"(v[4 * c + 2]), "f"(v[4 * c + 3])
                         : "memory");
    } else {
#pragma unroll
        for (int c = 0; c < 4; c++)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(buf + (uint32_t) row * 64u +
                                                                           (uint32_t) ((c ^ ((row >> 1) & 3)) << 4)),
                         "r"(bf16x2_bits(v[8 * c], v[8 * c + 1])), "r"(bf16x2_bits(v[8 * c + 2], v[8 * c + 3])),
                         "r"(bf16x2_bits(v[8 * c + 4], v[8 * c + 5])), "r"(bf16x2_bits(v[8 * c + 6], v[8 * c + 7]))
                         : "memory");
    }
}

// Adds row `row` of a bf16 32 x 32 block staged with the 64-byte swizzle to v.
__device__ __forceinline__ void add_staged_bf16_row(uint32_t buf, int row, float v[32]) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint32_t w0, w1, w2, w3;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                     : "r"(buf + (uint32_t) row * 64u + (uint32_t) ((c ^ ((row >> 1) & 3)) << 4))
                     : "memory");
        v[8 * c + 0] += bf16_lo(w0), v[8 * c + 1] += bf16_hi(w0), v[8 * c + 2] += bf16_lo(w1);
        v[8 * c + 3] += bf16_hi(w1), v[8 * c + 4] += bf16_lo(w2), v[8 * c + 5] += bf16_hi(w2);
        v[8 * c + 6] += bf16_lo(w3), v[8 * c + 7] += bf16_hi(w3);
    }
}

// rmap: the residual as bf16 32 x 32 blocks (64-byte swizzle), read by TMA when the output is bf16.
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap amap,
                                                           const __grid_constant__ CUtensorMap bmap,
                                                           const __grid_constant__ CUtensorMap omap,
                                                           const __grid_constant__ CUtensorMap rmap, const Params p) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(gemm_smem) + 1023) & ~uintptr_t(1023));
    Barriers *bars = reinterpret_cast<Barriers *>(base + kOffBar);
    const uint32_t s0 = smem_u32(base);
    volatile int *abort_flag = &bars->abort;

    if (threadIdx.x == 0) {
        bars->abort = 0;
        for (int s = 0; s < kStages; s++) {
            mbar_init(smem_u32(&bars->full[s]), 1);
            mbar_init(smem_u32(&bars->empty[s]), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_u32(&bars->acc_full[b]), 1);
            mbar_init(smem_u32(&bars->acc_empty[b]), kEpiWarps);
        }
        mbar_init(smem_u32(&bars->drain), 1);
        for (int e = 0; e < kEpiWarps; e++)
            for (int b = 0; b < 4; b++) mbar_init(smem_u32(&bars->res_full[e][b]), 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    // Set-up above overlaps the previous kernel (programmatic dependent launch); the operands
    // may come from it.
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        // ---- TMA producer ----
        if (lane == 0) {
            prefetch_tensormap(&amap);
            prefetch_tensormap(&bmap);
            int it = 0;
            bool ok = true;
            for (int w = blockIdx.x; ok && w < p.n_work; w += gridDim.x) {
                const int m0 = (w % p.m_tiles) * kBM, n0 = ((w / p.m_tiles) % p.n_tiles) * kBN;
                const int kb0 = (w / (p.m_tiles * p.n_tiles)) * p.kb_per_split;
                const int kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
                for (int kb = kb0; kb < kb1; kb++, it++) {
                    const int s = it % kStages;
                    const uint32_t use = (uint32_t) (it / kStages);
                    if (use > 0 && !(ok = mbar_wait_bounded(smem_u32(&bars->empty[s]), (use - 1) & 1, abort_flag,
                                                            p.wait_ns)))
                        break;
                    const uint32_t full = smem_u32(&bars->full[s]);
                    const uint32_t sa = s0 + (uint32_t) s * kStageBytes;
                    mbar_arrive_expect_tx(full, kStageBytes);
                    tma_load_2d(sa, &amap, full, kb * kBK, m0);
                    tma_load_2d(sa + kATile, &bmap, full, kb * kBK, n0);
                }
            }
            if (!ok) {
                report(p.status, kStatusTimeout, kSiteGemmWait, 0);
                *abort_flag = 1;
            }
            if (*abort_flag)  // every issued copy lands before shared memory is released
                for (int j = it > kStages ? it - kStages : 0; j < it; j++)
                    mbar_wait_bounded(smem_u32(&bars->full[j % kStages]), (uint32_t) (j / kStages) & 1, nullptr);
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            const uint64_t da = sdesc_sw128(s0, 16, 1024), db = sdesc_sw128(s0 + kATile, 16, 1024);
            const uint32_t la = (uint32_t) da, lb = (uint32_t) db;
            const uint64_t ha = da & 0xFFFFFFFF00000000ull, hb = db & 0xFFFFFFFF00000000ull;
            int it = 0, c = 0;
            bool ok = true, issued = false;
            for (int w = blockIdx.x; ok && w < p.n_work; w += gridDim.x, c++) {
                const int buf = c & 1;
                if (c >= 2 && !(ok = mbar_wait_bounded(smem_u32(&bars->acc_empty[buf]), (uint32_t) ((c >> 1) - 1) & 1,
                                                       abort_flag, p.wait_ns)))
                    break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t) (buf * kBN);
                const int kb0 = (w / (p.m_tiles * p.n_tiles)) * p.kb_per_split;
                const int kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
                for (int kb = kb0; kb < kb1; kb++, it++) {
                    const int s = it % kStages;
                    if (!(ok = mbar_wait_bounded(smem_u32(&bars->full[s]), (uint32_t) (it / kStages) & 1, abort_flag,
                                                 p.wait_ns)))
                        break;
                    tc_fence_after();
                    const uint32_t so = (uint32_t) s * (kStageBytes >> 4);
                    if (kb == kb0) mma_f16_ss_k<0>(d, ha | (la + so), hb | (lb + so), kIdesc);
                    else mma_f16_ss_k<1>(d, ha | (la + so), hb | (lb + so), kIdesc);
#pragma unroll
                    for (int kk = 1; kk < 4; kk++)  // K steps of 16 elements = 32 bytes inside the swizzle row
                        mma_f16_ss_k<1>(d, ha | (la + so + 2 * kk), hb | (lb + so + 2 * kk), kIdesc);
                    mma_commit(smem_u32(&bars->empty[s]));
                    issued = true;
                }
                if (!ok) break;
                mma_commit(smem_u32(&bars->acc_full[buf]));
            }
            if (!ok) {
                report(p.status, kStatusTimeout, kSiteGemmWait, 1);
                *abort_flag = 1;
            }
            if (issued) {  // every MMA completes before tensor memory is released
                mma_commit(smem_u32(&bars->drain));
                mbar_wait_bounded(smem_u32(&bars->drain), 0, nullptr);
            }
        }
    } else {
        // ---- epilogue: one output row per thread, 32 columns per tensor-memory load, out through
        // TMA stores of 32 x 32 blocks staged in this warp's ring of buffers. A bf16 output's
        // residual block is brought into the same buffer by a TMA load one block ahead. ----
        const int quad = warp & 3;
        const int ew = warp - 2;
        const int r = quad * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t) (quad * 32) << 16);
        const uint32_t stage0 = s0 + kOffOut + (uint32_t) ew * kWarpStageBytes;
        const bool f32 = p.out_f32 != 0;
        const bool res_tma = p.res != nullptr && !f32;
        const int nbuf = f32 ? 2 : 4;
        const uint32_t buf_bytes = f32 ? 4096u : 2048u;
        int c = 0, j = 0, n_res = 0;  // tiles seen; blocks staged; residual loads issued (lane 0)
        bool ok = true;
        // Lane 0: residual block of output block jj (columns gn, rows m0 + 32 quad ..) into buffer jj % 4,
        // once the store that last read that buffer (block jj - 4) is done with it.
        auto load_res = [&](int jj, int gn, int m0) {
            tma_store_wait_read_n<2>();
            const uint32_t bar = smem_u32(&bars->res_full[ew][jj & 3]);
            mbar_arrive_expect_tx(bar, 2048);
            tma_load_2d(stage0 + (uint32_t) (jj & 3) * 2048u, &rmap, bar, gn, m0 + quad * 32);
            n_res++;
        };
        for (int w = blockIdx.x; ok && w < p.n_work; w += gridDim.x, c++) {
            const int buf = c & 1;
            const int m0 = (w % p.m_tiles) * kBM;
            const int64_t gm = (int64_t) m0 + r;
            const int n0 = ((w / p.m_tiles) % p.n_tiles) * kBN;
            const int slice = w / (p.m_tiles * p.n_tiles);
            const int nch = min(kBN / 32, (p.n - n0 + 31) / 32);  // column blocks inside the matrix
            if (res_tma && lane == 0 && !*abort_flag) load_res(j, n0, m0);
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&bars->acc_full[buf]), (uint32_t) (c >> 1) & 1,
                                                            abort_flag, p.wait_ns))) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll 1
            for (int ch = 0; ch < kBN / 32; ch++) {
                if (ch >= nch) break;  // warp-uniform: the rest lies right of the matrix (released below)
                const int gn = n0 + ch * 32;
                if (res_tma && lane == 0 && ch + 1 < nch && !*abort_flag) load_res(j + 1, gn + 32, m0);
                float v[32];
                tmem_ld32(lane_base + (uint32_t) (buf * kBN + ch * 32), v);
                tmem_wait_ld();
                if (ch == nch - 1) {  // the accumulator's columns in the matrix are read: the MMAs may reuse it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&bars->acc_empty[buf]));
                }
                const uint32_t sb = stage0 + (uint32_t) (j % nbuf) * buf_bytes;
                if (res_tma) {
                    if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&bars->res_full[ew][j & 3]),
                                                                    (uint32_t) (j >> 2) & 1, abort_flag, p.wait_ns))) {
                        ok = false;
                        break;
                    }
                    add_staged_bf16_row(sb, lane, v);
                } else {
                    if (gm < p.m) add_residual32(p, gm, gn, min(32, p.n - gn), v);
                    if (lane == 0) {  // the store that last read sb (nbuf blocks back) is done with it
                        if (f32) tma_store_wait_read_n<1>();
                        else tma_store_wait_read_n<3>();
                    }
                }
                __syncwarp();
                stage_row32(sb, lane, f32, v);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && !*abort_flag) {  // rows / columns past the matrix are clipped by the store
                    if (p.k_splits > 1) tma_store_3d(&omap, sb, gn, m0 + quad * 32, slice);
                    else tma_store_2d(&omap, sb, gn, m0 + quad * 32);
                    tma_store_commit();
                }
                j++;
            }
        }
        if (lane == 0) {
            // residual loads still in flight land before shared memory is released
            for (int jj = j; jj < n_res; jj++)
                mbar_wait_bounded(smem_u32(&bars->res_full[ew][jj & 3]), (uint32_t) (jj >> 2) & 1, nullptr);
            tma_store_wait_read_n<0>();  // staging buffers are read before the CTA exits
            if (!ok) {
                report(p.status, kStatusTimeout, kSiteGemmWait, warp);
                *abort_flag = 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// Sum of the K split's f32 slices ws [k_splits][m][n] in slice order, plus the optional bf16
// residual, rounded once to the output type (out [m][ldo]). One CTA row per output row (blockIdx.y),
// four columns per thread as 16-byte slice loads (n is a multiple of 4 in a split).
__global__ void __launch_bounds__(256) split_reduce_kernel(const float *ws, int k_splits, int m, int n,
                                                           const __nv_bfloat16 *res, int64_t ldr, void *out,
                                                           int out_f32, int64_t ldo) {
    pdl_wait();
    pdl_launch_dependents();
    const int row = blockIdx.y;
    const int64_t slice = (int64_t) m * n;
    for (int c = (blockIdx.x * blockDim.x + threadIdx.x) * 4; c < n; c += gridDim.x * blockDim.x * 4) {
        const int64_t i = (int64_t) row * n + c;
        float4 v = *reinterpret_cast<const float4 *>(ws + i);
        for (int s = 1; s < k_splits; s++) {
            const float4 u = *reinterpret_cast<const float4 *>(ws + s * slice + i);
            v.x += u.x, v.y += u.y, v.z += u.z, v.w += u.w;
        }
        if (res != nullptr) {
            const uint2 rr = *reinterpret_cast<const uint2 *>(res + (int64_t) row * ldr + c);
            v.x += bf16_lo(rr.x), v.y += bf16_hi(rr.x), v.z += bf16_lo(rr.y), v.w += bf16_hi(rr.y);
        }
        if (out_f32)
            *reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + (int64_t) row * ldo + c) = v;
        else
            *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(out) + (int64_t) row * ldo + c) =
                make_uint2(bf16x2_bits(v.x, v.y), bf16x2_bits(v.z, v.w));
    }
}

// ---- row kernels around the projections ----------------------------------------------------------

// rms(x, gamma) of attn_block (src/qwen3.cpp:112-114): y = x / sqrt(mean(x^2) + eps) * gamma per row,
// one warp per row, f32 sums of squares; bf16 or f32 in, bf16 out.
__global__ void __launch_bounds__(256) rms_norm_kernel(const void *x, int x_f32, int64_t ldx, const float *gamma,
                                                       float eps, __nv_bfloat16 *y, int64_t ldy, int rows, int cols) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= rows) return;
    float ss = 0.f;
    if (x_f32) {
        const float *xr = reinterpret_cast<const float *>(x) + row * ldx;
        for (int c = lane * 4; c < cols; c += 128) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + c);
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    } else {
        const __nv_bfloat16 *xr = reinterpret_cast<const __nv_bfloat16 *>(x) + row * ldx;
        for (int c = lane * 8; c < cols; c += 256) {
            const uint4 u = *reinterpret_cast<const uint4 *>(xr + c);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int j = 0; j < 4; j++) ss += bf16_lo(w[j]) * bf16_lo(w[j]) + bf16_hi(w[j]) * bf16_hi(w[j]);
        }
    }
    ss = warp_sum_xor(ss, 1);
    const float scale = 1.0f / sqrtf(ss / (float) cols + eps);
    __nv_bfloat16 *yr = y + row * ldy;
    if (x_f32) {
        const float *xr = reinterpret_cast<const float *>(x) + row * ldx;
        for (int c = lane * 4; c < cols; c += 128) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + c);
            const float4 g = gamma ? *reinterpret_cast<const float4 *>(gamma + c) : make_float4(1.f, 1.f, 1.f, 1.f);
            *reinterpret_cast<uint2 *>(yr + c) =
                make_uint2(bf16x2_bits(v.x * scale * g.x, v.y * scale * g.y), bf16x2_bits(v.z * scale * g.z, v.w * scale * g.w));
        }
    } else {
        const __nv_bfloat16 *xr = reinterpret_cast<const __nv_bfloat16 *>(x) + row * ldx;
        for (int c = lane * 8; c < cols; c += 256) {
            const uint4 u = *reinterpret_cast<const uint4 *>(xr + c);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
            float g[8];
            if (gamma) {
                const float4 g0 = *reinterpret_cast<const float4 *>(gamma + c), g1 = *reinterpret_cast<const float4 *>(gamma + c + 4);
                g[0] = g0.x, g[1] = g0.y, g[2] = g0.z, g[3] = g0.w, g[4] = g1.x, g[5] = g1.y, g[6] = g1.z, g[7] = g1.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) g[j] = 1.f;
            }
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                o[j] = bf16x2_bits(bf16_lo(w[j]) * scale * g[2 * j], bf16_hi(w[j]) * scale * g[2 * j + 1]);
            *reinterpret_cast<uint4 *>(yr + c) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// f32 -> bf16 copy of a [rows][cols] block (row strides in elements; cols a multiple of 4).
__global__ void __launch_bounds__(256) to_bf16_kernel(const float *x, int64_t ldx, __nv_bfloat16 *y, int64_t ldy,
                                                      int rows, int cols) {
    pdl_wait();
    pdl_launch_dependents();
    const int per_row = cols / 4;
    const int64_t total = (int64_t) rows * per_row;
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t r = i / per_row;
        const int c = (int) (i % per_row) * 4;
        const float4 v = *reinterpret_cast<const float4 *>(x + r * ldx + c);
        *reinterpret_cast<uint2 *>(y + r * ldy + c) = make_uint2(bf16x2_bits(v.x, v.y), bf16x2_bits(v.z, v.w));
    }
}

}  // namespace gemm
}  // namespace lstk
