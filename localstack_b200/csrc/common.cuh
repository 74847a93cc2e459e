// common.cuh - device helpers shared by the attention kernels: the device status word,
// mbarrier operations with bounded waits, TMA tile loads, and small numeric utilities.
// sm_100a only.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lstk {

// ---------------------------------------------------------------------------------------------
// Device status. Kernels never trap: a bounded wait that runs out or an out-of-range index is
// recorded here (first error wins) and the kernel returns cleanly; lstk_cuda_status() reads it.
enum : int { kStatusOk = 0, kStatusTimeout = 1, kStatusBadIndex = 2 };

struct DeviceStatus {
    int code;
    int where;   // kernel-specific site id
    int detail;  // offending value (index, stage, ...)
    int pad;
};

// Where a status was raised (kept in DeviceStatus::where).
enum : int {
    kSiteAppendCell = 1,
    kSiteAppendPos = 2,
    kSiteAppendWait = 3,
    kSiteDecodePage = 10,
    kSiteDecodeLen = 11,
    kSiteDecodeWaitFull = 12,
    kSiteDecodeWaitEmpty = 13,
    kSiteDecodeWaitStart = 14,
    kSiteDecodeWaitMerge = 15,
    kSitePrefillPage = 20,
    kSitePrefillWait = 21,
    kSitePrefillSmem = 22,
    kSitePrefillRows = 23,
    kSitePrefillWaitStart = 24,
    kSiteExchangeWait = 30,
    kSiteGemmWait = 50,
    kSiteGemmSmem = 51,
    kSitePagesSlot = 40,
    kSitePagesTokens = 41,
};

__device__ __forceinline__ void report(DeviceStatus *st, int code, int where, int detail) {
    if (st != nullptr && atomicCAS(&st->code, 0, code) == 0) {
        st->where = where;
        st->detail = detail;
    }
}

// Upper bound for any single wait inside a kernel. Normal waits last microseconds. The pipeline
// waits of the attention kernels take their limit from the launch (default this value); the drain
// waits before a kernel exits always use this one, so no CTA leaves with copies in flight.
constexpr uint64_t kWaitLimitNs = 4ull * 1000 * 1000 * 1000;

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------------------------
// Shared-memory addresses and mbarriers.
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async (TMA / tensor-core) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of the barrier. Gives up (returns false) when *abort becomes
// non-zero or after limit_ns; the caller records the timeout and unwinds.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, const volatile int *abort,
                                                  uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1; i < (1u << 30); i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0) {
            if (abort != nullptr && *abort) return false;
            if (global_timer_ns() - t0 > limit_ns) return false;
        }
    }
    return false;
}

__device__ __forceinline__ int32_t ld_acquire_sys_s32(const int32_t *p) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until *flag != 0 (published by work outside this kernel's stream: another stream, process
// or GPU), bounded like mbar_wait_bounded. Returns false on abort or when limit_ns runs out.
__device__ __forceinline__ bool flag_wait_bounded(const int32_t *flag, const volatile int *abort, uint64_t limit_ns) {
    if (ld_acquire_sys_s32(flag) != 0) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1; i < (1u << 30); i++) {
        if (ld_acquire_sys_s32(flag) != 0) return true;
        if ((i & 63u) == 0) {
            if (abort != nullptr && *abort) return false;
            if (global_timer_ns() - t0 > limit_ns) return false;
        }
    }
    return false;
}

// ---------------------------------------------------------------------------------------------
// TMA: tiled tensor loads global -> shared, completion counted on an mbarrier (single CTA).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(uint32_t dst, const CUtensorMap *map, uint32_t bar, int c0, int c1,
                                                 int c2, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
        "%4, %5}], [%2], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
        : "memory");
}

// L2 policy for data read exactly once (streamed KV pages).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// TMA tiled store shared -> global (bulk group), and the wait until every committed store has
// completed (its shared-memory source may then be reused and its writes are done).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
// Bulk stores: commit the issued ones as a group; wait until every committed group has read its
// shared-memory source (the buffer may then be reused or released). The global writes complete
// asynchronously; they are part of the grid's work, so stream order and griddepcontrol.wait in a
// dependent grid see them.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src), "r"(c0), "r"(c1)
                 : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until at most N committed store groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void tma_store_wait_read_n() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void tma_store_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Pulls the 128-byte line holding p into L2. Only a hint: L2 is where every SM's (and the
// previous kernel's) writes land, so a line prefetched early never makes a later load stale.
__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}

// Programmatic dependent launch. A grid launched with programmatic stream serialization may be
// scheduled before its predecessor in the stream has finished; pdl_wait() blocks until every
// grid it depends on has completed and its memory is visible (a no-op for an ordinary launch),
// so everything a kernel reads from earlier work comes after it. pdl_launch_dependents() lets
// the next such grid be scheduled now (otherwise that happens when this grid completes).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------------------------------------
// Numerics.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float warp_max_xor(float v, int lane_mask_lo) {
    for (int m = lane_mask_lo; m < 32; m <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

__device__ __forceinline__ float warp_sum_xor(float v, int lane_mask_lo) {
    for (int m = lane_mask_lo; m < 32; m <<= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
    return v;
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of 128-byte row `row` inside a 1024-byte
// aligned tile written by TMA with CU_TENSOR_MAP_SWIZZLE_128B: the chunk index is XORed with
// the row index modulo 8.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace lstk
