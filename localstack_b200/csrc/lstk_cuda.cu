// lstk_cuda.cu - the extern "C" entry points of include/lstk_cuda_attn.h: argument validation,
// device binding, TMA tensor-map construction and kernel launches. No allocation, no host sync
// (except lstk_cuda_status, whose job is to synchronise and read the device status word).
#include "common.cuh"
#include "decode.cuh"
#include "exchange.cuh"
#include "gemm.cuh"
#include "host_util.h"
#include "kv_append.cuh"
#include "kv_pages.cuh"
#include "q8_layout.cuh"
#include "prefill.cuh"

#include "lstk_cuda_attn.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

namespace lstk {

// One status word per device that has loaded this library.
__device__ DeviceStatus g_device_status;

namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
    bool ready = false;
    int n_sms = 0;
    DeviceStatus *status = nullptr;
    // Dynamic shared-memory limits raised so far on this device, per kernel (ensure_smem).
    size_t decode_smem = 0;
    size_t decode_q8_smem = 0;
    size_t prefill_smem = 0;
    size_t append_smem[8] = {};  // per kv_append instantiation (append_kernel)
    size_t gemm_smem = 0;
    // Resident kv_append CTAs per SM, per [instantiation][rows per group / 4]; 0 = not asked yet.
    int append_occ[8][append::kMaxGroupRows / 4 + 1] = {};
};

DeviceInfo g_devices[kMaxDevices];
std::mutex g_devices_mu;
thread_local int t_last_device = -1;

// Bounded-wait policy for the decode and prefill launches of this host thread
// (lstk_cuda_set_wait_policy).
thread_local uint64_t t_pipeline_wait_ns = kWaitLimitNs;
thread_local const int32_t *t_start_flag = nullptr;

std::string cuda_msg(const char *what, cudaError_t e) {
    return std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
}

// Makes the device that owns `ptr` current for this runtime and returns its info.
int bind_device(const void *ptr, DeviceInfo **info) {
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
    if (e != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
        cudaGetLastError();
        return set_error(LSTK_ERR_INVALID_ARG, "pointer is not device memory" +
                                                   (e != cudaSuccess ? std::string(": ") + cudaGetErrorName(e) : ""));
    }
    const int dev = attr.device;
    if (dev < 0 || dev >= kMaxDevices) return set_error(LSTK_ERR_UNSUPPORTED, "device ordinal out of range");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != dev && (e = cudaSetDevice(dev)) != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg("cudaSetDevice", e));
    std::lock_guard<std::mutex> lock(g_devices_mu);
    DeviceInfo &d = g_devices[dev];
    if (!d.ready) {
        if ((e = cudaDeviceGetAttribute(&d.n_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return set_error(LSTK_ERR_CUDA, cuda_msg("cudaDeviceGetAttribute", e));
        void *addr = nullptr;
        if ((e = cudaGetSymbolAddress(&addr, g_device_status)) != cudaSuccess)
            return set_error(LSTK_ERR_CUDA, cuda_msg("cudaGetSymbolAddress", e));
        d.status = static_cast<DeviceStatus *>(addr);
        d.ready = true;
    }
    t_last_device = dev;
    *info = &d;
    return LSTK_OK;
}

// Raises `kernel`'s dynamic shared-memory limit on the current device to at least `bytes`, once
// per device (`*have` is the DeviceInfo field that records it). Serialised with the other
// first-use set-up, so host threads making their first calls on a device at once do not race.
template <typename Kernel>
int ensure_smem(size_t *have, Kernel kernel, size_t bytes, const char *what) {
    std::lock_guard<std::mutex> lock(g_devices_mu);
    if (*have >= bytes) return LSTK_OK;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) bytes);
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg(what, e));
    *have = bytes;
    return LSTK_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        cudaGetLastError();
    });
    return fn;
}

// 3-D f16 map over [dim2][dim1][dim0] (dim0 contiguous) with a (box0, box1, box2) box and
// 128-byte swizzle; out-of-range boxes fill zeros.
static int encode_3d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, uint64_t esize, uint64_t dim0,
                     uint64_t dim1, uint64_t dim2, uint32_t box0, uint32_t box1, uint32_t box2) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[3] = {dim0, dim1, dim2};
    const cuuint64_t strides[2] = {dim0 * esize, dim0 * dim1 * esize};
    const cuuint32_t box[3] = {box0, box1, box2};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int) r));
    return LSTK_OK;
}

// 2-D bf16 map over [rows][ld] (k contiguous, `cols` of each row in the tensor) with a
// (64, box_rows) box and the 128-byte swizzle; out-of-range boxes fill zeros.
int encode_bf16_2d(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int) r));
    return LSTK_OK;
}

// 2-D map for the projection's TMA stores: [rows][ld] of bf16 or f32 with a 32 x 32 box in the
// swizzled staging layout (64-byte swizzle for bf16 rows of 64 B, 128-byte for f32 rows of 128 B).
int encode_out_2d(CUtensorMap *map, void *base, bool f32, uint64_t cols, uint64_t rows, uint64_t ld) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const uint64_t es = f32 ? 4 : 2;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * es};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int) r));
    return LSTK_OK;
}

int encode_f16_3d(CUtensorMap *map, const void *base, uint64_t dim0, uint64_t dim1, uint64_t dim2, uint32_t box0,
                  uint32_t box1, uint32_t box2) {
    return encode_3d(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dim0, dim1, dim2, box0, box1, box2);
}

int encode_f32_3d(CUtensorMap *map, const void *base, uint64_t dim0, uint64_t dim1, uint64_t dim2, uint32_t box0,
                  uint32_t box1, uint32_t box2) {
    return encode_3d(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dim0, dim1, dim2, box0, box1, box2);
}

// 2-D map over a q8_0 scale plane [rows][cols] f16 (cols = n_head_kv * 4 scales per cell), box
// (box_cols, 32), no swizzle; out-of-range columns fill zeros.
int encode_scales_2d(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint32_t box_cols) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {box_cols, 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int) r));
    return LSTK_OK;
}

// 3-D map over the projection's K-split workspace [slices][rows][cols] f32 with the store box of
// encode_out_2d (32 x 32, 128-byte swizzle) in one slice: rows past `rows` are clipped per slice.
int encode_3d_f32_out(CUtensorMap *map, void *base, uint64_t cols, uint64_t rows, uint64_t slices) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[3] = {cols, rows, slices};
    const cuuint64_t strides[2] = {cols * 4, cols * rows * 4};
    const cuuint32_t box[3] = {32, 32, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(LSTK_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int) r));
    return LSTK_OK;
}

bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int check_layout(const lstk_kv_layout *L, const char *fn) {
    if (L == nullptr) return set_error(LSTK_ERR_INVALID_ARG, std::string(fn) + ": layout is NULL");
    if (L->head_dim != 128 || L->block_size != 32)
        return set_error(LSTK_ERR_UNSUPPORTED, std::string(fn) + ": kernels implement head_dim 128, block_size 32");
    if (L->n_head_kv <= 0 || L->n_cells <= 0 || L->n_cells % L->block_size != 0 || L->n_cells > (int64_t) INT32_MAX)
        return set_error(LSTK_ERR_INVALID_ARG, std::string(fn) + ": bad layout (n_head_kv, n_cells)");
    return LSTK_OK;
}

int launch_check(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg(what, e));
    return clear_error();
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Decode workspace: [prefix (n_seqs+1) int32][part_lse][part_o], each 256-byte aligned.
size_t decode_ws_prefix_bytes(int32_t n_seqs) { return align_up(sizeof(int32_t) * ((size_t) n_seqs + 1), 256); }
constexpr size_t kDecodePartLseBytes = sizeof(float) * decode::kMaxCtas * 2 * decode::kPartRows;
constexpr size_t kDecodePartOBytes = sizeof(float) * decode::kMaxCtas * 2 * decode::kPartRows * decode::kD;

}  // namespace
}  // namespace lstk

using namespace lstk;

// A cudaLaunchKernelEx result and any launch error, as a status.
static int launch_pdl_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg(what, e));
    return launch_check(what);
}

extern "C" {

int lstk_cuda_status(void *stream) {
    if (t_last_device < 0) return clear_error();
    DeviceInfo &d = g_devices[t_last_device];
    cudaError_t e = cudaSetDevice(t_last_device);
    if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg("lstk_cuda_status", e));
    DeviceStatus st;
    if ((e = cudaMemcpy(&st, d.status, sizeof(st), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return set_error(LSTK_ERR_CUDA, cuda_msg("lstk_cuda_status read", e));
    if (st.code == kStatusOk) return clear_error();
    const DeviceStatus zero = {0, 0, 0, 0};
    cudaMemcpy(d.status, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    char buf[160];
    snprintf(buf, sizeof(buf), "device status: %s at site %d (detail %d)",
             st.code == kStatusTimeout ? "bounded wait timed out" : "index out of range", st.where, st.detail);
    return set_error(st.code == kStatusTimeout ? LSTK_ERR_TIMEOUT : LSTK_ERR_DEVICE_INDEX, buf);
}

int lstk_cuda_set_wait_policy(uint64_t pipeline_wait_ns, const int32_t *start_flag) {
    if (start_flag != nullptr && !aligned(start_flag, 4))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_set_wait_policy: start_flag must be 4-byte aligned");
    t_pipeline_wait_ns = pipeline_wait_ns ? pipeline_wait_ns : kWaitLimitNs;
    t_start_flag = start_flag;
    return clear_error();
}

typedef void (*AppendKernel)(append::Params);
// The kv_append instantiation for bf16 / f32 inputs, an f16 / f32 Q output and a q8_0 / f16
// cache; index bf16 * 4 + q16 * 2 + q8.
static AppendKernel append_kernel(int idx) {
    using namespace append;
    static const AppendKernel k[8] = {kv_append_kernel<false, false, false>, kv_append_kernel<false, false, true>,
                                      kv_append_kernel<false, true, false>,  kv_append_kernel<false, true, true>,
                                      kv_append_kernel<true, false, false>,  kv_append_kernel<true, false, true>,
                                      kv_append_kernel<true, true, false>,   kv_append_kernel<true, true, true>};
    return k[idx];
}

// Resident CTAs per SM of kv_append instantiation `idx` for groups of `rows` rows (two stage
// buffers per warp), asked of the runtime once per device and shape. Returns the count (>= 1) or
// a negative error code.
static int append_occupancy(DeviceInfo *dev, int idx, int rows) {
    int &slot = dev->append_occ[idx][rows / 4];
    {
        std::lock_guard<std::mutex> lock(g_devices_mu);
        if (slot > 0) return slot;
    }
    const int smem = append::smem_bytes(rows, idx >= 4);
    int n = 0;
    const cudaError_t e =
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, append_kernel(idx), append::kWarps * 32, (size_t) smem);
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg("cudaOccupancyMaxActiveBlocksPerMultiprocessor(kv_append)", e));
    if (n < 1) return set_error(LSTK_ERR_CUDA, "kv_append_kernel: no CTA fits on an SM");
    std::lock_guard<std::mutex> lock(g_devices_mu);
    slot = n;
    return n;
}

// The q8_0 planes of a K / V cache pair (lstk_cuda_kv_append_q8, lstk_cuda_attn_decode_q8).
struct Q8Planes {
    void *k_qs, *k_d, *v_qs, *v_d;
};

static int kv_append_impl(const lstk_kv_layout *layout, void *k_cache, void *v_cache, const Q8Planes *q8,
                          const void *q_in, const void *k_in, const void *v_in, int32_t in_dtype,
                          int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride, int32_t n_tokens,
                          int32_t n_head, const int32_t *positions, const int64_t *cells, const float *q_gamma,
                          const float *k_gamma, float eps, const float *rope_table, int32_t rope_n_pos, void *q_out,
                          int32_t q_out_dtype, void *stream) {
    int rc = check_layout(layout, "lstk_cuda_kv_append");
    if (rc) return rc;
    if (n_tokens < 0 || n_head <= 0 || n_head % layout->n_head_kv != 0)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_append: bad n_tokens / n_head");
    if (in_dtype != LSTK_DTYPE_F32 && in_dtype != LSTK_DTYPE_BF16)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_kv_append: in_dtype must be f32 or bf16");
    if (q_out_dtype != LSTK_DTYPE_F32 && q_out_dtype != LSTK_DTYPE_F16)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_kv_append: q_out_dtype must be f32 or f16");
    if (!k_cache || !v_cache || !q_in || !k_in || !v_in || !positions || !cells || !rope_table || !q_out ||
        rope_n_pos <= 0)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_append: NULL pointer or empty rope table");
    const int hd = layout->head_dim;
    if (q_row_stride < (int64_t) n_head * hd || k_row_stride < (int64_t) layout->n_head_kv * hd ||
        v_row_stride < (int64_t) layout->n_head_kv * hd)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_append: row strides too small");
    const int64_t smul = in_dtype == LSTK_DTYPE_BF16 ? 8 : 4;  // rows start on 16-byte boundaries
    if (q_row_stride % smul || k_row_stride % smul || v_row_stride % smul)
        return set_error(LSTK_ERR_INVALID_ARG,
                         "lstk_cuda_kv_append: row strides must be multiples of 16 bytes (4 f32 / 8 bf16 elements)");
    if (!aligned(q_in, 16) || !aligned(k_in, 16) || !aligned(v_in, 16) || !aligned(q_out, 16) ||
        !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(rope_table, 16))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_append: pointers must be 16-byte aligned");
    if (q8 && (!aligned(q8->k_d, 8) || !aligned(q8->v_d, 8)))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_append_q8: scale planes must be 8-byte aligned");
    if (n_tokens == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    if ((rc = bind_device(k_cache, &dev))) return rc;
    append::Params p;
    p.q_in = q_in;
    p.k_in = k_in;
    p.v_in = v_in;
    p.q_stride = q_row_stride;
    p.k_stride = k_row_stride;
    p.v_stride = v_row_stride;
    p.in_bf16 = in_dtype == LSTK_DTYPE_BF16;
    p.n_tokens = n_tokens;
    p.n_head = n_head;
    p.n_head_kv = layout->n_head_kv;
    p.positions = positions;
    p.cells = cells;
    p.q_gamma = q_gamma;
    p.k_gamma = k_gamma;
    p.eps = eps;
    p.rope = reinterpret_cast<const float2 *>(rope_table);
    p.rope_n_pos = rope_n_pos;
    p.k_cache = static_cast<__half *>(k_cache);
    p.v_cache = static_cast<__half *>(v_cache);
    p.n_cells = layout->n_cells;
    p.q_out = q_out;
    p.q_out_f16 = q_out_dtype == LSTK_DTYPE_F16;
    p.k_qs = q8 ? static_cast<int8_t *>(q8->k_qs) : nullptr;
    p.v_qs = q8 ? static_cast<int8_t *>(q8->v_qs) : nullptr;
    p.k_d = q8 ? static_cast<__half *>(q8->k_d) : nullptr;
    p.v_d = q8 ? static_cast<__half *>(q8->v_d) : nullptr;
    p.status = dev->status;
    // Rows per group: the largest (fewest steps and groups per row) that keeps at least four CTAs
    // (16 warps) resident per SM - the warps hide each other's latencies - and gives every resident
    // warp a group; short appends (decode steps), bound by one warp's chain of dependent steps, go
    // down to one step per group.
    const int kidx = (p.in_bf16 ? 4 : 0) + (p.q_out_f16 ? 2 : 0) + (q8 ? 1 : 0);
    if ((rc = ensure_smem(&dev->append_smem[kidx], append_kernel(kidx), append::kSmemBytes,
                          "cudaFuncSetAttribute(kv_append)")))
        return rc;
    const int R = n_head + 2 * layout->n_head_kv;
    int G = 4, gpt = (R + 3) / 4, per_sm = 0;
    for (int cand = p.in_bf16 ? append::kMaxGroupRows : append::kMaxGroupRows / 2; cand >= 4; cand /= 2) {
        gpt = (R + cand - 1) / cand;
        G = ((R + gpt - 1) / gpt + 3) / 4 * 4;  // the token's rows spread evenly over its groups
        if ((per_sm = append_occupancy(dev, kidx, G)) < 0) return per_sm;
        if (per_sm >= 4 && (int64_t) n_tokens * gpt >= (int64_t) dev->n_sms * per_sm * append::kWarps) break;
    }
    p.group_rows = G;
    p.groups_per_token = gpt;
    const int smem_bytes = append::smem_bytes(G, p.in_bf16 != 0);
    const int64_t groups = (int64_t) n_tokens * gpt;
    const int64_t blocks = std::min<int64_t>((groups + append::kWarps - 1) / append::kWarps, (int64_t) dev->n_sms * per_sm);
    if (groups + 3 * blocks * append::kWarps >= INT32_MAX)  // the kernel walks groups in 32-bit indices
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_append: too many rows for one call");
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) blocks);
    cfg.blockDim = dim3(append::kWarps * 32);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return launch_pdl_check(cudaLaunchKernelEx(&cfg, append_kernel(kidx), p), "kv_append_kernel");
}

int lstk_cuda_kv_append(const lstk_kv_layout *layout, void *k_cache, void *v_cache, const void *q_in,
                        const void *k_in, const void *v_in, int32_t in_dtype, int64_t q_row_stride,
                        int64_t k_row_stride, int64_t v_row_stride, int32_t n_tokens, int32_t n_head,
                        const int32_t *positions, const int64_t *cells, const float *q_gamma, const float *k_gamma,
                        float eps, const float *rope_table, int32_t rope_n_pos, void *q_out, int32_t q_out_dtype,
                        void *stream) {
    return kv_append_impl(layout, k_cache, v_cache, nullptr, q_in, k_in, v_in, in_dtype, q_row_stride, k_row_stride,
                          v_row_stride, n_tokens, n_head, positions, cells, q_gamma, k_gamma, eps, rope_table,
                          rope_n_pos, q_out, q_out_dtype, stream);
}

int lstk_cuda_kv_append_q8(const lstk_kv_layout *layout, int8_t *k_qs, void *k_d, int8_t *v_qs, void *v_d,
                           const void *q_in, const void *k_in, const void *v_in, int32_t in_dtype,
                           int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride, int32_t n_tokens,
                           int32_t n_head, const int32_t *positions, const int64_t *cells, const float *q_gamma,
                           const float *k_gamma, float eps, const float *rope_table, int32_t rope_n_pos, void *q_out,
                           int32_t q_out_dtype, void *stream) {
    if (!k_qs || !k_d || !v_qs || !v_d) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_append_q8: NULL plane");
    const Q8Planes q8 = {k_qs, k_d, v_qs, v_d};
    return kv_append_impl(layout, k_qs, v_qs, &q8, q_in, k_in, v_in, in_dtype, q_row_stride, k_row_stride,
                          v_row_stride, n_tokens, n_head, positions, cells, q_gamma, k_gamma, eps, rope_table,
                          rope_n_pos, q_out, q_out_dtype, stream);
}

// Launches the split kernel and the combine kernel with programmatic stream serialization:
// each grid can be scheduled while its predecessor in the stream finishes, and waits for it
// (pdl_wait) before reading anything it produced.
// The cross-rank exchange fused into the combine (lstk_cuda_attn_decode_exchange).
struct ExchangeSpec {
    uint8_t *const *mailboxes;
    int rank, n_ranks;
    uint64_t wait_ns;
};

// kdmap / vdmap: the scale-plane maps of a q8_0 cache (q8 true), else ignored.
static int launch_decode(const CUtensorMap &kmap, const CUtensorMap &vmap, const CUtensorMap &kdmap,
                         const CUtensorMap &vdmap, bool q8, const decode::Params &p, int grid, size_t smem,
                         int n_sms, cudaStream_t s, const ExchangeSpec *ex = nullptr) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) grid);
    cfg.blockDim = dim3(q8 ? decode::SplitCfg<true>::kThreads : decode::SplitCfg<false>::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int rc = q8 ? launch_pdl_check(cudaLaunchKernelEx(&cfg, decode::decode_split_kernel<true>, kmap, vmap, kdmap,
                                                      vdmap, p),
                                   "decode_split_kernel (q8_0)")
                : launch_pdl_check(cudaLaunchKernelEx(&cfg, decode::decode_split_kernel<false>, kmap, vmap, kdmap,
                                                      vdmap, p),
                                   "decode_split_kernel");
    if (rc) return rc;
    decode::CombineParams c;
    c.n_seqs = p.n_seqs;
    c.n_head = p.n_head;
    c.n_head_kv = p.n_head_kv;
    c.group = p.group;
    c.n_hg = p.n_hg;
    c.grid = grid;
    c.prefix = p.prefix;
    c.part_o = p.part_o;
    c.part_lse = p.part_lse;
    c.out = p.out;
    c.lse_out = p.lse_out;
    c.mailboxes = ex ? ex->mailboxes : nullptr;
    c.rank = ex ? ex->rank : 0;
    c.n_ranks = ex ? ex->n_ranks : 1;
    c.wait_ns = ex ? ex->wait_ns : 0;
    c.status = p.status;
    c.dsplit = decode::combine_dsplit(p.n_seqs, p.n_hg, grid, ex != nullptr, exchange::kMaxCtas, n_sms);
    cfg.blockDim = dim3(decode::kCombineThreads);
    cfg.dynamicSmemBytes = 0;
    if (!ex && decode::combine_by_rows(p.n_seqs, p.n_hg, grid)) {
        cfg.gridDim = dim3((unsigned) p.n_seqs, (unsigned) p.n_hg, decode::kHeadsPerGroup);
        return launch_pdl_check(cudaLaunchKernelEx(&cfg, decode::decode_combine_rows_kernel, c),
                                "decode_combine_rows_kernel");
    }
    cfg.gridDim = dim3((unsigned) p.n_seqs, (unsigned) p.n_hg, (unsigned) (decode::kPartRows * c.dsplit));
    if (ex)
        return launch_pdl_check(cudaLaunchKernelEx(&cfg, decode::decode_combine_kernel<true>, c),
                                "decode_combine_kernel (exchange)");
    return launch_pdl_check(cudaLaunchKernelEx(&cfg, decode::decode_combine_kernel<false>, c), "decode_combine_kernel");
}

size_t lstk_cuda_attn_decode_workspace_size(int32_t n_seqs, int32_t n_head, int32_t n_head_kv, int32_t head_dim) {
    (void) n_head;
    (void) n_head_kv;
    (void) head_dim;
    if (n_seqs < 0) return 0;
    return decode_ws_prefix_bytes(n_seqs) + kDecodePartLseBytes + kDecodePartOBytes;
}

static int decode_range(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache, const void *q,
                        int32_t q_dtype, int32_t n_seqs, int32_t n_head, const int32_t *block_tables,
                        int32_t max_blocks_per_seq, const int32_t *seq_lens, int32_t max_seq_len, int32_t kv_begin,
                        int32_t kv_end, float scale, float *out, float *lse_out, void *workspace,
                        size_t workspace_bytes, int32_t n_ctas, void *stream, const ExchangeSpec *ex = nullptr,
                        const Q8Planes *q8 = nullptr) {
    int rc = check_layout(layout, "lstk_cuda_attn_decode");
    if (rc) return rc;
    const int hkv = layout->n_head_kv;
    if (n_seqs < 0 || n_head <= 0 || n_head % hkv != 0 || max_blocks_per_seq <= 0)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode: bad n_seqs / n_head / max_blocks_per_seq");
    const int group = n_head / hkv;
    if (group > decode::kMaxGroup)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_decode: n_head / n_head_kv must be at most 8");
    if (n_seqs > decode::kMaxSeqs)
        return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_decode: more than 4096 sequences in one call");
    if (q_dtype != LSTK_DTYPE_F32 && q_dtype != LSTK_DTYPE_F16)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_decode: q_dtype must be f32 or f16");
    if (!k_cache || !v_cache || !q || !block_tables || !seq_lens || !out || !workspace)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode: NULL pointer");
    if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q, 16) || !aligned(out, 16) ||
        !aligned(workspace, 256))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode: misaligned pointer");
    if (workspace_bytes < lstk_cuda_attn_decode_workspace_size(n_seqs, n_head, hkv, layout->head_dim))
        return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_decode: workspace too small");
    if (max_seq_len <= 0 || max_seq_len > max_blocks_per_seq * layout->block_size)
        max_seq_len = max_blocks_per_seq * layout->block_size;
    if (kv_begin < 0 || kv_end < kv_begin || kv_begin % layout->block_size != 0 ||
        kv_begin > max_blocks_per_seq * layout->block_size)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode_partial: kv_begin must be a page multiple <= kv_end");
    max_seq_len = std::max(0, std::min(max_seq_len, kv_end) - kv_begin);
    if (n_seqs == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    if ((rc = bind_device(k_cache, &dev))) return rc;

    CUtensorMap kmap, vmap, kdmap, vdmap;
    int dpitch = 0;
    if (q8) {
        if (hkv % 2 != 0)
            return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_decode_q8: n_head_kv must be even (16-byte scale rows)");
        if (!aligned(q8->k_qs, 16) || !aligned(q8->v_qs, 16) || !aligned(q8->k_d, 16) || !aligned(q8->v_d, 16))
            return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode_q8: planes must be 16-byte aligned");
        dpitch = std::min(hkv, decode::kHeadsPerGroup) * 8;  // the scale tile's row: 4 f16 per head
        if ((rc = encode_3d(&kmap, q8->k_qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 128, hkv, layout->n_cells, 128, 1, 32)))
            return rc;
        if ((rc = encode_3d(&vmap, q8->v_qs, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 128, hkv, layout->n_cells, 128, 1, 32)))
            return rc;
        if ((rc = encode_scales_2d(&kdmap, q8->k_d, (uint64_t) hkv * 4, layout->n_cells, (uint32_t) dpitch / 2)))
            return rc;
        if ((rc = encode_scales_2d(&vdmap, q8->v_d, (uint64_t) hkv * 4, layout->n_cells, (uint32_t) dpitch / 2)))
            return rc;
    } else {
        if ((rc = encode_f16_3d(&kmap, k_cache, 128, hkv, layout->n_cells, 64, 1, 32))) return rc;
        if ((rc = encode_f16_3d(&vmap, v_cache, 128, hkv, layout->n_cells, 64, 1, 32))) return rc;
        kdmap = kmap;
        vdmap = vmap;
    }

    const int n_hg = (hkv + decode::kHeadsPerGroup - 1) / decode::kHeadsPerGroup;
    const int64_t max_groups = (int64_t) n_seqs * n_hg * ((max_seq_len + decode::kPage - 1) / decode::kPage);
    // q8_0: two CTAs per SM (a slab's dependent chain of int8 MMAs, scales and conversions needs
    // more warps per SM than the f16 kernel to keep HBM busy)
    int64_t grid = n_ctas > 0 ? n_ctas : (q8 ? 2 : 1) * dev->n_sms;
    grid = std::max<int64_t>(1, std::min<int64_t>({grid, max_groups, (int64_t) decode::kMaxCtas}));

    uint8_t *ws = static_cast<uint8_t *>(workspace);
    decode::Params p;
    p.q = q;
    p.q_f16 = q_dtype == LSTK_DTYPE_F16;
    p.block_tables = block_tables;
    p.max_blocks = max_blocks_per_seq;
    p.seq_lens = seq_lens;
    p.kv_page0 = kv_begin / layout->block_size;
    p.kv_end = kv_end;
    p.n_seqs = n_seqs;
    p.n_head = n_head;
    p.n_head_kv = hkv;
    p.group = group;
    p.n_hg = n_hg;
    p.n_pages = layout->n_cells / layout->block_size;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.lse_out = lse_out;
    p.prefix = reinterpret_cast<int32_t *>(ws);
    p.part_lse = reinterpret_cast<float *>(ws + decode_ws_prefix_bytes(n_seqs));
    p.part_o = reinterpret_cast<float *>(ws + decode_ws_prefix_bytes(n_seqs) + kDecodePartLseBytes);
    p.status = dev->status;
    p.wait_ns = t_pipeline_wait_ns;
    p.start_flag = t_start_flag;
    p.q8_dpitch = dpitch;

    const size_t smem = q8 ? decode::split_smem_bytes<true>(n_seqs) : decode::split_smem_bytes<false>(n_seqs);
    if (q8) {
        if ((rc = ensure_smem(&dev->decode_q8_smem, decode::decode_split_kernel<true>, smem,
                              "cudaFuncSetAttribute(decode q8_0)")))
            return rc;
    } else if ((rc = ensure_smem(&dev->decode_smem, decode::decode_split_kernel<false>, smem,
                                 "cudaFuncSetAttribute(decode)"))) {
        return rc;
    }
    return launch_decode(kmap, vmap, kdmap, vdmap, q8 != nullptr, p, (int) grid, smem, dev->n_sms,
                         static_cast<cudaStream_t>(stream), ex);
}

int lstk_cuda_attn_decode(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache, const void *q,
                          int32_t q_dtype, int32_t n_seqs, int32_t n_head, const int32_t *block_tables,
                          int32_t max_blocks_per_seq, const int32_t *seq_lens, int32_t max_seq_len, float scale,
                          float *out, float *lse_out, void *workspace, size_t workspace_bytes, int32_t n_ctas,
                          void *stream) {
    return decode_range(layout, k_cache, v_cache, q, q_dtype, n_seqs, n_head, block_tables, max_blocks_per_seq,
                        seq_lens, max_seq_len, 0, INT32_MAX, scale, out, lse_out, workspace, workspace_bytes, n_ctas,
                        stream);
}

int lstk_cuda_attn_decode_partial(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache,
                                  const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                                  const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *seq_lens,
                                  int32_t max_seq_len, int32_t kv_begin, int32_t kv_end, float scale, float *out,
                                  float *lse_out, void *workspace, size_t workspace_bytes, int32_t n_ctas,
                                  void *stream) {
    return decode_range(layout, k_cache, v_cache, q, q_dtype, n_seqs, n_head, block_tables, max_blocks_per_seq,
                        seq_lens, max_seq_len, kv_begin, kv_end, scale, out, lse_out, workspace, workspace_bytes,
                        n_ctas, stream);
}

int lstk_cuda_attn_decode_exchange(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache,
                                   const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                                   const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *seq_lens,
                                   int32_t max_seq_len, float scale, float *out, float *lse_out, void *workspace,
                                   size_t workspace_bytes, int32_t n_ctas, void *const *mailboxes, int32_t rank,
                                   int32_t n_ranks, uint64_t wait_ns, void *stream) {
    if (!mailboxes || !lse_out || n_ranks <= 0 || rank < 0 || rank >= n_ranks)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode_exchange: bad mailboxes / rank / lse_out");
    // One thread per source raises and awaits its flag; one mailbox epoch counter per combine CTA.
    if (n_ranks > decode::kCombineThreads)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_decode_exchange: at most 256 ranks");
    if (layout && layout->n_head_kv > 0 &&
        (int64_t) n_seqs * ((layout->n_head_kv + decode::kHeadsPerGroup - 1) / decode::kHeadsPerGroup) *
                decode::kPartRows >
            exchange::kMaxCtas)
        return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_decode_exchange: too many sequences x KV heads for the mailbox");
    const ExchangeSpec ex = {reinterpret_cast<uint8_t *const *>(mailboxes), rank, n_ranks,
                             wait_ns ? wait_ns : 1000000000ull};
    return decode_range(layout, k_cache, v_cache, q, q_dtype, n_seqs, n_head, block_tables, max_blocks_per_seq,
                        seq_lens, max_seq_len, 0, INT32_MAX, scale, out, lse_out, workspace, workspace_bytes, n_ctas,
                        stream, &ex);
}

int lstk_cuda_attn_decode_q8(const lstk_kv_layout *layout, const int8_t *k_qs, const void *k_d, const int8_t *v_qs,
                             const void *v_d, const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                             const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *seq_lens,
                             int32_t max_seq_len, float scale, float *out, float *lse_out, void *workspace,
                             size_t workspace_bytes, int32_t n_ctas, void *stream) {
    if (!k_qs || !k_d || !v_qs || !v_d) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode_q8: NULL plane");
    const Q8Planes q8 = {const_cast<int8_t *>(k_qs), const_cast<void *>(k_d), const_cast<int8_t *>(v_qs),
                         const_cast<void *>(v_d)};
    return decode_range(layout, k_qs, v_qs, q, q_dtype, n_seqs, n_head, block_tables, max_blocks_per_seq, seq_lens,
                        max_seq_len, 0, INT32_MAX, scale, out, lse_out, workspace, workspace_bytes, n_ctas, stream,
                        nullptr, &q8);
}

static int launch_pdl(cudaLaunchConfig_t &cfg, cudaLaunchAttribute *attr, cudaStream_t s);

// Copies between ggml's block_q8_0 rows and the q8_0 planes (q8_layout.cuh).
static int q8_convert(const void *src_a, const void *src_b, int64_t n_rows, void *dst_a, void *dst_b, bool to_blocks,
                      void *stream) {
    if (n_rows < 0 || !src_a || !dst_a || (!to_blocks && !dst_b) || (to_blocks && !src_b))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_q8 conversion: bad arguments");
    if (!aligned(src_a, 2) || !aligned(dst_a, 2) || (src_b && !aligned(src_b, 2)) || (dst_b && !aligned(dst_b, 2)))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_q8 conversion: pointers must be 2-byte aligned");
    if (n_rows == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    int rc = bind_device(dst_a, &dev);
    if (rc) return rc;
    const int64_t n_blocks = n_rows * 4;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) std::min<int64_t>((n_blocks * q8::kBlockWords + 255) / 256, (int64_t) dev->n_sms * 16));
    cfg.blockDim = dim3(256);
    launch_pdl(cfg, attr, static_cast<cudaStream_t>(stream));
    if (to_blocks)
        return launch_pdl_check(cudaLaunchKernelEx(&cfg, q8::to_blocks_kernel, static_cast<const uint16_t *>(src_a),
                                                   static_cast<const uint16_t *>(src_b), n_blocks,
                                                   static_cast<uint16_t *>(dst_a)),
                                "q8 to_blocks_kernel");
    return launch_pdl_check(cudaLaunchKernelEx(&cfg, q8::from_blocks_kernel, static_cast<const uint16_t *>(src_a), n_blocks,
                                               static_cast<uint16_t *>(dst_a), static_cast<uint16_t *>(dst_b)),
                            "q8 from_blocks_kernel");
}

int lstk_cuda_q8_from_ggml_blocks(const void *blocks, int64_t n_rows, int8_t *qs, void *d, void *stream) {
    return q8_convert(blocks, nullptr, n_rows, qs, d, false, stream);
}

int lstk_cuda_q8_to_ggml_blocks(const int8_t *qs, const void *d, int64_t n_rows, void *blocks, void *stream) {
    return q8_convert(qs, d, n_rows, blocks, nullptr, true, stream);
}

int lstk_cuda_attn_merge(const float *o_parts, const float *lse_parts, int32_t n_parts, int64_t n_rows,
                         int32_t head_dim, int64_t o_part_stride, int64_t lse_part_stride, float *out,
                         float *lse_out, void *stream) {
    if (!o_parts || !lse_parts || !out || n_parts <= 0 || n_rows < 0 || head_dim <= 0 || o_part_stride < 0 ||
        lse_part_stride < 0)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_merge: bad arguments");
    if (o_part_stride == 0) o_part_stride = n_rows * head_dim;
    if (lse_part_stride == 0) lse_part_stride = n_rows;
    if (o_part_stride < n_rows * head_dim || lse_part_stride < n_rows)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_merge: part stride smaller than a part");
    if (n_rows == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    int rc = bind_device(o_parts, &dev);
    if (rc) return rc;
    const int64_t blocks = (n_rows + 7) / 8;
    decode::lse_merge_kernel<<<(unsigned) blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        o_parts, lse_parts, n_parts, n_rows, head_dim, o_part_stride, lse_part_stride, out, lse_out);
    return launch_check("lse_merge_kernel");
}

size_t lstk_cuda_attn_prefill_workspace_size(int32_t n_seqs, int32_t n_head, int32_t n_head_kv, int32_t head_dim,
                                             int32_t max_q_len, int32_t max_blocks_per_seq, int64_t total_tokens,
                                             int32_t q_dtype) {
    // The launch shape is part of the signature so that a schedule which needs per-launch scratch
    // (partial results of split KV ranges) can size it; the current kernel needs only the f16
    // copy of f32 queries.
    if (n_seqs < 0 || n_head <= 0 || n_head_kv <= 0 || head_dim <= 0 || max_q_len < 0 || max_blocks_per_seq < 0 ||
        total_tokens < 0)
        return 0;
    if (q_dtype == LSTK_DTYPE_F16) return 0;
    return align_up((size_t) total_tokens * n_head * head_dim * 2, 256);
}

int lstk_cuda_attn_prefill(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache, const void *q,
                           int32_t q_dtype, int32_t n_seqs, int32_t n_head, const int32_t *q_seq_start,
                           int32_t max_q_len, int64_t total_tokens, const int32_t *q_pos0, const int32_t *kv_lens,
                           const int32_t *block_tables, int32_t max_blocks_per_seq, float scale, float *out,
                           void *workspace, size_t workspace_bytes, void *stream) {
    int rc = check_layout(layout, "lstk_cuda_attn_prefill");
    if (rc) return rc;
    const int hkv = layout->n_head_kv;
    if (n_seqs < 0 || n_head <= 0 || n_head % hkv != 0 || max_blocks_per_seq <= 0 || max_q_len < 0 ||
        total_tokens < 0 || total_tokens > (int64_t) INT32_MAX)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_prefill: bad sizes");
    const int group = n_head / hkv;
    if (group > 8 || prefill::kBM % group != 0)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_prefill: n_head / n_head_kv must be 1, 2, 4 or 8");
    if (q_dtype != LSTK_DTYPE_F16 && q_dtype != LSTK_DTYPE_F32)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_prefill: q_dtype must be f16 or f32");
    if (!k_cache || !v_cache || !q || !q_seq_start || !q_pos0 || !kv_lens || !block_tables || !out)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_prefill: NULL pointer");
    if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q, 16) || !aligned(out, 16))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_prefill: misaligned pointer");
    if (workspace_bytes < lstk_cuda_attn_prefill_workspace_size(n_seqs, n_head, hkv, layout->head_dim, max_q_len,
                                                                max_blocks_per_seq, total_tokens, q_dtype) ||
        (q_dtype == LSTK_DTYPE_F32 && (!workspace || !aligned(workspace, 256))))
        return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_prefill: workspace too small or misaligned");
    if (n_seqs == 0 || total_tokens == 0 || max_q_len == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    if ((rc = bind_device(k_cache, &dev))) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    const void *q16 = q;
    if (q_dtype == LSTK_DTYPE_F32) {
        const int64_t n = total_tokens * n_head * layout->head_dim;
        const int64_t blocks = std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t) dev->n_sms * 8);
        prefill::q_to_f16_kernel<<<(unsigned) blocks, 256, 0, s>>>(static_cast<const float *>(q),
                                                                    static_cast<__half *>(workspace), n);
        if ((rc = launch_check("q_to_f16_kernel"))) return rc;
        q16 = workspace;
    }

    CUtensorMap qmap, kmap, vmap, omap;
    const int tpt = prefill::kBM / group;
    if ((rc = encode_f16_3d(&qmap, q16, 128, n_head, total_tokens, 64, group, tpt))) return rc;
    if ((rc = encode_f32_3d(&omap, out, 128, n_head, total_tokens, 32, group, tpt))) return rc;
    if ((rc = encode_f16_3d(&kmap, k_cache, 128, hkv, layout->n_cells, 64, 1, 32))) return rc;
    if ((rc = encode_f16_3d(&vmap, v_cache, 128, hkv, layout->n_cells, 64, 1, 32))) return rc;

    prefill::Params p;
    p.n_seqs = n_seqs;
    p.n_head = n_head;
    p.n_head_kv = hkv;
    p.group = group;
    p.n_qt = (max_q_len + tpt - 1) / tpt;
    p.total_tokens = (int) total_tokens;
    p.q_seq_start = q_seq_start;
    p.q_pos0 = q_pos0;
    p.kv_lens = kv_lens;
    p.block_tables = block_tables;
    p.max_blocks = max_blocks_per_seq;
    p.n_pages = layout->n_cells / layout->block_size;
    p.n_cells = layout->n_cells;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.status = dev->status;
    p.wait_ns = t_pipeline_wait_ns;
    p.start_flag = t_start_flag;
    const int64_t n_items = (int64_t) n_seqs * p.n_qt * hkv;
    if (n_items > (int64_t) INT32_MAX) return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_prefill: too many tiles");
    p.n_items = (int) n_items;
    // Persistent: one CTA per SM walks its share of the items (snake order over heaviest-first).
    const int64_t grid = std::min<int64_t>(n_items, dev->n_sms);
    if ((rc = ensure_smem(&dev->prefill_smem, prefill::prefill_kernel, prefill::kSmemBytes,
                          "cudaFuncSetAttribute(prefill)")))
        return rc;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) grid);
    cfg.blockDim = dim3(prefill::kThreads);
    cfg.dynamicSmemBytes = prefill::kSmemBytes;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return launch_pdl_check(cudaLaunchKernelEx(&cfg, prefill::prefill_kernel, qmap, kmap, vmap, omap, p),
                            "prefill_kernel");
}

// Scratch of lstk_cuda_attn_prefill_q8: the compact f16 K and V caches (n_seqs * max_blocks pages)
// and their dense block tables, each 256-byte aligned.
static size_t q8_scratch_cache_bytes(int32_t n_seqs, int32_t max_blocks, int32_t n_head_kv) {
    return align_up((size_t) n_seqs * max_blocks * 32 * n_head_kv * 128 * sizeof(__half), 256);
}

size_t lstk_cuda_q8_prefill_scratch_size(int32_t n_seqs, int32_t max_blocks_per_seq, int32_t n_head_kv) {
    if (n_seqs <= 0 || max_blocks_per_seq <= 0 || n_head_kv <= 0) return 0;
    return 2 * q8_scratch_cache_bytes(n_seqs, max_blocks_per_seq, n_head_kv) +
           align_up(sizeof(int32_t) * (size_t) n_seqs * max_blocks_per_seq, 256);
}

int lstk_cuda_attn_prefill_q8(const lstk_kv_layout *layout, const int8_t *k_qs, const void *k_d, const int8_t *v_qs,
                              const void *v_d, const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                              const int32_t *q_seq_start, int32_t max_q_len, int64_t total_tokens,
                              const int32_t *q_pos0, const int32_t *kv_lens, const int32_t *block_tables,
                              int32_t max_blocks_per_seq, float scale, float *out, void *workspace,
                              size_t workspace_bytes, void *scratch, size_t scratch_bytes, void *stream) {
    int rc = check_layout(layout, "lstk_cuda_attn_prefill_q8");
    if (rc) return rc;
    if (!k_qs || !k_d || !v_qs || !v_d || !kv_lens || !block_tables || !scratch || n_seqs < 0 || max_blocks_per_seq <= 0)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_prefill_q8: bad arguments");
    if (max_blocks_per_seq > 65535 || n_seqs > 65535)
        return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_prefill_q8: more than 65535 sequences or pages per sequence");
    if (!aligned(k_qs, 16) || !aligned(v_qs, 16) || !aligned(k_d, 2) || !aligned(v_d, 2) || !aligned(scratch, 256))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_prefill_q8: misaligned plane or scratch");
    const int hkv = layout->n_head_kv;
    if (scratch_bytes < lstk_cuda_q8_prefill_scratch_size(n_seqs, max_blocks_per_seq, hkv))
        return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_prefill_q8: scratch too small");
    if (n_seqs == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    if ((rc = bind_device(k_qs, &dev))) return rc;
    uint8_t *sc = static_cast<uint8_t *>(scratch);
    const size_t cache_bytes = q8_scratch_cache_bytes(n_seqs, max_blocks_per_seq, hkv);
    __half *k16 = reinterpret_cast<__half *>(sc);
    __half *v16 = reinterpret_cast<__half *>(sc + cache_bytes);
    int32_t *bt16 = reinterpret_cast<int32_t *>(sc + 2 * cache_bytes);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) max_blocks_per_seq, (unsigned) n_seqs);
    cfg.blockDim = dim3(256);
    launch_pdl(cfg, attr, static_cast<cudaStream_t>(stream));
    if ((rc = launch_pdl_check(cudaLaunchKernelEx(&cfg, q8::gather_dequant_kernel, k_qs,
                                                  static_cast<const __half *>(k_d), v_qs,
                                                  static_cast<const __half *>(v_d), hkv,
                                                  (int64_t) (layout->n_cells / layout->block_size), block_tables,
                                                  (int) max_blocks_per_seq, kv_lens, k16, v16, bt16, dev->status),
                               "q8 gather_dequant_kernel")))
        return rc;
    lstk_kv_layout l16 = *layout;
    l16.n_cells = (int64_t) n_seqs * max_blocks_per_seq * 32;
    return lstk_cuda_attn_prefill(&l16, k16, v16, q, q_dtype, n_seqs, n_head, q_seq_start, max_q_len, total_tokens,
                                  q_pos0, kv_lens, bt16, max_blocks_per_seq, scale, out, workspace, workspace_bytes,
                                  stream);
}

static int pages_state(const lstk_kv_pages *st, pages::State *out) {
    if (!st || !st->free_blocks || !st->free_top || !st->block_tables || !st->seq_lens || !st->used_hwm ||
        st->n_slots <= 0 || st->max_blocks <= 0)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_kv_pages: bad state");
    if (st->block_size != pages::kBlock)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_kv_pages: block_size must be 32");
    *out = {st->free_blocks, st->free_top, st->block_tables, st->seq_lens, st->used_hwm, st->n_slots, st->max_blocks};
    return LSTK_OK;
}

int lstk_cuda_kv_alloc(const lstk_kv_pages *state, const int32_t *slots, const int32_t *counts, int32_t n,
                       int32_t max_tokens, int64_t *cells, int32_t *positions, int32_t *ok, void *stream) {
    pages::State st;
    int rc = pages_state(state, &st);
    if (rc) return rc;
    if (n < 0 || max_tokens < 0 || (n > 0 && (!slots || !ok || (max_tokens > 0 && (!cells || !positions)))))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_alloc: bad arguments");
    if (n > pages::kMaxSlots) return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_kv_alloc: more than 2048 slots");
    if (n == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    if ((rc = bind_device(state->block_tables, &dev))) return rc;
    pages::alloc_kernel<<<1, pages::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(st, slots, counts, n, max_tokens,
                                                                                    cells, positions, ok, dev->status);
    return launch_check("alloc_kernel");
}

int lstk_cuda_kv_release(const lstk_kv_pages *state, int32_t slot, int32_t keep, void *stream) {
    pages::State st;
    int rc = pages_state(state, &st);
    if (rc) return rc;
    if (slot < 0 || slot >= state->n_slots) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_kv_release: bad slot");
    DeviceInfo *dev = nullptr;
    if ((rc = bind_device(state->block_tables, &dev))) return rc;
    pages::release_kernel<<<1, pages::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(st, slot, keep);
    return launch_check("release_kernel");
}

size_t lstk_cuda_mailbox_bytes(int32_t n_ranks, int64_t n_rows, int32_t head_dim) {
    if (n_ranks <= 0 || n_rows < 0 || head_dim != exchange::kD) return 0;
    return exchange::mailbox_bytes(n_ranks, n_rows);
}

int lstk_cuda_mailbox_alloc(size_t bytes, void **mailbox, void *ipc_handle) {
    if (!mailbox || !ipc_handle || bytes == 0) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_mailbox_alloc: bad arguments");
    *mailbox = nullptr;
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg("cudaMalloc(mailbox)", e));
    if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess ||
        (e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t *>(ipc_handle), p)) != cudaSuccess) {
        cudaFree(p);
        return set_error(LSTK_ERR_CUDA, cuda_msg("mailbox set-up", e));
    }
    *mailbox = p;
    return clear_error();
}

int lstk_cuda_mailbox_free(void *mailbox) {
    if (!mailbox) return clear_error();
    const cudaError_t e = cudaFree(mailbox);
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg("cudaFree(mailbox)", e));
    return clear_error();
}

int lstk_cuda_mailbox_open(const void *ipc_handle, void **peer_mailbox) {
    if (!ipc_handle || !peer_mailbox) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_mailbox_open: bad arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(peer_mailbox, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg("cudaIpcOpenMemHandle", e));
    return clear_error();
}

int lstk_cuda_mailbox_close(void *peer_mailbox) {
    if (!peer_mailbox) return clear_error();
    const cudaError_t e = cudaIpcCloseMemHandle(peer_mailbox);
    if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg("cudaIpcCloseMemHandle", e));
    return clear_error();
}

int lstk_cuda_attn_exchange_merge(void *const *mailboxes, int32_t rank, int32_t n_ranks, const float *local_o,
                                  const float *local_lse, int64_t n_rows, int32_t head_dim, uint64_t wait_ns,
                                  float *out, float *lse_out, void *stream) {
    if (!mailboxes || !local_o || !local_lse || !out || n_ranks <= 0 || rank < 0 || rank >= n_ranks || n_rows < 0)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_exchange_merge: bad arguments");
    if (head_dim != exchange::kD) return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_exchange_merge: head_dim must be 128");
    // One thread per source raises and awaits its flag.
    if (n_ranks > exchange::kThreads)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_exchange_merge: at most 128 ranks");
    if (n_rows == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    int rc = bind_device(local_o, &dev);
    if (rc) return rc;
    exchange::Params p;
    p.mailboxes = reinterpret_cast<uint8_t *const *>(mailboxes);
    p.rank = rank;
    p.n_ranks = n_ranks;
    p.n_rows = n_rows;
    p.local_o = local_o;
    p.local_lse = local_lse;
    p.wait_ns = wait_ns ? wait_ns : 1000000000ull;
    p.out = out;
    p.lse_out = lse_out;
    p.status = dev->status;
    // Every CTA must be resident at once (they push before they wait): 8 small CTAs per SM.
    const int64_t grid = std::min<int64_t>({n_rows, (int64_t) dev->n_sms * 8, (int64_t) exchange::kMaxCtas});
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) grid);
    cfg.blockDim = dim3(exchange::kThreads);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return launch_pdl_check(cudaLaunchKernelEx(&cfg, exchange::exchange_merge_kernel, p), "exchange_merge_kernel");
}

// ---- projections (tcgen05 GEMM) and the row kernels around them --------------------------------

static int launch_pdl(cudaLaunchConfig_t &cfg, cudaLaunchAttribute *attr, cudaStream_t s) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return LSTK_OK;
}

// K slices for a projection, by a cost model in units of one K block of one tile (~0.42 us on
// B200): rounds of the persistent grid x K blocks per slice, plus the reduce kernel's pass over
// the f32 slices (measured ~3 TB/s: ~1.26 MB per unit). 1 = no split; at most 8 slices, each at
// least 8 K blocks deep; n must be a multiple of 4 (the slices' rows are 16-byte multiples).
static int proj_k_splits(int n_sms, int64_t m, int64_t n, int64_t k) {
    const int64_t tiles = ((m + gemm::kBM - 1) / gemm::kBM) * ((n + gemm::kBN - 1) / gemm::kBN);
    const int64_t kb = (k + gemm::kBK - 1) / gemm::kBK;
    if (n % 4) return 1;
    int best = 1;
    double best_cost = (double) ((tiles + n_sms - 1) / n_sms) * (double) kb;
    for (int s = 2; s <= 8 && kb / s >= 8; s++) {
        const int64_t per = (kb + s - 1) / s;
        const double cost = (double) ((tiles * s + n_sms - 1) / n_sms) * (double) per +
                            (double) s * (double) m * (double) n * 4.0 / 1.26e6;
        if (cost < best_cost) best = s, best_cost = cost;
    }
    return best;
}

size_t lstk_cuda_proj_workspace_size(int32_t m, int32_t n, int32_t k) {
    int dev = 0, n_sms = 0;
    if (m <= 0 || n <= 0 || k <= 0 || cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    const int splits = proj_k_splits(n_sms, m, n, k);
    return splits > 1 ? (size_t) splits * (size_t) m * (size_t) n * sizeof(float) : 0;
}

static int proj_impl(const void *x, int64_t ldx, const void *w, int64_t ldw, int32_t m, int32_t n, int32_t k,
                     const void *residual, int64_t ldr, void *out, int32_t out_dtype, int64_t ldo, void *workspace,
                     size_t workspace_bytes, void *stream) {
    if (m < 0 || n < 0 || k <= 0) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_proj: bad sizes (k must be > 0)");
    if (out_dtype != LSTK_DTYPE_BF16 && out_dtype != LSTK_DTYPE_F32)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_proj: out_dtype must be bf16 or f32");
    if (!x || !w || !out) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_proj: NULL pointer");
    const int64_t oe = out_dtype == LSTK_DTYPE_F32 ? 4 : 2;
    if (ldx < k || ldw < k || ldo < n || (residual && ldr < n))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_proj: leading dimension smaller than the row");
    if (ldx % 8 || ldw % 8 || (ldo * oe) % 16 || (residual && ldr % 8))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_proj: row strides must be multiples of 16 bytes");
    if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16) || (residual && !aligned(residual, 16)))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_proj: pointers must be 16-byte aligned");
    if (m == 0 || n == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    int rc = bind_device(out, &dev);
    if (rc) return rc;
    CUtensorMap amap, bmap, omap;
    if ((rc = encode_bf16_2d(&amap, x, (uint64_t) k, (uint64_t) m, (uint64_t) ldx, gemm::kBM))) return rc;
    if ((rc = encode_bf16_2d(&bmap, w, (uint64_t) k, (uint64_t) n, (uint64_t) ldw, gemm::kBN))) return rc;
    if ((rc = encode_out_2d(&omap, out, out_dtype == LSTK_DTYPE_F32, (uint64_t) n, (uint64_t) m, (uint64_t) ldo)))
        return rc;
    // the residual as TMA blocks (read that way for bf16 outputs); without one, any valid map
    CUtensorMap rmap = omap;
    if (residual && (rc = encode_out_2d(&rmap, const_cast<void *>(residual), false, (uint64_t) n, (uint64_t) m,
                                        (uint64_t) ldr)))
        return rc;
    gemm::Params p;
    p.m = m;
    p.n = n;
    p.k = k;
    p.m_tiles = (m + gemm::kBM - 1) / gemm::kBM;
    p.n_tiles = (n + gemm::kBN - 1) / gemm::kBN;
    p.k_blocks = (k + gemm::kBK - 1) / gemm::kBK;
    const int64_t n_work = (int64_t) p.m_tiles * p.n_tiles;
    if (n_work > INT32_MAX) return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_proj: too many tiles");
    // K split into f32 slices of the workspace when the tiles alone would leave most SMs idle
    const int splits = workspace ? proj_k_splits(dev->n_sms, m, n, k) : 1;
    const bool split = splits > 1 && workspace_bytes >= (size_t) splits * m * n * sizeof(float) &&
                       aligned(workspace, 16);
    p.k_splits = split ? splits : 1;
    p.kb_per_split = split ? (p.k_blocks + splits - 1) / splits : p.k_blocks;
    if (split) {
        p.k_splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;  // no empty slice
        if ((rc = encode_3d_f32_out(&omap, workspace, (uint64_t) n, (uint64_t) m, (uint64_t) p.k_splits))) return rc;
    }
    p.n_work = (int) n_work * p.k_splits;
    p.out = split ? workspace : out;
    p.ldo = split ? n : ldo;
    p.out_f32 = split ? 1 : out_dtype == LSTK_DTYPE_F32;
    p.res = split ? nullptr : static_cast<const __nv_bfloat16 *>(residual);
    p.ldr = ldr;
    p.status = dev->status;
    p.wait_ns = t_pipeline_wait_ns;
    if ((rc = ensure_smem(&dev->gemm_smem, gemm::gemm_kernel, gemm::kSmemBytes, "cudaFuncSetAttribute(gemm)")))
        return rc;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) std::min<int64_t>(p.n_work, dev->n_sms));
    cfg.blockDim = dim3(gemm::kThreads);
    cfg.dynamicSmemBytes = gemm::kSmemBytes;
    launch_pdl(cfg, attr, static_cast<cudaStream_t>(stream));
    rc = launch_pdl_check(cudaLaunchKernelEx(&cfg, gemm::gemm_kernel, amap, bmap, omap, rmap, p), "gemm_kernel");
    if (rc || !split) return rc;
    cudaLaunchConfig_t rcfg = {};
    rcfg.gridDim = dim3((unsigned) ((n / 4 + 255) / 256), (unsigned) m);
    rcfg.blockDim = dim3(256);
    launch_pdl(rcfg, attr, static_cast<cudaStream_t>(stream));
    return launch_pdl_check(cudaLaunchKernelEx(&rcfg, gemm::split_reduce_kernel, static_cast<const float *>(workspace),
                                               p.k_splits, (int) m, (int) n,
                                               static_cast<const __nv_bfloat16 *>(residual), ldr, out,
                                               (int) (out_dtype == LSTK_DTYPE_F32), ldo),
                            "split_reduce_kernel");
}

int lstk_cuda_proj(const void *x, int64_t ldx, const void *w, int64_t ldw, int32_t m, int32_t n, int32_t k,
                   const void *residual, int64_t ldr, void *out, int32_t out_dtype, int64_t ldo, void *stream) {
    return proj_impl(x, ldx, w, ldw, m, n, k, residual, ldr, out, out_dtype, ldo, nullptr, 0, stream);
}

int lstk_cuda_proj_ws(const void *x, int64_t ldx, const void *w, int64_t ldw, int32_t m, int32_t n, int32_t k,
                      const void *residual, int64_t ldr, void *out, int32_t out_dtype, int64_t ldo, void *workspace,
                      size_t workspace_bytes, void *stream) {
    return proj_impl(x, ldx, w, ldw, m, n, k, residual, ldr, out, out_dtype, ldo, workspace, workspace_bytes, stream);
}

int lstk_cuda_rms_norm(const void *x, int32_t x_dtype, int64_t ldx, const float *gamma, float eps, void *y,
                       int64_t ldy, int32_t rows, int32_t cols, void *stream) {
    if (rows < 0 || cols <= 0 || !x || !y) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_rms_norm: bad arguments");
    if (x_dtype != LSTK_DTYPE_BF16 && x_dtype != LSTK_DTYPE_F32)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_rms_norm: x_dtype must be bf16 or f32");
    const int vec = x_dtype == LSTK_DTYPE_BF16 ? 8 : 4;
    if (cols % vec || ldx < cols || ldy < cols || ldx % vec || ldy % 8 || !aligned(x, 16) || !aligned(y, 16) ||
        (gamma && !aligned(gamma, 16)))
        return set_error(LSTK_ERR_INVALID_ARG,
                         "lstk_cuda_rms_norm: rows must be whole 16-byte vectors (cols and strides) and 16-byte aligned");
    if (rows == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    int rc = bind_device(y, &dev);
    if (rc) return rc;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) ((rows + 7) / 8));
    cfg.blockDim = dim3(256);
    launch_pdl(cfg, attr, static_cast<cudaStream_t>(stream));
    return launch_pdl_check(cudaLaunchKernelEx(&cfg, gemm::rms_norm_kernel, x, (int) (x_dtype == LSTK_DTYPE_F32), ldx,
                                               gamma, eps, static_cast<__nv_bfloat16 *>(y), ldy, (int) rows, (int) cols),
                            "rms_norm_kernel");
}

int lstk_cuda_to_bf16(const float *x, int64_t ldx, void *y, int64_t ldy, int32_t rows, int32_t cols, void *stream) {
    if (rows < 0 || cols < 0 || !x || !y) return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_to_bf16: bad arguments");
    if (cols % 4 || ldx < cols || ldy < cols || ldx % 4 || ldy % 4 || !aligned(x, 16) || !aligned(y, 8))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_to_bf16: cols and strides must be multiples of 4, x 16-byte "
                                               "and y 8-byte aligned");
    if (rows == 0 || cols == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    int rc = bind_device(y, &dev);
    if (rc) return rc;
    const int64_t total = (int64_t) rows * (cols / 4);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) std::min<int64_t>((total + 255) / 256, (int64_t) dev->n_sms * 8));
    cfg.blockDim = dim3(256);
    launch_pdl(cfg, attr, static_cast<cudaStream_t>(stream));
    return launch_pdl_check(cudaLaunchKernelEx(&cfg, gemm::to_bf16_kernel, x, ldx, static_cast<__nv_bfloat16 *>(y), ldy,
                                               (int) rows, (int) cols),
                            "to_bf16_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Decode without caller-provided workspace.
//
// Some hosts of this backend cannot call cudaMalloc when they want to run a decode step: an
// inference engine that hands all device memory to its own pool at start-up, a caller running
// inside a context where allocation is forbidden or would synchronise, or an embedding through a
// plain C FFI that only owns the tensors it passes in. For them the split-K scratch of the decode
// kernel lives in a fixed array inside this library instead of a caller buffer.
//
// Scratch layout (the same as lstk_cuda_attn_decode's workspace, for at most
// kStaticMaxSeqs sequences and kStaticMaxCtas CTAs): a page prefix of (n_seqs + 1) int32, then
// per-CTA partial log-sum-exp values and partial outputs. Nothing in it has to start at zero:
// every entry the combine kernel reads is written earlier in the same call.
namespace lstk {
namespace {

constexpr int kStaticMaxSeqs = 1024;
constexpr int kStaticMaxCtas = 160;
constexpr size_t kStaticPrefixBytes = sizeof(int32_t) * (kStaticMaxSeqs + 1 + 63);  // 256-byte multiple
constexpr size_t kStaticLseBytes = sizeof(float) * kStaticMaxCtas * 2 * decode::kPartRows;
constexpr size_t kStaticOBytes = sizeof(float) * kStaticMaxCtas * 2 * decode::kPartRows * decode::kD;
constexpr size_t kStaticScratchBytes = kStaticPrefixBytes + kStaticLseBytes + kStaticOBytes;  // ~5.3 MiB
static_assert(kStaticPrefixBytes % 256 == 0, "prefix region must keep the next regions aligned");

// Loaded onto every device that uses this library and kept until the process exits. In host
// code this name is only a stand-in: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

uint8_t *g_decode_scratch_ptr[kMaxDevices] = {};

}  // namespace
}  // namespace lstk

extern "C" {

int lstk_cuda_attn_decode_static(const lstk_kv_layout *layout, const void *k_cache, const void *v_cache,
                                 const void *q, int32_t q_dtype, int32_t n_seqs, int32_t n_head,
                                 const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *seq_lens,
                                 int32_t max_seq_len, float scale, float *out, float *lse_out, int32_t n_ctas,
                                 void *stream) {
    int rc = check_layout(layout, "lstk_cuda_attn_decode_static");
    if (rc) return rc;
    const int hkv = layout->n_head_kv;
    if (n_seqs < 0 || n_head <= 0 || n_head % hkv != 0 || max_blocks_per_seq <= 0)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode_static: bad n_seqs / n_head / max_blocks");
    if (n_seqs > kStaticMaxSeqs)
        return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_decode_static: at most 1024 sequences per call "
                                            "(the built-in scratch is sized for that); use lstk_cuda_attn_decode "
                                            "with a workspace for larger batches");
    if (n_ctas > kStaticMaxCtas)
        return set_error(LSTK_ERR_CAPACITY, "lstk_cuda_attn_decode_static: at most 160 CTAs");
    const int group = n_head / hkv;
    if (group > decode::kMaxGroup)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_decode_static: n_head / n_head_kv must be at most 8");
    if (q_dtype != LSTK_DTYPE_F32 && q_dtype != LSTK_DTYPE_F16)
        return set_error(LSTK_ERR_UNSUPPORTED, "lstk_cuda_attn_decode_static: q_dtype must be f32 or f16");
    if (!k_cache || !v_cache || !q || !block_tables || !seq_lens || !out)
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode_static: NULL pointer");
    if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(q, 16) || !aligned(out, 16))
        return set_error(LSTK_ERR_INVALID_ARG, "lstk_cuda_attn_decode_static: misaligned pointer");
    if (max_seq_len <= 0 || max_seq_len > max_blocks_per_seq * layout->block_size)
        max_seq_len = max_blocks_per_seq * layout->block_size;
    if (n_seqs == 0) return clear_error();
    DeviceInfo *dev = nullptr;
    if ((rc = bind_device(k_cache, &dev))) return rc;

    // First call on this device (which bind_device made current): resolve the array's device
    // address once, under the same lock as the rest of the first-use set-up, so host threads
    // making their first calls on one device at once do not race on the cached pointer.
    const int dev_id = t_last_device;
    uint8_t *ws = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_devices_mu);
        if (g_decode_scratch_ptr[dev_id] == nullptr) {
            void *addr = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&addr, g_decode_scratch);
            if (e != cudaSuccess) return set_error(LSTK_ERR_CUDA, cuda_msg("cudaGetSymbolAddress(decode scratch)", e));
            g_decode_scratch_ptr[dev_id] = static_cast<uint8_t *>(addr);
        }
        ws = g_decode_scratch_ptr[dev_id];
    }

    CUtensorMap kmap, vmap;
    if ((rc = encode_f16_3d(&kmap, k_cache, 128, hkv, layout->n_cells, 64, 1, 32))) return rc;
    if ((rc = encode_f16_3d(&vmap, v_cache, 128, hkv, layout->n_cells, 64, 1, 32))) return rc;

    const int n_hg = (hkv + decode::kHeadsPerGroup - 1) / decode::kHeadsPerGroup;
    const int64_t max_groups = (int64_t) n_seqs * n_hg * ((max_seq_len + decode::kPage - 1) / decode::kPage);
    int64_t grid = n_ctas > 0 ? n_ctas : dev->n_sms;
    grid = std::max<int64_t>(1, std::min<int64_t>({grid, max_groups, (int64_t) kStaticMaxCtas}));

    decode::Params p;
    p.q = q;
    p.q_f16 = q_dtype == LSTK_DTYPE_F16;
    p.block_tables = block_tables;
    p.max_blocks = max_blocks_per_seq;
    p.seq_lens = seq_lens;
    p.kv_page0 = 0;
    p.kv_end = INT32_MAX;
    p.n_seqs = n_seqs;
    p.n_head = n_head;
    p.n_head_kv = hkv;
    p.group = group;
    p.n_hg = n_hg;
    p.n_pages = layout->n_cells / layout->block_size;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.lse_out = lse_out;
    p.prefix = reinterpret_cast<int32_t *>(ws);
    p.part_lse = reinterpret_cast<float *>(ws + kStaticPrefixBytes);
    p.part_o = reinterpret_cast<float *>(ws + kStaticPrefixBytes + kStaticLseBytes);
    p.status = dev->status;
    p.wait_ns = t_pipeline_wait_ns;
    p.start_flag = t_start_flag;
    p.q8_dpitch = 0;

    const size_t smem = decode::split_smem_bytes<false>(n_seqs);
    if ((rc = ensure_smem(&dev->decode_smem, decode::decode_split_kernel<false>, smem, "cudaFuncSetAttribute(decode)")))
        return rc;
    return launch_decode(kmap, vmap, kmap, vmap, false, p, (int) grid, smem, dev->n_sms,
                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"
