// node.cu - a ggml-compatible front end that runs the reference's own model graph on this backend.
//
// The reference records its model as a ggml graph (src/qwen3.cpp: qwen3_build_graph, attn_block
// at :128-171) over ggml tensors, with the KV cache in ggml tensors managed by KvCache
// (src/kv_cache.cpp). Those two files compile unchanged against the declarations in include/;
// this file implements those declarations: ops record nodes, ggml_build_forward_expand orders
// them, and lstk_node_step() executes the graph on the GPU.
//
// Execution. Every tensor lives in device memory. For each layer's attention node the executor
// recognises the ops attn_block records - RMSNorm and the q_norm / k_norm multiply, rope_ext of
// Q and K, set_rows of K and V into kv.k[l] / kv.v[l], flash_attn_ext over the cache - and runs
// them as two calls of this library's C ABI: lstk_cuda_kv_append (the norm, rope and the f16 page
// writes, fused) and lstk_cuda_attn_decode (one new token) or lstk_cuda_attn_prefill (a prompt
// chunk) over the sequence's block table, which replaces the dense [n_kv x T] mask. The other ops
// (embedding rows, the RMSNorms of the residual stream, projections, SwiGLU FFN, residual adds,
// the output head) run as cuBLAS f32 GEMMs and small elementwise kernels. MoE ops are recorded
// (the file must compile) but not executed: the front end serves dense Qwen2/Qwen3 graphs.
#include "ggml-backend.h"
#include "ggml.h"
#include "gguf_model.h"
#include "kv_cache.h"
#include "qwen3.h"

#include "lstk_cuda_attn.h"
#include "lstk_kv_cache.h"

#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

// ---------------------------------------------------------------------------------------------
// Contexts, tensors, graphs.

struct ggml_context {
    std::vector<ggml_tensor *> tensors;
};

struct ggml_cgraph {
    size_t capacity = 0;
    std::vector<ggml_tensor *> nodes;
    std::unordered_set<ggml_tensor *> seen;
};

struct ggml_backend_buffer {
    ggml_context *ctx;
    void *base;
    size_t size;
};

static size_t type_size(ggml_type t) {
    switch (t) {
        case GGML_TYPE_F16:
        case GGML_TYPE_BF16: return 2;
        case GGML_TYPE_I64: return 8;
        default: return 4;
    }
}

static size_t nbytes(const ggml_tensor *t) {
    size_t n = type_size(t->type);
    for (int d = 0; d < 4; d++) n += (size_t) (t->ne[d] - 1) * t->nb[d];
    return n;
}

static bool contiguous(const ggml_tensor *t) {
    size_t nb = type_size(t->type);
    for (int d = 0; d < 4; d++) {
        if (t->ne[d] > 1 && t->nb[d] != nb) return false;
        nb *= (size_t) t->ne[d];
    }
    return true;
}

static ggml_tensor *new_tensor(ggml_context *ctx, ggml_type type, const int64_t ne[4]) {
    ggml_tensor *t = new ggml_tensor();
    std::memset(t, 0, sizeof(*t));
    t->type = type;
    for (int d = 0; d < 4; d++) t->ne[d] = ne[d];
    t->nb[0] = type_size(type);
    for (int d = 1; d < 4; d++) t->nb[d] = t->nb[d - 1] * (size_t) ne[d - 1];
    ctx->tensors.push_back(t);
    return t;
}

static ggml_tensor *new_op(ggml_context *ctx, ggml_op op, ggml_type type, const int64_t ne[4], ggml_tensor *a,
                           ggml_tensor *b = nullptr, ggml_tensor *c = nullptr, ggml_tensor *d = nullptr) {
    ggml_tensor *t = new_tensor(ctx, type, ne);
    t->op = op;
    t->src[0] = a;
    t->src[1] = b;
    t->src[2] = c;
    t->src[3] = d;
    return t;
}

// A view of `a` (shares its root's storage at a byte offset).
static ggml_tensor *new_view(ggml_context *ctx, ggml_op op, ggml_tensor *a, const int64_t ne[4], const size_t nb[4],
                             size_t offset) {
    ggml_tensor *t = new_tensor(ctx, a->type, ne);
    for (int d = 0; d < 4; d++) t->nb[d] = nb[d];
    t->op = op;
    t->src[0] = a;
    t->view_src = a->view_src ? a->view_src : a;
    t->view_offs = a->view_offs + offset;
    return t;
}

size_t ggml_tensor_overhead(void) { return sizeof(ggml_tensor) + 16; }
ggml_context *ggml_init(ggml_init_params) { return new ggml_context(); }

void ggml_free(ggml_context *ctx) {
    if (!ctx) return;
    for (ggml_tensor *t : ctx->tensors) delete t;
    delete ctx;
}

ggml_tensor *ggml_new_tensor_2d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1) {
    const int64_t ne[4] = {ne0, ne1, 1, 1};
    return new_tensor(ctx, type, ne);
}

ggml_tensor *ggml_format_name(ggml_tensor *tensor, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(tensor->name, sizeof(tensor->name), fmt, ap);
    va_end(ap);
    return tensor;
}

ggml_tensor *ggml_set_name(ggml_tensor *tensor, const char *name) {
    snprintf(tensor->name, sizeof(tensor->name), "%s", name);
    return tensor;
}

void ggml_set_input(ggml_tensor *tensor) { tensor->flags |= 1; }
void ggml_set_output(ggml_tensor *tensor) { tensor->flags |= 2; }
size_t ggml_row_size(ggml_type type, int64_t ne) { return type_size(type) * (size_t) ne; }

ggml_fp16_t ggml_fp32_to_fp16(float x) {
    _Float16 h = (_Float16) x;
    ggml_fp16_t b;
    std::memcpy(&b, &h, 2);
    return b;
}

float ggml_fp16_to_fp32(ggml_fp16_t b) {
    _Float16 h;
    std::memcpy(&h, &b, 2);
    return (float) h;
}

ggml_cgraph *ggml_new_graph_custom(ggml_context *, size_t size, bool) {
    ggml_cgraph *g = new ggml_cgraph();
    g->capacity = size;
    return g;
}

// Post-order (sources before their consumers), each node once.
static void visit(ggml_cgraph *g, ggml_tensor *t) {
    if (t == nullptr || g->seen.count(t)) return;
    g->seen.insert(t);
    for (int i = 0; i < GGML_MAX_SRC; i++) visit(g, t->src[i]);
    if (t->op != GGML_OP_NONE) g->nodes.push_back(t);
}

void ggml_build_forward_expand(ggml_cgraph *cgraph, ggml_tensor *tensor) { visit(cgraph, tensor); }

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(ggml_context *ctx, ggml_backend_t) {
    size_t total = 0;
    for (ggml_tensor *t : ctx->tensors) total += (nbytes(t) + 255) / 256 * 256;
    void *base = nullptr;
    if (cudaMalloc(&base, total ? total : 256) != cudaSuccess) return nullptr;
    size_t off = 0;
    for (ggml_tensor *t : ctx->tensors) {
        t->data = static_cast<uint8_t *>(base) + off;
        off += (nbytes(t) + 255) / 256 * 256;
    }
    ggml_backend_buffer *buf = new ggml_backend_buffer{ctx, base, total};
    for (ggml_tensor *t : ctx->tensors) t->buffer = buf;
    return buf;
}

void ggml_backend_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value) {
    cudaMemset(buffer->base, value, buffer->size);
}

void ggml_backend_buffer_free(ggml_backend_buffer_t buffer) {
    if (!buffer) return;
    cudaFree(buffer->base);
    delete buffer;
}

size_t ggml_backend_buffer_get_size(ggml_backend_buffer_t buffer) { return buffer->size; }

// ---------------------------------------------------------------------------------------------
// Operations: record nodes with ggml's shapes.

ggml_tensor *ggml_get_rows(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    const int64_t ne[4] = {a->ne[0], b->ne[0], 1, 1};
    return new_op(ctx, GGML_OP_GET_ROWS, GGML_TYPE_F32, ne, a, b);
}

ggml_tensor *ggml_rms_norm(ggml_context *ctx, ggml_tensor *a, float eps) {
    ggml_tensor *t = new_op(ctx, GGML_OP_RMS_NORM, GGML_TYPE_F32, a->ne, a);
    std::memcpy(&t->op_params[0], &eps, sizeof(float));
    return t;
}

ggml_tensor *ggml_mul(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    return new_op(ctx, GGML_OP_MUL, GGML_TYPE_F32, a->ne, a, b);
}
ggml_tensor *ggml_add(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    return new_op(ctx, GGML_OP_ADD, GGML_TYPE_F32, a->ne, a, b);
}
ggml_tensor *ggml_div(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    return new_op(ctx, GGML_OP_DIV, GGML_TYPE_F32, a->ne, a, b);
}

ggml_tensor *ggml_mul_mat(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    const int64_t ne[4] = {a->ne[1], b->ne[1], b->ne[2], b->ne[3]};
    return new_op(ctx, GGML_OP_MUL_MAT, GGML_TYPE_F32, ne, a, b);
}

ggml_tensor *ggml_mul_mat_id(ggml_context *ctx, ggml_tensor *as, ggml_tensor *b, ggml_tensor *ids) {
    const int64_t ne[4] = {as->ne[1], ids->ne[0], b->ne[2], 1};
    return new_op(ctx, GGML_OP_MUL_MAT_ID, GGML_TYPE_F32, ne, as, b, ids);
}

ggml_tensor *ggml_reshape_2d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1) {
    const int64_t ne[4] = {ne0, ne1, 1, 1};
    const size_t es = type_size(a->type);
    const size_t nb[4] = {es, es * ne0, es * ne0 * ne1, es * ne0 * ne1};
    return new_view(ctx, GGML_OP_RESHAPE, a, ne, nb, 0);
}

ggml_tensor *ggml_reshape_3d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2) {
    const int64_t ne[4] = {ne0, ne1, ne2, 1};
    const size_t es = type_size(a->type);
    const size_t nb[4] = {es, es * ne0, es * ne0 * ne1, es * ne0 * ne1 * ne2};
    return new_view(ctx, GGML_OP_RESHAPE, a, ne, nb, 0);
}

ggml_tensor *ggml_view_2d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, size_t nb1, size_t offset) {
    const int64_t ne[4] = {ne0, ne1, 1, 1};
    const size_t nb[4] = {a->nb[0], nb1, nb1 * ne1, nb1 * ne1};
    return new_view(ctx, GGML_OP_VIEW, a, ne, nb, offset);
}

ggml_tensor *ggml_view_3d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2, size_t nb1,
                          size_t nb2, size_t offset) {
    const int64_t ne[4] = {ne0, ne1, ne2, 1};
    const size_t nb[4] = {a->nb[0], nb1, nb2, nb2 * ne2};
    return new_view(ctx, GGML_OP_VIEW, a, ne, nb, offset);
}

ggml_tensor *ggml_permute(ggml_context *ctx, ggml_tensor *a, int axis0, int axis1, int axis2, int axis3) {
    const int ax[4] = {axis0, axis1, axis2, axis3};
    int64_t ne[4];
    size_t nb[4];
    for (int d = 0; d < 4; d++) {
        ne[ax[d]] = a->ne[d];
        nb[ax[d]] = a->nb[d];
    }
    ggml_tensor *t = new_view(ctx, GGML_OP_PERMUTE, a, ne, nb, 0);
    for (int d = 0; d < 4; d++) t->op_params[d] = ax[d];
    return t;
}

ggml_tensor *ggml_cont(ggml_context *ctx, ggml_tensor *a) { return new_op(ctx, GGML_OP_CONT, a->type, a->ne, a); }

ggml_tensor *ggml_cpy(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    const size_t nb[4] = {b->nb[0], b->nb[1], b->nb[2], b->nb[3]};
    ggml_tensor *t = new_view(ctx, GGML_OP_CPY, b, b->ne, nb, 0);
    t->src[1] = a;
    return t;
}

ggml_tensor *ggml_rope_ext(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, ggml_tensor *c, int n_dims, int mode,
                           int n_ctx_orig, float freq_base, float freq_scale, float ext_factor, float attn_factor,
                           float beta_fast, float beta_slow) {
    ggml_tensor *t = new_op(ctx, GGML_OP_ROPE, GGML_TYPE_F32, a->ne, a, b, c);
    t->op_params[0] = n_dims;
    t->op_params[1] = mode;
    t->op_params[2] = n_ctx_orig;
    const float f[6] = {freq_base, freq_scale, ext_factor, attn_factor, beta_fast, beta_slow};
    std::memcpy(&t->op_params[3], f, sizeof(f));
    return t;
}

ggml_tensor *ggml_set_rows(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, ggml_tensor *c) {
    const size_t nb[4] = {a->nb[0], a->nb[1], a->nb[2], a->nb[3]};
    ggml_tensor *t = new_view(ctx, GGML_OP_SET_ROWS, a, a->ne, nb, 0);
    t->src[1] = b;
    t->src[2] = c;
    return t;
}

ggml_tensor *ggml_flash_attn_ext(ggml_context *ctx, ggml_tensor *q, ggml_tensor *k, ggml_tensor *v,
                                 ggml_tensor *mask, float scale, float max_bias, float logit_softcap) {
    // q [D, T, Hq] (permuted view), k/v [D, n_kv, Hkv] -> out [D, Hq, T] (contiguous).
    const int64_t ne[4] = {v->ne[0], q->ne[2], q->ne[1], 1};
    ggml_tensor *t = new_op(ctx, GGML_OP_FLASH_ATTN_EXT, GGML_TYPE_F32, ne, q, k, v, mask);
    const float f[3] = {scale, max_bias, logit_softcap};
    std::memcpy(&t->op_params[0], f, sizeof(f));
    return t;
}

void ggml_prec_set_acc(ggml_tensor *a, ggml_prec prec) { a->op_params[3] = (int32_t) prec; }

ggml_tensor *ggml_swiglu_split(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b) {
    return new_op(ctx, GGML_OP_SWIGLU, GGML_TYPE_F32, a->ne, a, b);
}
ggml_tensor *ggml_soft_max(ggml_context *ctx, ggml_tensor *a) {
    return new_op(ctx, GGML_OP_SOFT_MAX, GGML_TYPE_F32, a->ne, a);
}
ggml_tensor *ggml_argsort_top_k(ggml_context *ctx, ggml_tensor *a, int k) {
    const int64_t ne[4] = {k, a->ne[1], a->ne[2], a->ne[3]};
    return new_op(ctx, GGML_OP_ARGSORT_TOP_K, GGML_TYPE_I32, ne, a);
}
ggml_tensor *ggml_sum_rows(ggml_context *ctx, ggml_tensor *a) {
    const int64_t ne[4] = {1, a->ne[1], a->ne[2], a->ne[3]};
    return new_op(ctx, GGML_OP_SUM_ROWS, GGML_TYPE_F32, ne, a);
}
ggml_tensor *ggml_clamp(ggml_context *ctx, ggml_tensor *a, float min, float max) {
    ggml_tensor *t = new_op(ctx, GGML_OP_CLAMP, GGML_TYPE_F32, a->ne, a);
    const float f[2] = {min, max};
    std::memcpy(&t->op_params[0], f, sizeof(f));
    return t;
}

// ---------------------------------------------------------------------------------------------
// GGUF reader: the model file format of llama.cpp (versions 2 and 3): "GGUF", version,
// tensor count, metadata count; typed metadata key/value pairs; the tensor index (name,
// dimensions, ggml type, offset); tensor data from the first multiple of general.alignment
// (default 32) after the index. Written here from the published format; GgufModel's members
// (declared by the reference's gguf_model.h) are served from it, so the reference's own
// qwen3_load_hparams / qwen3_map_weights read real files. Tensors load as f32 (the projections
// run on f32 GEMMs): F32, F16, BF16 and Q8_0 (blocks of 32: an f16 scale and 32 int8) convert;
// other ggml types are refused with their type id.

struct GgufValue {
    uint32_t type = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    bool is_num = false;
};

struct gguf_context {
    uint32_t version = 0;
    std::unordered_map<std::string, GgufValue> kv;
    struct Tensor {
        std::string name;
        uint32_t type = 0;
        int64_t ne[4] = {1, 1, 1, 1};
        uint32_t n_dims = 0;
        uint64_t offset = 0;
    };
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
};

namespace {

enum : uint32_t {  // GGUF metadata value types
    kGgufU8 = 0, kGgufI8, kGgufU16, kGgufI16, kGgufU32, kGgufI32, kGgufF32, kGgufBool, kGgufString,
    kGgufArray, kGgufU64, kGgufI64, kGgufF64
};
constexpr uint32_t kTypeF32 = 0, kTypeF16 = 1, kTypeQ8_0 = 8, kTypeBF16 = 30;  // ggml tensor types

struct Reader {
    std::FILE *f;
    bool ok = true;
    template <class T> T get() {
        T v{};
        if (ok && std::fread(&v, sizeof(T), 1, f) != 1) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 20)) {
            ok = false;
            return {};
        }
        std::string s(n, '\0');
        if (n && std::fread(&s[0], 1, n, f) != n) ok = false;
        return s;
    }
    void skip(uint64_t n) {
        if (ok && std::fseek(f, (long) n, SEEK_CUR) != 0) ok = false;
    }
    // One value of `type`; numbers and strings are kept, arrays skipped element by element.
    GgufValue value(uint32_t type, int depth = 0) {
        GgufValue v;
        v.type = type;
        switch (type) {
        case kGgufU8: v.i = get<uint8_t>(); v.is_num = true; break;
        case kGgufI8: v.i = get<int8_t>(); v.is_num = true; break;
        case kGgufU16: v.i = get<uint16_t>(); v.is_num = true; break;
        case kGgufI16: v.i = get<int16_t>(); v.is_num = true; break;
        case kGgufU32: v.i = get<uint32_t>(); v.is_num = true; break;
        case kGgufI32: v.i = get<int32_t>(); v.is_num = true; break;
        case kGgufBool: v.i = get<uint8_t>(); v.is_num = true; break;
        case kGgufU64: v.i = (int64_t) get<uint64_t>(); v.is_num = true; break;
        case kGgufI64: v.i = get<int64_t>(); v.is_num = true; break;
        case kGgufF32: v.f = get<float>(); v.i = (int64_t) v.f; v.is_num = true; break;
        case kGgufF64: v.f = get<double>(); v.i = (int64_t) v.f; v.is_num = true; break;
        case kGgufString: v.s = str(); break;
        case kGgufArray: {
            const uint32_t et = get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            static const int fixed[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
            if (!ok || et > kGgufF64 || depth > 2) {
                ok = false;
            } else if (et != kGgufString && et != kGgufArray) {
                skip(n * (uint64_t) fixed[et]);
            } else {
                for (uint64_t k = 0; k < n && ok; k++) value(et, depth + 1);
            }
            break;
        }
        default: ok = false;
        }
        if (v.is_num && type != kGgufF32 && type != kGgufF64) v.f = (double) v.i;
        return v;
    }
};

// Row of n values of ggml type `type` -> f32. False for a type this loader does not convert.
bool to_f32(uint32_t type, const uint8_t *src, int64_t n, float *dst) {
    switch (type) {
    case kTypeF32: std::memcpy(dst, src, (size_t) n * 4); return true;
    case kTypeF16:
        for (int64_t i = 0; i < n; i++) dst[i] = ggml_fp16_to_fp32(reinterpret_cast<const uint16_t *>(src)[i]);
        return true;
    case kTypeBF16:
        for (int64_t i = 0; i < n; i++) {
            const uint32_t b = (uint32_t) reinterpret_cast<const uint16_t *>(src)[i] << 16;
            std::memcpy(&dst[i], &b, 4);
        }
        return true;
    case kTypeQ8_0:
        for (int64_t blk = 0; blk < n / 32; blk++) {
            const uint8_t *b = src + blk * 34;
            uint16_t dh;
            std::memcpy(&dh, b, 2);
            const float d = ggml_fp16_to_fp32(dh);
            for (int j = 0; j < 32; j++) dst[blk * 32 + j] = d * (float) (int8_t) b[2 + j];
        }
        return true;
    default: return false;
    }
}

// Bytes of n values of a type this loader converts (0 for others).
size_t type_bytes(uint32_t type, int64_t n) {
    switch (type) {
    case kTypeF32: return (size_t) n * 4;
    case kTypeF16:
    case kTypeBF16: return (size_t) n * 2;
    case kTypeQ8_0: return (size_t) (n / 32) * 34;
    default: return 0;
    }
}

}  // namespace

GgufModel::~GgufModel() { close(); }

void GgufModel::close() {
    delete gguf;
    gguf = nullptr;
    loaded.clear();
}

bool GgufModel::open(const std::string &file, std::string &err) {
    close();
    path = file;
    std::FILE *f = std::fopen(file.c_str(), "rb");
    if (!f) {
        err = "cannot open " + file;
        return false;
    }
    Reader r{f};
    auto *g = new gguf_context();
    const uint32_t magic = r.get<uint32_t>();
    g->version = r.get<uint32_t>();
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || magic != 0x46554747u || (g->version != 2 && g->version != 3) || n_tensors > (1u << 24) ||
        n_kv > (1u << 20)) {
        err = "not a GGUF v2/v3 file: " + file;
        delete g;
        std::fclose(f);
        return false;
    }
    for (uint64_t k = 0; k < n_kv && r.ok; k++) {
        std::string key = r.str();
        const uint32_t type = r.get<uint32_t>();
        GgufValue v = r.value(type);
        if (r.ok) g->kv[key] = v;
    }
    for (uint64_t k = 0; k < n_tensors && r.ok; k++) {
        gguf_context::Tensor t;
        t.name = r.str();
        t.n_dims = r.get<uint32_t>();
        if (t.n_dims > 4) r.ok = false;
        for (uint32_t d = 0; d < t.n_dims && r.ok; d++) t.ne[d] = (int64_t) r.get<uint64_t>();
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        if (r.ok) {
            g->by_name[t.name] = g->tensors.size();
            g->tensors.push_back(t);
        }
    }
    if (!r.ok) {
        err = "truncated or malformed GGUF header: " + file;
        delete g;
        std::fclose(f);
        return false;
    }
    auto al = g->kv.find("general.alignment");
    const uint64_t align = al != g->kv.end() && al->second.is_num && al->second.i > 0 ? (uint64_t) al->second.i : 32;
    const uint64_t pos = (uint64_t) std::ftell(f);
    data_offset = (size_t) ((pos + align - 1) / align * align);
    std::fclose(f);
    gguf = g;
    auto ar = g->kv.find("general.architecture");
    arch = ar != g->kv.end() ? ar->second.s : "";
    return true;
}

bool GgufModel::has(const std::string &key) const { return gguf && gguf->kv.count(key); }

int64_t GgufModel::get_int(const std::string &key, int64_t def) const {
    if (!gguf) return def;
    auto it = gguf->kv.find(key);
    return it != gguf->kv.end() && it->second.is_num ? it->second.i : def;
}

double GgufModel::get_float(const std::string &key, double def) const {
    if (!gguf) return def;
    auto it = gguf->kv.find(key);
    return it != gguf->kv.end() && it->second.is_num ? it->second.f : def;
}

std::string GgufModel::get_str(const std::string &key, const std::string &def) const {
    if (!gguf) return def;
    auto it = gguf->kv.find(key);
    return it != gguf->kv.end() && it->second.type == kGgufString ? it->second.s : def;
}

ggml_tensor *GgufModel::tensor(const std::string &name) const {
    auto it = loaded.find(name);
    return it != loaded.end() ? it->second : nullptr;
}

bool GgufModel::info(const std::string &name, GgufTensorInfo &out) const {
    if (!gguf) return false;
    auto it = gguf->by_name.find(name);
    if (it == gguf->by_name.end()) return false;
    const gguf_context::Tensor &t = gguf->tensors[it->second];
    out.type = (ggml_type) t.type;
    for (int d = 0; d < 4; d++) out.ne[d] = t.ne[d];
    out.file_offset = data_offset + t.offset;
    out.nbytes = type_bytes(t.type, t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3]);
    return true;
}

// Reads every tensor (except skip(name)) as f32 into one device buffer owned by this model.
bool GgufModel::load_all(ggml_backend_t, std::string &err, const std::function<bool(const std::string &)> &skip) {
    if (!gguf) {
        err = "GGUF file not open";
        return false;
    }
    wctx = ggml_init({0, nullptr, true});
    std::vector<std::pair<const gguf_context::Tensor *, ggml_tensor *>> todo;
    for (const auto &t : gguf->tensors) {
        if (skip && skip(t.name)) continue;
        const int64_t n = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
        if (type_bytes(t.type, n) == 0 || (t.type == kTypeQ8_0 && t.ne[0] % 32 != 0)) {
            err = "tensor " + t.name + ": ggml type " + std::to_string(t.type) +
                  " is not supported (F32, F16, BF16, Q8_0)";
            return false;
        }
        if (t.ne[2] != 1 || t.ne[3] != 1) {
            err = "tensor " + t.name + ": more than two dimensions (stacked experts) is not supported";
            return false;
        }
        ggml_tensor *w = ggml_new_tensor_2d(wctx, GGML_TYPE_F32, t.ne[0], t.ne[1]);
        ggml_set_name(w, t.name.c_str());
        todo.emplace_back(&t, w);
    }
    buffer = ggml_backend_alloc_ctx_tensors(wctx, nullptr);
    if (!buffer) {
        err = "device allocation for the weights failed";
        return false;
    }
    std::FILE *f = std::fopen(path.c_str(), "rb");
    if (!f) {
        err = "cannot reopen " + path;
        return false;
    }
    std::vector<uint8_t> raw;
    std::vector<float> conv;
    for (auto &[t, w] : todo) {
        const int64_t n = t->ne[0] * t->ne[1];
        raw.resize(type_bytes(t->type, n));
        conv.resize((size_t) n);
        if (std::fseek(f, (long) (data_offset + t->offset), SEEK_SET) != 0 ||
            std::fread(raw.data(), 1, raw.size(), f) != raw.size()) {
            err = "tensor " + t->name + ": data past the end of the file";
            std::fclose(f);
            return false;
        }
        to_f32(t->type, raw.data(), n, conv.data());
        cudaMemcpy(w->data, conv.data(), conv.size() * 4, cudaMemcpyHostToDevice);
        loaded[t->name] = w;
    }
    std::fclose(f);
    return true;
}

size_t GgufModel::total_bytes() const {
    size_t s = 0;
    if (gguf)
        for (const auto &t : gguf->tensors) s += type_bytes(t.type, t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3]);
    return s;
}

size_t GgufModel::loaded_bytes() const {
    size_t s = 0;
    for (const auto &kv : loaded) s += nbytes(kv.second);
    return s;
}

// ---------------------------------------------------------------------------------------------
// Device kernels for the ops around the attention node (f32).

struct Shape4 {
    int64_t ne[4];
    int64_t nb[4];  // bytes
};

static Shape4 shape_of(const ggml_tensor *t) {
    Shape4 s;
    for (int d = 0; d < 4; d++) {
        s.ne[d] = t->ne[d];
        s.nb[d] = (int64_t) t->nb[d];
    }
    return s;
}

// out (contiguous, shape of a) = a op b, b broadcast along every dimension where it has 1 element.
__global__ void binary_kernel(const uint8_t *a, Shape4 sa, const uint8_t *b, Shape4 sb, float *out, int64_t n, int op) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t r = i, oa = 0, ob = 0;
        for (int d = 0; d < 4; d++) {
            const int64_t id = r % sa.ne[d];
            r /= sa.ne[d];
            oa += id * sa.nb[d];
            ob += (id % sb.ne[d]) * sb.nb[d];
        }
        const float x = *reinterpret_cast<const float *>(a + oa);
        const float y = *reinterpret_cast<const float *>(b + ob);
        out[i] = op == 0 ? x + y : op == 1 ? x * y : x / y;
    }
}

// One block per row of ne0 contiguous floats: y = x / sqrt(mean(x^2) + eps).
__global__ void rms_norm_kernel(const float *x, float *y, int64_t ne0, float eps) {
    const float *xr = x + (int64_t) blockIdx.x * ne0;
    float *yr = y + (int64_t) blockIdx.x * ne0;
    __shared__ float red[32];
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < ne0; i += blockDim.x) s += xr[i] * xr[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) red[0] = s;
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf(red[0] / (float) ne0 + eps);
    for (int64_t i = threadIdx.x; i < ne0; i += blockDim.x) yr[i] = xr[i] * scale;
}

// out[r][:] = a[idx[r]][:] (rows of ne0 elements; a rows at stride a_nb1 bytes, f32).
__global__ void get_rows_kernel(const uint8_t *a, int64_t a_nb1, const int32_t *idx, float *out, int64_t ne0) {
    const float *src = reinterpret_cast<const float *>(a + (int64_t) idx[blockIdx.x] * a_nb1);
    for (int64_t i = threadIdx.x; i < ne0; i += blockDim.x) out[(int64_t) blockIdx.x * ne0 + i] = src[i];
}

__global__ void swiglu_kernel(const float *a, const float *b, float *out, int64_t n) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        const float x = a[i];
        out[i] = x / (1.0f + expf(-x)) * b[i];
    }
}

// Strided copy of any f32 tensor into a contiguous one.
__global__ void cont_kernel(const uint8_t *a, Shape4 sa, float *out, int64_t n) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t r = i, oa = 0;
        for (int d = 0; d < 4; d++) {
            oa += (r % sa.ne[d]) * sa.nb[d];
            r /= sa.ne[d];
        }
        out[i] = *reinterpret_cast<const float *>(a + oa);
    }
}

// ---------------------------------------------------------------------------------------------
// Executor.

namespace {

std::string g_err;

int fail(const std::string &msg) {
    g_err = msg;
    return -1;
}

int64_t nelements(const ggml_tensor *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

// The ops of one layer's attention node, found from its flash_attn_ext (attn_block's structure).
struct AttnNode {
    ggml_tensor *fa = nullptr;
    ggml_tensor *q_src = nullptr, *k_src = nullptr, *v_src = nullptr;  // [D, H, T] projections
    ggml_tensor *q_gamma = nullptr, *k_gamma = nullptr;                // nullptr without QK-norm
    ggml_tensor *q_rope = nullptr;                                     // Q after norm + rope
    ggml_tensor *pos = nullptr, *cells = nullptr;
    ggml_tensor *k_cache = nullptr, *v_cache = nullptr;
    float eps = 1e-6f, freq_base = 1e4f, scale = 1.f;
    std::vector<ggml_tensor *> fused;  // nodes the two C-ABI calls replace
};

// rope(mul(rms_norm(x), gamma)) or rope(x): the projection x, gamma and eps.
bool unwind_qk(ggml_tensor *rope, ggml_tensor **src, ggml_tensor **gamma, float *eps, std::vector<ggml_tensor *> &f) {
    if (rope == nullptr || rope->op != GGML_OP_ROPE) return false;
    f.push_back(rope);
    ggml_tensor *x = rope->src[0];
    *gamma = nullptr;
    if (x->op == GGML_OP_MUL && x->src[0]->op == GGML_OP_RMS_NORM) {
        *gamma = x->src[1];
        std::memcpy(eps, &x->src[0]->op_params[0], sizeof(float));
        f.push_back(x);
        f.push_back(x->src[0]);
        x = x->src[0]->src[0];
    }
    *src = x;
    return true;
}

ggml_tensor *root_of(ggml_tensor *t) { return t->view_src ? t->view_src : t; }

bool match_attention(ggml_cgraph *g, ggml_tensor *fa, AttnNode &a, std::string &why) {
    a.fa = fa;
    std::memcpy(&a.scale, &fa->op_params[0], sizeof(float));
    ggml_tensor *qp = fa->src[0];
    if (qp->op != GGML_OP_PERMUTE) return (why = "flash_attn_ext: Q is not a permuted rope"), false;
    a.q_rope = qp->src[0];
    float eps_q = 0.f, eps_k = 0.f;
    if (!unwind_qk(a.q_rope, &a.q_src, &a.q_gamma, &eps_q, a.fused)) return (why = "Q: no rope_ext"), false;
    a.pos = a.q_rope->src[1];
    std::memcpy(&a.freq_base, &a.q_rope->op_params[3], sizeof(float));
    if (a.q_rope->op_params[1] != GGML_ROPE_TYPE_NEOX || a.q_rope->op_params[0] != 128)
        return (why = "rope_ext: only NEOX over 128 dims is implemented"), false;
    a.k_cache = root_of(fa->src[1]);
    a.v_cache = root_of(fa->src[2]);
    for (ggml_tensor *n : g->nodes) {
        if (n->op != GGML_OP_SET_ROWS) continue;
        ggml_tensor *rows = n->src[1];
        ggml_tensor *inner = rows->op == GGML_OP_VIEW ? rows->src[0] : rows;
        if (root_of(n) == a.k_cache) {
            ggml_tensor *gk = nullptr;
            if (!unwind_qk(inner, &a.k_src, &gk, &eps_k, a.fused)) return (why = "K: no rope_ext"), false;
            a.k_gamma = gk;
            a.cells = n->src[2];
            a.fused.push_back(n);
        } else if (root_of(n) == a.v_cache) {
            a.v_src = inner;
            a.fused.push_back(n);
        }
    }
    if (!a.k_src || !a.v_src) return (why = "set_rows of K / V into the cache not found"), false;
    if ((a.q_gamma == nullptr) != (a.k_gamma == nullptr)) return (why = "QK-norm on only one of Q, K"), false;
    a.eps = a.q_gamma ? eps_q : 1e-6f;
    for (ggml_tensor *t : {a.q_src, a.k_src, a.v_src})
        if (t->type != GGML_TYPE_F32 || !contiguous(t)) return (why = "Q/K/V projections must be contiguous f32"), false;
    return true;
}

}  // namespace

struct lstk_node_model {
    Qwen3HParams hp;
    Qwen3Weights w;
    KvCache kv;
    std::unique_ptr<GgufModel> file;  // weights loaded from a GGUF file (lstk_node_create_gguf)
    ggml_context *wctx = nullptr;
    ggml_backend_buffer_t wbuf = nullptr;
    cublasHandle_t blas = nullptr;
    float *rope = nullptr;  // device RoPE table
    int rope_n_pos = 0;
};

// Runs the graph; copies `result` (f32, contiguous) to `host_out` before the node storage goes.
static int run_graph(lstk_node_model *m, ggml_cgraph *g, int32_t seq, int n_tokens, ggml_tensor *result,
                     float *host_out) {
    // Match every attention node first; their fused ops are skipped below.
    std::unordered_map<ggml_tensor *, AttnNode> attn;
    std::unordered_set<ggml_tensor *> fused;
    for (ggml_tensor *n : g->nodes) {
        if (n->op != GGML_OP_FLASH_ATTN_EXT) continue;
        AttnNode a;
        std::string why;
        if (!match_attention(g, n, a, why)) return fail("attention node not recognised: " + why);
        for (ggml_tensor *f : a.fused) fused.insert(f);
        attn[n] = a;
    }
    // Storage for every node that produces new data (views alias their root).
    size_t total = 0;
    for (ggml_tensor *n : g->nodes)
        if (!n->view_src && !fused.count(n)) total += (nbytes(n) + 255) / 256 * 256;
    void *arena = nullptr;
    if (cudaMalloc(&arena, total + 256) != cudaSuccess) return fail("cudaMalloc(arena) failed");
    size_t off = 0;
    for (ggml_tensor *n : g->nodes)
        if (!n->view_src && !fused.count(n)) {
            n->data = static_cast<uint8_t *>(arena) + off;
            off += (nbytes(n) + 255) / 256 * 256;
        }
    // Block table of the step's sequence (what the mask encodes), for the attention calls.
    std::vector<int32_t> table;
    int32_t len = 0;
    {
        auto it = m->kv.seq_blocks.find(seq);
        if (it != m->kv.seq_blocks.end())
            for (uint32_t b : it->second) table.push_back((int32_t) b);
        len = m->kv.length(seq);
    }
    if (table.empty()) table.push_back(0);
    int32_t *d_table = nullptr, *d_meta = nullptr;
    void *ws = nullptr;
    const int32_t n_head = (int32_t) m->hp.n_head, hkv = (int32_t) m->hp.n_head_kv;
    const size_t ws_dec = lstk_cuda_attn_decode_workspace_size(1, n_head, hkv, 128);
    const size_t ws_pre = lstk_cuda_attn_prefill_workspace_size(1, n_head, hkv, 128, n_tokens, (int32_t) table.size(),
                                                               n_tokens, LSTK_DTYPE_F16);
    void *qbuf = nullptr;  // the appended queries: f16 for the prefill, f32 for the decode
    const size_t qbytes = (size_t) n_tokens * n_head * 128 * 4;
    int rc = 0;
    if (cudaMalloc(&d_table, table.size() * 4) != cudaSuccess || cudaMalloc(&d_meta, 16) != cudaSuccess ||
        cudaMalloc(&ws, std::max(ws_dec, ws_pre) + 256) != cudaSuccess ||
        cudaMalloc(&qbuf, qbytes) != cudaSuccess) {
        rc = fail("cudaMalloc(attention scratch) failed");
    }
    const int pos0 = len - n_tokens;
    const int32_t meta[4] = {0, n_tokens, pos0, len};  // q_seq_start[2], q_pos0, kv_len
    if (!rc) {
        cudaMemcpy(d_table, table.data(), table.size() * 4, cudaMemcpyHostToDevice);
        cudaMemcpy(d_meta, meta, sizeof(meta), cudaMemcpyHostToDevice);
    }
    const lstk_kv_layout layout = {(int64_t) m->kv.size, hkv, 128, 32};
    for (ggml_tensor *n : g->nodes) {
        if (rc) break;
        if (n->view_src) {  // views (also set_rows / cpy results): alias the root
            n->data = static_cast<uint8_t *>(n->view_src->data) + n->view_offs;
            if (n->op == GGML_OP_CPY) rc = fail("cpy is not implemented (MoE graphs only)");
            continue;
        }
        if (fused.count(n)) continue;
        const int64_t ne = nelements(n);
        const unsigned blocks = (unsigned) std::min<int64_t>((ne + 255) / 256, 148 * 32);
        switch (n->op) {
            case GGML_OP_GET_ROWS: {
                ggml_tensor *a = n->src[0], *b = n->src[1];
                if (a->type != GGML_TYPE_F32 || b->type != GGML_TYPE_I32) { rc = fail("get_rows: f32 rows, i32 ids"); break; }
                get_rows_kernel<<<(unsigned) n->ne[1], 256>>>(static_cast<const uint8_t *>(a->data), (int64_t) a->nb[1],
                                                               static_cast<const int32_t *>(b->data),
                                                               static_cast<float *>(n->data), n->ne[0]);
                break;
            }
            case GGML_OP_RMS_NORM: {
                float eps;
                std::memcpy(&eps, &n->op_params[0], sizeof(float));
                if (!contiguous(n->src[0])) { rc = fail("rms_norm: contiguous input expected"); break; }
                rms_norm_kernel<<<(unsigned) (ne / n->ne[0]), 256>>>(static_cast<const float *>(n->src[0]->data),
                                                                     static_cast<float *>(n->data), n->ne[0], eps);
                break;
            }
            case GGML_OP_ADD:
            case GGML_OP_MUL:
            case GGML_OP_DIV:
                binary_kernel<<<blocks, 256>>>(static_cast<const uint8_t *>(n->src[0]->data), shape_of(n->src[0]),
                                               static_cast<const uint8_t *>(n->src[1]->data), shape_of(n->src[1]),
                                               static_cast<float *>(n->data), ne,
                                               n->op == GGML_OP_ADD ? 0 : n->op == GGML_OP_MUL ? 1 : 2);
                break;
            case GGML_OP_MUL_MAT: {
                ggml_tensor *a = n->src[0], *b = n->src[1];
                if (a->type != GGML_TYPE_F32 || b->type != GGML_TYPE_F32 || !contiguous(a) || !contiguous(b) ||
                    b->ne[2] != 1 || b->ne[3] != 1) {
                    rc = fail("mul_mat: contiguous 2-D f32 operands expected");
                    break;
                }
                // out[n][m] = sum_k a[m][k] b[n][k]: column-major C(M x N) = A^T(M x K) B(K x N).
                const int M = (int) a->ne[1], N = (int) b->ne[1], K = (int) a->ne[0];
                const float one = 1.f, zero = 0.f;
                if (cublasSgemm(m->blas, CUBLAS_OP_T, CUBLAS_OP_N, M, N, K, &one, static_cast<const float *>(a->data),
                                K, static_cast<const float *>(b->data), K, &zero, static_cast<float *>(n->data),
                                M) != CUBLAS_STATUS_SUCCESS)
                    rc = fail("cublasSgemm failed");
                break;
            }
            case GGML_OP_SWIGLU:
                if (!contiguous(n->src[0]) || !contiguous(n->src[1])) { rc = fail("swiglu: contiguous inputs"); break; }
                swiglu_kernel<<<blocks, 256>>>(static_cast<const float *>(n->src[0]->data),
                                               static_cast<const float *>(n->src[1]->data),
                                               static_cast<float *>(n->data), ne);
                break;
            case GGML_OP_CONT:
                if (n->src[0]->type != GGML_TYPE_F32) { rc = fail("cont: f32 only"); break; }
                cont_kernel<<<blocks, 256>>>(static_cast<const uint8_t *>(n->src[0]->data), shape_of(n->src[0]),
                                             static_cast<float *>(n->data), ne);
                break;
            case GGML_OP_FLASH_ATTN_EXT: {
                const AttnNode &a = attn[n];
                const int T = (int) a.q_src->ne[2];
                if (T != n_tokens) { rc = fail("attention: token count mismatch"); break; }
                // lstk_cuda_kv_append: QK-RMSNorm, NEOX RoPE, f16 K/V into the step's cells.
                const bool prefill = T > 1;
                int r = lstk_cuda_kv_append(&layout, a.k_cache->data, a.v_cache->data, a.q_src->data, a.k_src->data,
                                            a.v_src->data, LSTK_DTYPE_F32, n_head * 128, hkv * 128, hkv * 128, T,
                                            n_head, static_cast<const int32_t *>(a.pos->data),
                                            static_cast<const int64_t *>(a.cells->data),
                                            a.q_gamma ? static_cast<const float *>(a.q_gamma->data) : nullptr,
                                            a.k_gamma ? static_cast<const float *>(a.k_gamma->data) : nullptr, a.eps,
                                            m->rope, m->rope_n_pos, qbuf, prefill ? LSTK_DTYPE_F16 : LSTK_DTYPE_F32,
                                            nullptr);
                if (r) { rc = fail(std::string("lstk_cuda_kv_append: ") + lstk_cuda_last_error()); break; }
                if (prefill) {
                    r = lstk_cuda_attn_prefill(&layout, a.k_cache->data, a.v_cache->data, qbuf, LSTK_DTYPE_F16, 1,
                                               n_head, d_meta, T, T, d_meta + 2, d_meta + 3, d_table,
                                               (int32_t) table.size(), a.scale, static_cast<float *>(n->data), ws,
                                               std::max(ws_dec, ws_pre) + 256, nullptr);
                } else {
                    r = lstk_cuda_attn_decode(&layout, a.k_cache->data, a.v_cache->data, qbuf, LSTK_DTYPE_F32, 1,
                                              n_head, d_table, (int32_t) table.size(), d_meta + 3, len, a.scale,
                                              static_cast<float *>(n->data), nullptr, ws, std::max(ws_dec, ws_pre) + 256,
                                              0, nullptr);
                }
                if (r) rc = fail(std::string("attention: ") + lstk_cuda_last_error());
                break;
            }
            default:
                rc = fail("op not implemented by the front end (MoE graph?)");
        }
        if (!rc && cudaGetLastError() != cudaSuccess) rc = fail("kernel launch failed");
    }
    if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = fail("device error while running the graph");
    if (!rc && lstk_cuda_status(nullptr) != LSTK_OK) rc = fail(std::string("device status: ") + lstk_cuda_last_error());
    if (!rc && cudaMemcpy(host_out, result->data, (size_t) nelements(result) * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = fail("copying the result failed");
    cudaFree(arena);
    cudaFree(d_table);
    cudaFree(d_meta);
    cudaFree(ws);
    cudaFree(qbuf);
    return rc;
}

// ---------------------------------------------------------------------------------------------
// C entry points for the harness (no counterpart in the reference: its Engine drives ggml's
// scheduler instead).

extern "C" {

const char *lstk_node_last_error(void) { return g_err.c_str(); }

// Dense Qwen3 (or Qwen2 with qk_norm = 0) with f32 weights given in host memory, in this order:
// tok_embd [n_vocab][n_embd], output_norm [n_embd], output [n_vocab][n_embd], then per layer
// attn_norm [n_embd], wq [Hq*128][n_embd], wk [Hkv*128][n_embd], wv [Hkv*128][n_embd],
// wo [n_embd][Hq*128], q_norm [128], k_norm [128] (if qk_norm), ffn_norm [n_embd],
// ffn_gate [n_ff][n_embd], ffn_up [n_ff][n_embd], ffn_down [n_embd][n_ff] (ggml row order: a
// weight [rows][cols] is the ggml tensor [cols, rows]). head_dim is 128.
lstk_node_model *lstk_node_create(int n_layer, int n_embd, int n_ff, int n_head, int n_head_kv, int n_vocab,
                                  int kv_size, float rope_base, float rms_eps, int qk_norm, const float *const *weights) {
    lstk_node_model *m = new lstk_node_model();
    Qwen3HParams &hp = m->hp;
    hp.n_layer = n_layer;
    hp.n_embd = n_embd;
    hp.n_ff = n_ff;
    hp.n_head = n_head;
    hp.n_head_kv = n_head_kv;
    hp.head_dim = 128;
    hp.n_vocab = n_vocab;
    hp.n_ctx_train = kv_size;
    hp.rms_eps = rms_eps;
    hp.rope_freq_base = rope_base;
    m->wctx = ggml_init({0, nullptr, true});
    std::vector<ggml_tensor *> order;
    auto W = [&](int64_t cols, int64_t rows) {
        ggml_tensor *t = ggml_new_tensor_2d(m->wctx, GGML_TYPE_F32, cols, rows);
        order.push_back(t);
        return t;
    };
    m->w.tok_embd = W(n_embd, n_vocab);
    m->w.output_norm = W(n_embd, 1);
    m->w.output = W(n_embd, n_vocab);
    m->w.layers.resize(n_layer);
    for (int l = 0; l < n_layer; l++) {
        Qwen3Layer &L = m->w.layers[l];
        L.attn_norm = W(n_embd, 1);
        L.wq = W(n_embd, (int64_t) n_head * 128);
        L.wk = W(n_embd, (int64_t) n_head_kv * 128);
        L.wv = W(n_embd, (int64_t) n_head_kv * 128);
        L.wo = W((int64_t) n_head * 128, n_embd);
        if (qk_norm) {
            L.q_norm = W(128, 1);
            L.k_norm = W(128, 1);
        }
        L.ffn_norm = W(n_embd, 1);
        L.ffn_gate = W(n_embd, n_ff);
        L.ffn_up = W(n_embd, n_ff);
        L.ffn_down = W(n_ff, n_embd);
    }
    m->wbuf = ggml_backend_alloc_ctx_tensors(m->wctx, nullptr);
    std::string err;
    if (!m->wbuf || cublasCreate(&m->blas) != CUBLAS_STATUS_SUCCESS ||
        !m->kv.init(nullptr, n_layer, n_head_kv * 128, n_head_kv * 128, kv_size, GGML_TYPE_F16, err)) {
        g_err = "model set-up failed " + err;
        delete m;
        return nullptr;
    }
    cublasSetMathMode(m->blas, CUBLAS_PEDANTIC_MATH);
    for (size_t i = 0; i < order.size(); i++)
        cudaMemcpy(order[i]->data, weights[i], nbytes(order[i]), cudaMemcpyHostToDevice);
    m->rope_n_pos = kv_size;
    std::vector<float> rope(lstk_rope_table_bytes(kv_size, 128) / sizeof(float));
    lstk_rope_table_fill(rope.data(), kv_size, 128, rope_base, 1.0f);
    cudaMalloc(&m->rope, rope.size() * sizeof(float));
    cudaMemcpy(m->rope, rope.data(), rope.size() * sizeof(float), cudaMemcpyHostToDevice);
    return m;
}

void lstk_node_destroy(lstk_node_model *m) {
    if (!m) return;
    if (m->blas) cublasDestroy(m->blas);
    cudaFree(m->rope);
    ggml_backend_buffer_free(m->wbuf);
    ggml_free(m->wctx);
    if (m->file) {
        ggml_backend_buffer_free(m->file->buffer);
        ggml_free(m->file->wctx);
    }
    delete m;
}

// A dense Qwen3 / Qwen2 model from a GGUF file: the reference's own qwen3_load_hparams and
// qwen3_map_weights (src/qwen3.cpp:16-90) read it through GgufModel; head_dim 128, no experts.
lstk_node_model *lstk_node_create_gguf(const char *path, int kv_size) {
    std::unique_ptr<lstk_node_model> m(new lstk_node_model());
    m->file.reset(new GgufModel());
    std::string err;
    if (!m->file->open(path ? path : "", err) || !m->file->load_all(nullptr, err) ||
        !qwen3_load_hparams(*m->file, m->hp, err)) {
        g_err = err;
        return nullptr;
    }
    if (m->hp.moe() || m->hp.head_dim != 128) {
        g_err = "the front end runs dense models with head_dim 128";
        return nullptr;
    }
    if (!qwen3_map_weights(*m->file, m->hp, m->w, false, err)) {
        g_err = err;
        return nullptr;
    }
    if (cublasCreate(&m->blas) != CUBLAS_STATUS_SUCCESS ||
        !m->kv.init(nullptr, m->hp.n_layer, m->hp.n_head_kv * 128, m->hp.n_head_kv * 128, kv_size, GGML_TYPE_F16,
                    err)) {
        g_err = "model set-up failed " + err;
        return nullptr;
    }
    cublasSetMathMode(m->blas, CUBLAS_PEDANTIC_MATH);
    m->rope_n_pos = kv_size;
    std::vector<float> rope(lstk_rope_table_bytes(kv_size, 128) / sizeof(float));
    lstk_rope_table_fill(rope.data(), kv_size, 128, m->hp.rope_freq_base, 1.0f);
    cudaMalloc(&m->rope, rope.size() * sizeof(float));
    cudaMemcpy(m->rope, rope.data(), rope.size() * sizeof(float), cudaMemcpyHostToDevice);
    return m.release();
}

// One engine step for sequence `seq`: its next n_tokens tokens. Follows Engine::make_step_inputs
// (src/engine.cpp:200-243): n_kv from the cache high-water mark, cells and positions from
// KvCache::alloc, the mask from KvCache::fill_mask; then the reference's qwen3_build_graph records
// the model and the graph runs here. Writes the last token's logits [n_vocab].
int lstk_node_step(lstk_node_model *m, int32_t seq, const int32_t *tokens, int n_tokens, float *logits) {
    const int n_kv = lstk_n_kv_for(m->kv.size, (int32_t) m->kv.used_hwm + n_tokens);
    std::vector<int64_t> cells;
    std::vector<int32_t> pos;
    if (!m->kv.alloc(seq, n_tokens, cells, pos)) return fail("KV cache full");
    std::vector<ggml_fp16_t> mask((size_t) n_kv * n_tokens);
    m->kv.fill_mask(seq, pos.data(), n_tokens, n_kv, mask.data());
    ggml_context *ctx = ggml_init({0, nullptr, true});
    Qwen3StepInputs in;
    in.tokens = ggml_new_tensor_2d(ctx, GGML_TYPE_I32, n_tokens, 1);
    in.pos = ggml_new_tensor_2d(ctx, GGML_TYPE_I32, n_tokens, 1);
    in.kv_idxs = ggml_new_tensor_2d(ctx, GGML_TYPE_I64, n_tokens, 1);
    in.mask = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, n_kv, n_tokens);
    in.out_ids = ggml_new_tensor_2d(ctx, GGML_TYPE_I32, 1, 1);
    ggml_backend_buffer_t ibuf = ggml_backend_alloc_ctx_tensors(ctx, nullptr);
    if (!ibuf) {
        ggml_free(ctx);
        return fail("input allocation failed");
    }
    const int32_t out_id = n_tokens - 1;
    cudaMemcpy(in.tokens->data, tokens, 4 * (size_t) n_tokens, cudaMemcpyHostToDevice);
    cudaMemcpy(in.pos->data, pos.data(), 4 * (size_t) n_tokens, cudaMemcpyHostToDevice);
    cudaMemcpy(in.kv_idxs->data, cells.data(), 8 * (size_t) n_tokens, cudaMemcpyHostToDevice);
    cudaMemcpy(in.mask->data, mask.data(), 2 * mask.size(), cudaMemcpyHostToDevice);
    cudaMemcpy(in.out_ids->data, &out_id, 4, cudaMemcpyHostToDevice);
    std::vector<ggml_tensor *> selected;
    ggml_tensor *out = nullptr;
    ggml_cgraph *g = qwen3_build_graph(ctx, 8192, m->hp, m->w, m->kv, in, n_tokens, n_kv, selected, &out);
    const int rc = run_graph(m, g, seq, n_tokens, out, logits);
    delete g;
    ggml_backend_buffer_free(ibuf);
    ggml_free(ctx);
    return rc;
}

// KvCache::truncate_seq (keep > 0) / remove_seq (keep <= 0) on the model's cache
// (src/kv_cache.cpp:85-132), as the server's prefix reuse does (src/server.cpp:212-219): keep
// the common prefix, then step the rest of the new prompt.
void lstk_node_truncate(lstk_node_model *m, int32_t seq, int32_t keep) {
    if (m) m->kv.truncate_seq(seq, keep);
}

}  // extern "C"
