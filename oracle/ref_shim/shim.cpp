// Host-memory definitions for the ggml stand-in declared in ggml.h / ggml-backend.h.
// Test infrastructure only: tensors are plain host allocations so that the reference's
// KvCache::init (src/kv_cache.cpp:11-42) can run unchanged; no GPU and no ggml kernels.
#include "ggml.h"
#include "ggml-backend.h"

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

struct ggml_context {
    std::vector<ggml_tensor *> tensors;
};

struct ggml_backend_buffer {
    ggml_context *ctx;
    size_t size;
};

static size_t type_size(ggml_type t) { return t == GGML_TYPE_F16 ? 2 : 4; }

size_t ggml_tensor_overhead(void) { return sizeof(ggml_tensor) + 16; }

ggml_context *ggml_init(ggml_init_params) { return new ggml_context(); }

void ggml_free(ggml_context *ctx) {
    if (!ctx) return;
    for (ggml_tensor *t : ctx->tensors) {
        std::free(t->data);
        delete t;
    }
    delete ctx;
}

ggml_tensor *ggml_new_tensor_2d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1) {
    ggml_tensor *t = new ggml_tensor();
    t->type = type;
    t->ne[0] = ne0;
    t->ne[1] = ne1;
    t->ne[2] = t->ne[3] = 1;
    t->nb[0] = type_size(type);
    t->nb[1] = t->nb[0] * (size_t) ne0;
    t->nb[2] = t->nb[3] = t->nb[1] * (size_t) ne1;
    t->data = nullptr;
    t->name[0] = 0;
    ctx->tensors.push_back(t);
    return t;
}

ggml_tensor *ggml_format_name(ggml_tensor *tensor, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(tensor->name, sizeof(tensor->name), fmt, ap);
    va_end(ap);
    return tensor;
}

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(ggml_context *ctx, ggml_backend_t) {
    ggml_backend_buffer *buf = new ggml_backend_buffer{ctx, 0};
    for (ggml_tensor *t : ctx->tensors) {
        const size_t bytes = t->nb[1] * (size_t) t->ne[1];
        t->data = std::malloc(bytes ? bytes : 1);
        if (!t->data) {
            delete buf;
            return nullptr;
        }
        buf->size += bytes;
    }
    return buf;
}

void ggml_backend_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value) {
    for (ggml_tensor *t : buffer->ctx->tensors) std::memset(t->data, value, t->nb[1] * (size_t) t->ne[1]);
}

void ggml_backend_buffer_free(ggml_backend_buffer_t buffer) { delete buffer; }

size_t ggml_backend_buffer_get_size(ggml_backend_buffer_t buffer) { return buffer->size; }

// IEEE binary16 round-to-nearest-even, the rounding ggml's fp32->fp16 conversion performs.
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
