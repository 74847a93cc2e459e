// Minimal stand-in for the few ggml declarations that the reference's src/kv_cache.h and
// src/kv_cache.cpp name (ggml itself lives in the reference's llama.cpp submodule, which is not
// present). Test infrastructure only: it lets the reference's own KvCache bookkeeping
// (alloc / remove_seq / truncate_seq / fill_mask, src/kv_cache.cpp:59-150) compile unchanged so
// the product's page-table logic can be checked against it. No tensor math lives here.
#pragma once

#include <cstddef>
#include <cstdint>

typedef uint16_t ggml_fp16_t;

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
};

struct ggml_context;

struct ggml_tensor {
    ggml_type type;
    int64_t ne[4];
    size_t nb[4];
    void *data;
    char name[64];
};

struct ggml_init_params {
    size_t mem_size;
    void *mem_buffer;
    bool no_alloc;
};

size_t ggml_tensor_overhead(void);
ggml_context *ggml_init(ggml_init_params params);
void ggml_free(ggml_context *ctx);
ggml_tensor *ggml_new_tensor_2d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1);
ggml_tensor *ggml_format_name(ggml_tensor *tensor, const char *fmt, ...);
ggml_fp16_t ggml_fp32_to_fp16(float x);
float ggml_fp16_to_fp32(ggml_fp16_t h);
