// Minimal stand-in for the ggml-backend names used by the reference's src/kv_cache.cpp:11-52.
// Test infrastructure only (see ggml.h in this folder).
#pragma once

#include "ggml.h"

struct ggml_backend;
typedef ggml_backend *ggml_backend_t;
struct ggml_backend_buffer;
typedef ggml_backend_buffer *ggml_backend_buffer_t;

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(ggml_context *ctx, ggml_backend_t backend);
void ggml_backend_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value);
void ggml_backend_buffer_free(ggml_backend_buffer_t buffer);
size_t ggml_backend_buffer_get_size(ggml_backend_buffer_t buffer);
