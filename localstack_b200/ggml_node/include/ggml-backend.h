// ggml-backend.h - the ggml-backend names that the reference's attention-node sources use (see
// ggml.h in this folder). The "backend" of this front end is the CUDA device current when a
// buffer is allocated: tensors of a context are placed in one device allocation.
#pragma once

#include "ggml.h"

struct ggml_backend;
typedef ggml_backend *ggml_backend_t;
struct ggml_backend_buffer;
typedef ggml_backend_buffer *ggml_backend_buffer_t;
struct ggml_backend_device;
typedef ggml_backend_device *ggml_backend_dev_t;

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(ggml_context *ctx, ggml_backend_t backend);
void ggml_backend_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value);
void ggml_backend_buffer_free(ggml_backend_buffer_t buffer);
size_t ggml_backend_buffer_get_size(ggml_backend_buffer_t buffer);
