// ggml.h - the ggml names that the reference's attention-node sources use, declared for the
// ggml-compatible front end of this backend (localstack_b200/ggml_node).
//
// The reference builds its model graph with ggml (src/qwen3.cpp) and keeps its KV cache in ggml
// tensors (src/kv_cache.cpp). Compiling those two files unchanged against these declarations lets
// the reference's own graph builder record a graph that node.cpp executes on the GPU: the
// attention node's ops (rms_norm + mul of the QK-norm, rope_ext, set_rows, flash_attn_ext) go to
// this library's C ABI, the rest (projections, FFN, embeddings) to cuBLAS and small kernels.
// Only the names those files use are declared; the signatures follow the calls they make.
#pragma once

#include <cstddef>
#include <cstdint>

typedef uint16_t ggml_fp16_t;

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_I32 = 26,
    GGML_TYPE_I64 = 27,
    GGML_TYPE_BF16 = 30,
};

enum ggml_prec {
    GGML_PREC_DEFAULT = 0,
    GGML_PREC_F32 = 10,
};

#define GGML_ROPE_TYPE_NEOX 2
#define GGML_MAX_DIMS 4
#define GGML_MAX_SRC 10
#define GGML_MAX_NAME 64
#define GGML_MAX_OP_PARAMS 64

// Operations recorded by the graph builder (the executor's dispatch keys).
enum ggml_op {
    GGML_OP_NONE = 0,
    GGML_OP_GET_ROWS,
    GGML_OP_RMS_NORM,
    GGML_OP_MUL,
    GGML_OP_ADD,
    GGML_OP_DIV,
    GGML_OP_MUL_MAT,
    GGML_OP_MUL_MAT_ID,
    GGML_OP_RESHAPE,
    GGML_OP_VIEW,
    GGML_OP_PERMUTE,
    GGML_OP_CONT,
    GGML_OP_CPY,
    GGML_OP_ROPE,
    GGML_OP_SET_ROWS,
    GGML_OP_FLASH_ATTN_EXT,
    GGML_OP_SWIGLU,
    GGML_OP_SOFT_MAX,
    GGML_OP_ARGSORT_TOP_K,
    GGML_OP_SUM_ROWS,
    GGML_OP_CLAMP,
};

struct ggml_context;
struct ggml_cgraph;
struct ggml_backend_buffer;

struct ggml_tensor {
    ggml_type type;
    ggml_backend_buffer *buffer;
    int64_t ne[GGML_MAX_DIMS];  // elements per dimension, ne[0] innermost
    size_t nb[GGML_MAX_DIMS];   // bytes between consecutive elements of each dimension
    ggml_op op;
    int32_t op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)];
    int32_t flags;
    ggml_tensor *src[GGML_MAX_SRC];
    ggml_tensor *view_src;
    size_t view_offs;
    void *data;  // device memory once allocated (views: the source's data plus view_offs)
    char name[GGML_MAX_NAME];
};

struct ggml_init_params {
    size_t mem_size;
    void *mem_buffer;
    bool no_alloc;
};

// Context and tensors.
size_t ggml_tensor_overhead(void);
ggml_context *ggml_init(ggml_init_params params);
void ggml_free(ggml_context *ctx);
ggml_tensor *ggml_new_tensor_2d(ggml_context *ctx, ggml_type type, int64_t ne0, int64_t ne1);
ggml_tensor *ggml_format_name(ggml_tensor *tensor, const char *fmt, ...);
ggml_tensor *ggml_set_name(ggml_tensor *tensor, const char *name);
void ggml_set_input(ggml_tensor *tensor);
void ggml_set_output(ggml_tensor *tensor);
size_t ggml_row_size(ggml_type type, int64_t ne);
ggml_fp16_t ggml_fp32_to_fp16(float x);
float ggml_fp16_to_fp32(ggml_fp16_t h);

// Graph.
ggml_cgraph *ggml_new_graph_custom(ggml_context *ctx, size_t size, bool grads);
void ggml_build_forward_expand(ggml_cgraph *cgraph, ggml_tensor *tensor);

// Operations (each records one node).
ggml_tensor *ggml_get_rows(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b);
ggml_tensor *ggml_rms_norm(ggml_context *ctx, ggml_tensor *a, float eps);
ggml_tensor *ggml_mul(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b);
ggml_tensor *ggml_add(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b);
ggml_tensor *ggml_div(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b);
ggml_tensor *ggml_mul_mat(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b);
ggml_tensor *ggml_mul_mat_id(ggml_context *ctx, ggml_tensor *as, ggml_tensor *b, ggml_tensor *ids);
ggml_tensor *ggml_reshape_2d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1);
ggml_tensor *ggml_reshape_3d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2);
ggml_tensor *ggml_view_2d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, size_t nb1, size_t offset);
ggml_tensor *ggml_view_3d(ggml_context *ctx, ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2, size_t nb1,
                          size_t nb2, size_t offset);
ggml_tensor *ggml_permute(ggml_context *ctx, ggml_tensor *a, int axis0, int axis1, int axis2, int axis3);
ggml_tensor *ggml_cont(ggml_context *ctx, ggml_tensor *a);
ggml_tensor *ggml_cpy(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b);
ggml_tensor *ggml_rope_ext(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, ggml_tensor *c, int n_dims, int mode,
                           int n_ctx_orig, float freq_base, float freq_scale, float ext_factor, float attn_factor,
                           float beta_fast, float beta_slow);
ggml_tensor *ggml_set_rows(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b, ggml_tensor *c);
ggml_tensor *ggml_flash_attn_ext(ggml_context *ctx, ggml_tensor *q, ggml_tensor *k, ggml_tensor *v,
                                 ggml_tensor *mask, float scale, float max_bias, float logit_softcap);
void ggml_prec_set_acc(ggml_tensor *a, ggml_prec prec);
ggml_tensor *ggml_swiglu_split(ggml_context *ctx, ggml_tensor *a, ggml_tensor *b);
ggml_tensor *ggml_soft_max(ggml_context *ctx, ggml_tensor *a);
ggml_tensor *ggml_argsort_top_k(ggml_context *ctx, ggml_tensor *a, int k);
ggml_tensor *ggml_sum_rows(ggml_context *ctx, ggml_tensor *a);
ggml_tensor *ggml_clamp(ggml_context *ctx, ggml_tensor *a, float min, float max);
