// host_util.cpp - error strings and the RoPE (cos, sin) table. Plain host C++; compiled with
// -ffp-contract=off so the table values are what separately-rounded float code produces.
#include "host_util.h"

#include "lstk_cuda_attn.h"

#include <cmath>
#include <string>

namespace lstk {

static thread_local std::string g_last_error;

int set_error(int code, const std::string &msg) {
    g_last_error = msg;
    return code;
}

int clear_error() {
    g_last_error.clear();
    return LSTK_OK;
}

}  // namespace lstk

extern "C" {

const char *lstk_cuda_last_error(void) { return lstk::g_last_error.c_str(); }

size_t lstk_rope_table_bytes(int32_t n_pos, int32_t head_dim) {
    if (n_pos <= 0 || head_dim <= 0 || head_dim % 2) return 0;
    return (size_t) n_pos * (size_t) (head_dim / 2) * 2 * sizeof(float);
}

// The per-position rotation ggml's CPU rope builds for the NEOX call in attn_block
// (src/qwen3.cpp:143-146): theta starts at the position and is multiplied by
// powf(freq_base, -2/head_dim) once per dimension pair; entries are cosf/sinf of
// freq_scale * theta (ext_factor 0 and attn_factor 1 leave them unscaled).
int lstk_rope_table_fill(float *host_table, int32_t n_pos, int32_t head_dim, float freq_base, float freq_scale) {
    if (host_table == nullptr || n_pos <= 0 || head_dim <= 0 || head_dim % 2)
        return lstk::set_error(LSTK_ERR_INVALID_ARG, "lstk_rope_table_fill: bad arguments");
    const int half = head_dim / 2;
    const float theta_scale = powf(freq_base, -2.0f / (float) head_dim);
    for (int32_t p = 0; p < n_pos; p++) {
        float theta = (float) p;
        float *row = host_table + (size_t) p * half * 2;
        for (int i = 0; i < half; i++) {
            const float t = freq_scale * theta;
            row[2 * i + 0] = cosf(t);
            row[2 * i + 1] = sinf(t);
            theta *= theta_scale;
        }
    }
    return lstk::clear_error();
}

}  // extern "C"
