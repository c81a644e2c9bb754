// Minimal stand-ins for the ggml declarations that the reference's GDN host
// mirror (src/bridge/ggml_d3d12.cpp:77-158) uses, so that range compiles on its
// own.  Test infrastructure for oracle/_ref only.
#pragma once
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <vector>

enum ggml_type { GGML_TYPE_F32 = 0 };
enum ggml_op { GGML_OP_NONE = 0, GGML_OP_GATED_DELTA_NET = 1 };

struct ggml_tensor {
    ggml_type type;
    int64_t ne[4];
    size_t nb[4];
    ggml_op op;
    int32_t op_params[16];
    ggml_tensor* src[10];
    void* data;
};

// ggml_is_contiguous: dense row-major storage, dims of extent 1 ignored.
inline bool ggml_is_contiguous(const ggml_tensor* t) {
    size_t next = sizeof(float);
    for (int i = 0; i < 4; ++i) {
        if (t->ne[i] != 1 && t->nb[i] != next)
            return false;
        next *= (size_t)t->ne[i];
    }
    return true;
}
// ggml_is_contiguous_rows: elements of a row are adjacent.
inline bool ggml_is_contiguous_rows(const ggml_tensor* t) {
    return t->ne[0] == 1 || t->nb[0] == sizeof(float);
}
inline bool d3d12_gdn_enabled() { return true; }
static int s_gdn_min_tokens = 1;
