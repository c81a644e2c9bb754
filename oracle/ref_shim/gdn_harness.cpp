// Drives the reference's d3d12_gdn_emulate with the inputs of its GDN selftest
// (src/bridge/ggml_d3d12.cpp:174-308: mt19937(1701 + j), uniform(-0.05, 0.05),
// g = -0.3 - |u|, beta = u + 0.5, optional Q/K/V head padding pad/pad+2/pad+4).
// Test infrastructure for oracle/_ref only.
#include <random>
#include "ggml_shim.h"

bool d3d12_gdn_supported(const ggml_tensor* op);
void d3d12_gdn_emulate(const ggml_tensor* op, float* out);

namespace {
struct Case {
    ggml_tensor src[6];
    ggml_tensor op;
    std::vector<float> in[6];
};

void make_case(Case& c, int tokens, int slots, int pad) {
    const int64_t shapes[6][4] = {{128, 16, tokens, 1}, {128, 16, tokens, 1},
                                  {128, 32, tokens, 1}, {1, 32, tokens, 1},
                                  {1, 32, tokens, 1},   {128, 128, 32, 1}};
    for (int j = 0; j < 6; ++j) {
        ggml_tensor& t = c.src[j];
        std::memset(&t, 0, sizeof(t));
        t.type = GGML_TYPE_F32;
        for (int d = 0; d < 4; ++d)
            t.ne[d] = shapes[j][d];
        t.nb[0] = 4;
        t.nb[1] = t.nb[0] * t.ne[0];
        t.nb[2] = t.nb[1] * t.ne[1];
        t.nb[3] = t.nb[2] * t.ne[2];
        if (pad && j < 3) {
            t.nb[1] = (128 + pad + 2 * j) * sizeof(float);
            t.nb[2] = t.nb[1] * t.ne[1];
            t.nb[3] = t.nb[2] * tokens;
        }
        const size_t bytes = t.nb[3] * t.ne[3];
        c.in[j].assign(bytes / 4, 1e30f);
        std::mt19937 rng(1701u + j);
        std::uniform_real_distribution<float> uni(-0.05f, 0.05f);
        for (int64_t a = 0; a < t.ne[2]; ++a)
            for (int64_t h = 0; h < t.ne[1]; ++h)
                for (int64_t i = 0; i < t.ne[0]; ++i) {
                    float v = uni(rng);
                    if (j == 3)
                        v = -0.3f - std::fabs(v);
                    if (j == 4)
                        v += 0.5f;
                    c.in[j][(a * t.nb[2] + h * t.nb[1]) / 4 + i] = v;
                }
        t.data = c.in[j].data();
    }
    std::memset(&c.op, 0, sizeof(c.op));
    c.op.type = GGML_TYPE_F32;
    c.op.op = GGML_OP_GATED_DELTA_NET;
    c.op.op_params[0] = slots;
    c.op.ne[0] = 4096;
    c.op.ne[1] = tokens + slots * 128;
    c.op.ne[2] = c.op.ne[3] = 1;
    c.op.nb[0] = 4;
    c.op.nb[1] = 4 * 4096;
    c.op.nb[2] = c.op.nb[3] = c.op.nb[1] * c.op.ne[1];
    for (int j = 0; j < 6; ++j)
        c.op.src[j] = &c.src[j];
}
} // namespace

extern "C" {
// Sizes in floats of input j (0..5 = q, k, v, g, beta, state) incl. padding.
long xq_gdn_ref_input_floats(int tokens, int pad, int j) {
    Case c;
    make_case(c, tokens, 1, pad);
    return (long)c.in[j].size();
}
// Copies the selftest inputs out and runs the reference mirror.
// out: 4096*T + 524288*K floats, pre-filled by the caller (sentinels survive
// where the mirror writes nothing).  Returns 0, or -1 if the contract refuses.
int xq_gdn_ref_run(int tokens, int slots, int pad, float* q, float* k, float* v, float* g,
                   float* beta, float* state, float* out) {
    Case c;
    make_case(c, tokens, slots, pad);
    float* dst[6] = {q, k, v, g, beta, state};
    for (int j = 0; j < 6; ++j)
        if (dst[j])
            std::memcpy(dst[j], c.in[j].data(), c.in[j].size() * 4);
    if (!d3d12_gdn_supported(&c.op))
        return -1;
    d3d12_gdn_emulate(&c.op, out);
    return 0;
}
// First n outputs of std::mt19937(seed) fed through
// std::uniform_real_distribution<float>(lo, hi), to pin a restated generator.
void xq_std_uniform(unsigned seed, float lo, float hi, int n, float* out) {
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> uni(lo, hi);
    for (int i = 0; i < n; ++i)
        out[i] = uni(rng);
}
}
