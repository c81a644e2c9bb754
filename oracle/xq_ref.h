/*
 * xq_ref -- CPU restatement of the reference's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity oracle and the timed
 * CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it.  The product path never
 * links, loads or falls back to it.
 *
 * What it restates (the reference's ggml-cpu sources live in the absent
 * llama.cpp submodule, beellama.cpp @ 982eaadaa9dbe761f00205bc20b6c04b7329b58d):
 *   - ggml block codecs Q8_0 / Q4_0 / F16 (ggml-quants.c reference quantizers,
 *     the same arithmetic gguf 0.19.0 gguf/quants.py pins bit for bit);
 *   - ggml-cpu GGML_OP_FLASH_ATTN_EXT: the per-row online softmax
 *     (patches/0008-flash-attn-query-consistency.patch:4-35 context lines),
 *     the single-query split-KV branch and its partial reduction
 *     (patches/0006-cpu-flash-attn-consistent-kv-reduction.patch:7-14), the
 *     GGML_FLASH_ATTN_NO_QUERY_TILING=4 policy (patches/README.md:58-73);
 *   - ggml-cpu GGML_OP_GATED_DELTA_NET with the fork's h mod H_k key-head map
 *     and K rollback snapshot slots (src/bridge/ggml_d3d12.cpp:113-158);
 *   - RKVA range attention partials and the LSE merge
 *     (shaders/rkva/rkva_range_attn.hlsl:59-106, rkva_range_reduce.hlsl:13-46,
 *     rkva_range_reduce_opt.hlsl:26-133) and the split policy
 *     (uwp/rkva/rkva-range-profile.h:82-147).
 * Arithmetic follows ggml-cpu's generic (non-SIMD) code paths: float products,
 * double accumulation in ggml_vec_dot_f32/f16, float accumulation in the
 * integer block dots.  The SIMD reduction order of the x86 build cannot be
 * restated without the absent source; tests compare within tolerance.
 */
#ifndef XQ_REF_H
#define XQ_REF_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type ids (stable across ggml versions). */
enum { XQR_F32 = 0, XQR_F16 = 1, XQR_Q4_0 = 2, XQR_Q8_0 = 8 };

typedef struct {
    int type;          /* XQR_* */
    const void *data;
    int64_t ne[4];     /* elements per dim */
    size_t nb[4];      /* byte strides */
} xqr_tensor;

/* ---- codecs ---- */
uint16_t xqr_fp32_to_fp16(float f);
float xqr_fp16_to_fp32(uint16_t h);
size_t xqr_row_size(int type, int64_t n);
/* ggml quantize_row_q8_0_ref / quantize_row_q4_0_ref (n multiple of 32). */
void xqr_quantize_q8_0(const float *x, void *y, int64_t n);
void xqr_quantize_q4_0(const float *x, void *y, int64_t n);
/* x86 AVX2 ggml-cpu quantize_row_q8_0 arithmetic (id = 127/amax, ties-to-even). */
void xqr_quantize_q8_0_x86(const float *x, void *y, int64_t n);
void xqr_quantize_f16(const float *x, void *y, int64_t n);
/* ggml to_float for F32/F16/Q8_0/Q4_0. */
void xqr_dequantize(int type, const void *x, float *y, int64_t n);

/* ---- FLASH_ATTN_EXT ---- */
enum {
    XQR_FA_NATIVE = 0,   /* ggml-cpu default dispatch (split-KV for 1 query) */
    XQR_FA_SCALAR = 1,   /* NO_QUERY_TILING=1: one_chunk per row, no tiling */
    XQR_FA_POLICY4 = 4,  /* NO_QUERY_TILING=4: F32 Q.K with expanded K      */
};

typedef struct {
    xqr_tensor q, k, v;
    xqr_tensor mask;      /* F16 [n_kv, n_q_pad, m2, m3]; data == NULL: none */
    const float *sinks;   /* [n_head] or NULL */
    float *dst;           /* F32 [DV, n_head, n_q, n_seq] contiguous */
    float scale, max_bias, softcap;
    int policy;           /* XQR_FA_* */
    int no_split_kv;      /* GGML_FLASH_ATTN_NO_SPLIT_KV=1 */
    int nth;              /* ggml n_threads: number of split-KV chunks */
    int n_workers;        /* real host threads used to compute (>=1) */
} xqr_fa_args;

int xqr_flash_attn_ext(const xqr_fa_args *a);

/* float64 softmax attention over the same ggml tensors (exact dequant), for
 * independent cross-checks.  Same dst layout; lse (may be NULL) gets
 * [n_seq][n_q][n_head] natural-log LSE. */
int xqr_flash_attn_f64(const xqr_fa_args *a, float *lse);

/* ---- RKVA range attention (O, LSE) ---- */
typedef struct {
    int storage;          /* XQR_F16 / XQR_Q8_0 / XQR_Q4_0 */
    const void *k, *v;    /* [capacity][n_head_kv][D] in storage format */
    const float *q;       /* [n_tokens][n_head][D] */
    const int32_t *positions; /* [n_tokens] absolute */
    uint32_t n_tokens, active, origin, n_head, n_head_kv, head_dim, split_k;
    float kq_scale;
    float *out;           /* [n_tokens][n_head][D] then */
    float *lse;           /* [n_tokens][n_head] */
} xqr_range_args;

/* rkva_range_attn.hlsl partials + rkva_range_reduce.hlsl merge, float32. */
int xqr_range_attn(const xqr_range_args *a);
/* partial records [split][n_rows][D+2] = (acc[D], max, denom) -> O, LSE with
 * rkva_range_reduce_opt.hlsl semantics (empty => O=0/LSE=-inf, NaN poison). */
void xqr_lse_merge(const float *partials, uint32_t n_splits, uint32_t n_rows, uint32_t D,
                   float *out, float *lse);
/* rkva-range-profile.h policies. mode 0 = reference (live259), 1/2/3 = opt. */
uint32_t xqr_split_k(uint32_t active, uint32_t mode);

/* ---- GATED_DELTA_NET ---- */
typedef struct {
    xqr_tensor q, k, v, g, beta, state;  /* all F32 */
    float *dst;     /* [S_v*H, n_seq*T + K*S_v*n_seq] contiguous */
    int slots;      /* op_params[0]: K >= 1 */
    int n_workers;
    int lanes8;     /* 1: eight-lane tree reductions of the D3D12 host mirror */
    /* v, g, beta, state, dst hold value heads [head_begin, head_begin + H) of
     * an op with n_head_total value heads (0: the whole op); head j of the
     * block reads key head (head_begin + j) % H_k, the fork's h mod H_k. */
    int64_t head_begin, n_head_total;
} xqr_gdn_args;

int xqr_gated_delta_net(const xqr_gdn_args *a);

/* std::mt19937(seed) through std::uniform_real_distribution<float>(lo, hi). */
void xqr_std_uniform(uint32_t seed, float lo, float hi, int64_t n, float *out);

#ifdef __cplusplus
}
#endif
#endif
