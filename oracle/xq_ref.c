/*
 * xq_ref.c -- CPU restatement of the reference's FLASH_ATTN_EXT / GATED_DELTA_NET
 * arithmetic.  TEST INFRASTRUCTURE ONLY (parity oracle + timed CPU baseline);
 * never loaded by the product path.  Header xq_ref.h lists the sources restated.
 *
 * Build: oracle/Makefile (gcc -O3 -ffp-contract=off -pthread).  Contraction is
 * off so every a*b+c below rounds twice, as ggml's generic C loops do.
 */
#include "xq_ref.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32, round-to-nearest-even (GGML_FP32_TO_FP16 / F16C mode 0).   */

uint16_t xqr_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf / nan (quiet) */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) /* >= 65520 rounds to inf */
        return (uint16_t)(sign | 0x7c00u);
    if (ax >= 0x38800000u) { /* normal half */
        const uint32_t mant = ax & 0x7fffffu;
        uint32_t h = (((ax >> 23) - 112u) << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u)))
            h++;
        return (uint16_t)(sign | h);
    }
    if (ax < 0x33000000u) /* below 2^-25: zero (2^-25 itself ties to even 0) */
        return (uint16_t)sign;
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const int shift = 126 - (int)e; /* 14..24 */
    uint32_t h = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1u)))
        h++;
    return (uint16_t)(sign | h);
}

float xqr_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {
            float f = (float)m * 5.9604644775390625e-08f; /* m * 2^-24, exact */
            memcpy(&x, &f, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline float h2f(const void *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return xqr_fp16_to_fp32(h);
}

size_t xqr_row_size(int type, int64_t n) {
    switch (type) {
    case XQR_F32: return (size_t)n * 4;
    case XQR_F16: return (size_t)n * 2;
    case XQR_Q8_0: return (size_t)(n / 32) * 34;
    case XQR_Q4_0: return (size_t)(n / 32) * 18;
    default: return 0;
    }
}

/* ------------------------------------------------------------------------ */
/* Block codecs (ggml-quants.c *_ref arithmetic; gguf/quants.py pins these). */

void xqr_quantize_q8_0(const float *x, void *vy, int64_t n) {
    uint8_t *y = (uint8_t *)vy;
    for (int64_t b = 0; b < n / 32; ++b) {
        const float *xb = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j)
            amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = xqr_fp32_to_fp16(d);
        memcpy(y + b * 34, &dh, 2);
        for (int j = 0; j < 32; ++j)
            y[b * 34 + 2 + j] = (uint8_t)(int8_t)roundf(xb[j] * id);
    }
}

void xqr_quantize_q8_0_x86(const float *x, void *vy, int64_t n) {
    uint8_t *y = (uint8_t *)vy;
    for (int64_t b = 0; b < n / 32; ++b) {
        const float *xb = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j)
            amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127.0f;
        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
        const uint16_t dh = xqr_fp32_to_fp16(d);
        memcpy(y + b * 34, &dh, 2);
        for (int j = 0; j < 32; ++j)
            y[b * 34 + 2 + j] = (uint8_t)(int8_t)rintf(xb[j] * id); /* ties to even */
    }
}

void xqr_quantize_q4_0(const float *x, void *vy, int64_t n) {
    uint8_t *y = (uint8_t *)vy;
    for (int64_t b = 0; b < n / 32; ++b) {
        const float *xb = x + b * 32;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            if (amax < fabsf(xb[j])) {
                amax = fabsf(xb[j]);
                vmax = xb[j];
            }
        }
        const float d = vmax / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = xqr_fp32_to_fp16(d);
        memcpy(y + b * 18, &dh, 2);
        for (int j = 0; j < 16; ++j) {
            int8_t a = (int8_t)(xb[j] * id + 8.5f);
            int8_t c = (int8_t)(xb[16 + j] * id + 8.5f);
            const uint8_t lo = (uint8_t)(a < 15 ? a : 15);
            const uint8_t hi = (uint8_t)(c < 15 ? c : 15);
            y[b * 18 + 2 + j] = (uint8_t)(lo | (hi << 4));
        }
    }
}

void xqr_quantize_f16(const float *x, void *vy, int64_t n) {
    uint16_t *y = (uint16_t *)vy;
    for (int64_t i = 0; i < n; ++i)
        y[i] = xqr_fp32_to_fp16(x[i]);
}

void xqr_dequantize(int type, const void *vx, float *y, int64_t n) {
    const uint8_t *x = (const uint8_t *)vx;
    switch (type) {
    case XQR_F32:
        memcpy(y, x, (size_t)n * 4);
        break;
    case XQR_F16:
        for (int64_t i = 0; i < n; ++i)
            y[i] = h2f(x + 2 * i);
        break;
    case XQR_Q8_0:
        for (int64_t b = 0; b < n / 32; ++b) {
            const float d = h2f(x + 34 * b);
            for (int j = 0; j < 32; ++j)
                y[b * 32 + j] = (float)(int8_t)x[34 * b + 2 + j] * d;
        }
        break;
    case XQR_Q4_0:
        for (int64_t b = 0; b < n / 32; ++b) {
            const float d = h2f(x + 18 * b);
            for (int j = 0; j < 16; ++j) {
                const uint8_t q = x[18 * b + 2 + j];
                y[b * 32 + j] = (float)((q & 0x0f) - 8) * d;
                y[b * 32 + j + 16] = (float)((q >> 4) - 8) * d;
            }
        }
        break;
    default:
        break;
    }
}

/* ------------------------------------------------------------------------ */
/* ggml-cpu generic vector kernels.                                          */

static float vec_dot_f32(int64_t n, const float *x, const float *y) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i)
        s += (double)(x[i] * y[i]);
    return (float)s;
}

static float vec_dot_f16(int64_t n, const uint8_t *x, const uint8_t *y) {
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i)
        s += (double)(h2f(x + 2 * i) * h2f(y + 2 * i));
    return (float)s;
}

static float vec_dot_q8_0_q8_0(int64_t n, const uint8_t *x, const uint8_t *y) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < n / 32; ++b) {
        int sumi = 0;
        for (int j = 0; j < 32; ++j)
            sumi += (int)(int8_t)x[34 * b + 2 + j] * (int)(int8_t)y[34 * b + 2 + j];
        const float dd = h2f(x + 34 * b) * h2f(y + 34 * b);
        sumf += (float)sumi * dd;
    }
    return sumf;
}

static float vec_dot_q4_0_q8_0(int64_t n, const uint8_t *x, const uint8_t *y) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < n / 32; ++b) {
        int s0 = 0, s1 = 0;
        for (int j = 0; j < 16; ++j) {
            const uint8_t q = x[18 * b + 2 + j];
            s0 += ((q & 0x0f) - 8) * (int)(int8_t)y[34 * b + 2 + j];
            s1 += ((q >> 4) - 8) * (int)(int8_t)y[34 * b + 2 + 16 + j];
        }
        sumf += (float)(s0 + s1) * h2f(x + 18 * b) * h2f(y + 34 * b);
    }
    return sumf;
}

static void vec_mad_f16(int64_t n, uint16_t *y, const uint8_t *x, float v) {
    for (int64_t i = 0; i < n; ++i)
        y[i] = xqr_fp32_to_fp16(xqr_fp16_to_fp32(y[i]) + h2f(x + 2 * i) * v);
}

static void vec_scale_f16(int64_t n, uint16_t *y, float v) {
    for (int64_t i = 0; i < n; ++i)
        y[i] = xqr_fp32_to_fp16(xqr_fp16_to_fp32(y[i]) * v);
}

static void vec_mad_f32(int64_t n, float *y, const float *x, float v) {
    for (int64_t i = 0; i < n; ++i)
        y[i] += x[i] * v;
}

static void vec_scale_f32(int64_t n, float *y, float v) {
    for (int64_t i = 0; i < n; ++i)
        y[i] *= v;
}

/* ------------------------------------------------------------------------ */
/* Worker pool: run fn(ctx, i) for i in [0, n) over n_workers threads.       */

typedef void (*xqr_job_fn)(void *ctx, int64_t i, int worker);

typedef struct {
    xqr_job_fn fn;
    void *ctx;
    int64_t n;
    int n_workers, worker;
} xqr_job;

static void *xqr_job_main(void *p) {
    xqr_job *j = (xqr_job *)p;
    for (int64_t i = j->worker; i < j->n; i += j->n_workers)
        j->fn(j->ctx, i, j->worker);
    return NULL;
}

static void xqr_parallel(xqr_job_fn fn, void *ctx, int64_t n, int n_workers) {
    if (n_workers < 1)
        n_workers = 1;
    if (n_workers > 256)
        n_workers = 256;
    if ((int64_t)n_workers > n)
        n_workers = (int)(n > 0 ? n : 1);
    xqr_job jobs[256];
    pthread_t th[256];
    for (int w = 0; w < n_workers; ++w) {
        jobs[w].fn = fn;
        jobs[w].ctx = ctx;
        jobs[w].n = n;
        jobs[w].n_workers = n_workers;
        jobs[w].worker = w;
    }
    for (int w = 1; w < n_workers; ++w)
        pthread_create(&th[w], NULL, xqr_job_main, &jobs[w]);
    xqr_job_main(&jobs[0]);
    for (int w = 1; w < n_workers; ++w)
        pthread_join(th[w], NULL);
}

/* ------------------------------------------------------------------------ */
/* FLASH_ATTN_EXT.                                                           */

typedef struct {
    const xqr_fa_args *a;
    int64_t DK, DV, n_q, n_head, n_seq, n_kv, n_head_kv;
    int64_t rk2, rk3, rv2, rv3;
    float scale, softcap, m0, m1;
    uint32_t n_head_log2;
    int q_dot_type;   /* type Q is converted to before the K dot */
    int use_f32_qk;   /* policy 4 with F16 K/V */
    int64_t n_chunks, chunk_size; /* split-KV */
    float *partials;  /* split-KV: [n_head][n_chunks][2+DV] */
    size_t scratch_floats;
    float *scratch;   /* per worker */
} fa_ctx;

static float fa_slope(const fa_ctx *c, uint32_t h) {
    if (!(c->a->max_bias > 0.0f))
        return 1.0f;
    return h < c->n_head_log2 ? powf(c->m0, (float)(h + 1))
                              : powf(c->m1, (float)(2 * (h - c->n_head_log2) + 1));
}

/* ggml_compute_forward_flash_attn_ext_f16_one_chunk for one query row over
 * KV rows [ic0, ic1).  partial != NULL: write (M, S, VKQ[DV]) unnormalised. */
static void fa_row(const fa_ctx *c, int64_t iq1, int64_t iq2, int64_t iq3, int64_t ic0,
                   int64_t ic1, float *partial, float *scratch) {
    const xqr_fa_args *a = c->a;
    const int64_t DK = c->DK, DV = c->DV;
    float *VKQ32 = scratch;
    float *V32 = VKQ32 + DV;
    uint16_t *VKQ16 = (uint16_t *)(V32 + DV);
    float *Kf = (float *)(VKQ16 + DV + (DV & 1));
    uint8_t *Qq = (uint8_t *)(Kf + DK);

    const int v_f16 = a->v.type == XQR_F16;
    if (v_f16)
        memset(VKQ16, 0, (size_t)DV * 2);
    else
        memset(VKQ32, 0, (size_t)DV * 4);

    const uint8_t *mp = NULL;
    if (a->mask.data) {
        mp = (const uint8_t *)a->mask.data + iq1 * a->mask.nb[1] +
             (iq2 % a->mask.ne[2]) * a->mask.nb[2] + (iq3 % a->mask.ne[3]) * a->mask.nb[3];
    }
    const float slope = fa_slope(c, (uint32_t)iq2);
    const int64_t ik3 = iq3 / c->rk3, ik2 = iq2 / c->rk2;
    const int64_t iv3 = iq3 / c->rv3, iv2 = iq2 / c->rv2;
    const float *pq = (const float *)((const uint8_t *)a->q.data + iq1 * a->q.nb[1] +
                                      iq2 * a->q.nb[2] + iq3 * a->q.nb[3]);
    if (!c->use_f32_qk) {
        switch (c->q_dot_type) {
        case XQR_F16: xqr_quantize_f16(pq, Qq, DK); break;
        case XQR_Q8_0: xqr_quantize_q8_0(pq, Qq, DK); break;
        default: memcpy(Qq, pq, (size_t)DK * 4); break;
        }
    }

    float S = 0.0f, M = -INFINITY;
    for (int64_t ic = ic0; ic < ic1; ++ic) {
        const float mv = mp ? slope * h2f(mp + 2 * ic) : 0.0f;
        if (mv == -INFINITY)
            continue;
        const uint8_t *kd = (const uint8_t *)a->k.data + ic * a->k.nb[1] + ik2 * a->k.nb[2] +
                            ik3 * a->k.nb[3];
        float s;
        if (c->use_f32_qk) {
            for (int64_t i = 0; i < DK; ++i)
                Kf[i] = h2f(kd + 2 * i);
            s = vec_dot_f32(DK, pq, Kf);
        } else {
            switch (a->k.type) {
            case XQR_F16: s = vec_dot_f16(DK, kd, Qq); break;
            case XQR_Q8_0: s = vec_dot_q8_0_q8_0(DK, kd, Qq); break;
            case XQR_Q4_0: s = vec_dot_q4_0_q8_0(DK, kd, Qq); break;
            default: s = vec_dot_f32(DK, (const float *)kd, (const float *)Qq); break;
            }
        }
        s = s * c->scale;
        if (c->softcap != 0.0f)
            s = c->softcap * tanhf(s);
        s += mv;

        const float Mold = M;
        float ms = 1.0f, vs = 1.0f;
        const uint8_t *vd = (const uint8_t *)a->v.data + ic * a->v.nb[1] + iv2 * a->v.nb[2] +
                            iv3 * a->v.nb[3];
        if (v_f16) {
            if (s > M) {
                M = s;
                ms = expf(Mold - M);
                vec_scale_f16(DV, VKQ16, ms);
            } else {
                vs = expf(s - M);
            }
            vec_mad_f16(DV, VKQ16, vd, vs);
        } else {
            if (s > M) {
                M = s;
                ms = expf(Mold - M);
                vec_scale_f32(DV, VKQ32, ms);
            } else {
                vs = expf(s - M);
            }
            xqr_dequantize(a->v.type, vd, V32, DV);
            vec_mad_f32(DV, VKQ32, V32, vs);
        }
        S = S * ms + vs;
    }
    if (v_f16)
        for (int64_t d = 0; d < DV; ++d)
            VKQ32[d] = xqr_fp16_to_fp32(VKQ16[d]);

    if (partial) {
        partial[0] = M;
        partial[1] = S;
        memcpy(partial + 2, VKQ32, (size_t)DV * 4);
        return;
    }
    if (a->sinks) {
        const float s = a->sinks[iq2];
        float ms = 1.0f, vs = 1.0f;
        if (s > M) {
            ms = expf(M - s);
            vec_scale_f32(DV, VKQ32, ms);
        } else {
            vs = expf(s - M);
        }
        S = S * ms + vs;
    }
    const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
    vec_scale_f32(DV, VKQ32, S_inv);
    float *dst = a->dst + ((iq3 * c->n_q + iq1) * c->n_head + iq2) * DV;
    memcpy(dst, VKQ32, (size_t)DV * 4);
}

static void fa_job_rows(void *p, int64_t ir, int w) {
    const fa_ctx *c = (const fa_ctx *)p;
    const int64_t iq3 = ir / (c->n_head * c->n_q);
    const int64_t iq2 = (ir - iq3 * c->n_head * c->n_q) / c->n_q;
    const int64_t iq1 = ir - iq3 * c->n_head * c->n_q - iq2 * c->n_q;
    fa_row(c, iq1, iq2, iq3, 0, c->n_kv, NULL, c->scratch + (size_t)w * c->scratch_floats);
}

/* Split-KV pass 1: chunk index = job index (ggml thread ith). */
static void fa_job_chunks(void *p, int64_t ith, int w) {
    const fa_ctx *c = (const fa_ctx *)p;
    const int64_t ic0 = ith * c->chunk_size;
    const int64_t ic1 = ic0 + c->chunk_size < c->n_kv ? ic0 + c->chunk_size : c->n_kv;
    for (int64_t h = 0; h < c->n_head; ++h) {
        float *part = c->partials + (h * c->n_chunks + ith) * (2 + c->DV);
        if (ic0 < c->n_kv) {
            fa_row(c, 0, h, 0, ic0, ic1, part, c->scratch + (size_t)w * c->scratch_floats);
        } else {
            part[0] = -INFINITY;
            part[1] = 0.0f;
        }
    }
}

/* ggml_flash_attn_ext_reduce_partials: sequential online merge in chunk order. */
static void fa_reduce_partials(const fa_ctx *c) {
    const int64_t DV = c->DV;
    float *acc = (float *)malloc((size_t)DV * 4);
    for (int64_t h = 0; h < c->n_head; ++h) {
        float Mf = -INFINITY, Sf = 0.0f;
        memset(acc, 0, (size_t)DV * 4);
        for (int64_t ch = 0; ch < c->n_chunks; ++ch) {
            if (ch * c->chunk_size >= c->n_kv)
                continue;
            const float *part = c->partials + (h * c->n_chunks + ch) * (2 + DV);
            const float Mc = part[0], Sc = part[1];
            if (Sc == 0.0f)
                continue;
            const float Mn = fmaxf(Mf, Mc);
            const float so = expf(Mf - Mn), sn = expf(Mc - Mn);
            for (int64_t d = 0; d < DV; ++d)
                acc[d] = acc[d] * so + part[2 + d] * sn;
            Sf = Sf * so + Sc * sn;
            Mf = Mn;
        }
        if (Sf != 0.0f)
            vec_scale_f32(DV, acc, 1.0f / Sf);
        memcpy(c->a->dst + h * DV, acc, (size_t)DV * 4);
    }
    free(acc);
}

/* Tiled multi-query path (ggml-cpu ..._tiled, selected for F32 Q with F16/F32
 * K == V type).  Its source is absent; restated as F32 Q against K/V expanded
 * to F32, online softmax over KV tiles of 64 with an F32 value accumulator. */
static void fa_row_tiled(const fa_ctx *c, int64_t iq1, int64_t iq2, int64_t iq3,
                         float *scratch) {
    const xqr_fa_args *a = c->a;
    const int64_t DK = c->DK, DV = c->DV, T = 64;
    float *acc = scratch;
    float *kf = acc + DV;
    float *vf = kf + DK;
    float sc[64];
    memset(acc, 0, (size_t)DV * 4);
    const uint8_t *mp = NULL;
    if (a->mask.data)
        mp = (const uint8_t *)a->mask.data + iq1 * a->mask.nb[1] +
             (iq2 % a->mask.ne[2]) * a->mask.nb[2] + (iq3 % a->mask.ne[3]) * a->mask.nb[3];
    const float slope = fa_slope(c, (uint32_t)iq2);
    const int64_t ik3 = iq3 / c->rk3, ik2 = iq2 / c->rk2;
    const int64_t iv3 = iq3 / c->rv3, iv2 = iq2 / c->rv2;
    const float *pq = (const float *)((const uint8_t *)a->q.data + iq1 * a->q.nb[1] +
                                      iq2 * a->q.nb[2] + iq3 * a->q.nb[3]);
    float M = -INFINITY, S = 0.0f;
    for (int64_t t0 = 0; t0 < c->n_kv; t0 += T) {
        const int64_t t1 = t0 + T < c->n_kv ? t0 + T : c->n_kv;
        float tmax = -INFINITY;
        for (int64_t ic = t0; ic < t1; ++ic) {
            const float mv = mp ? slope * h2f(mp + 2 * ic) : 0.0f;
            if (mv == -INFINITY) {
                sc[ic - t0] = -INFINITY;
                continue;
            }
            const uint8_t *kd = (const uint8_t *)a->k.data + ic * a->k.nb[1] +
                                ik2 * a->k.nb[2] + ik3 * a->k.nb[3];
            xqr_dequantize(a->k.type, kd, kf, DK);
            float s = 0.0f;
            for (int64_t i = 0; i < DK; ++i)
                s += pq[i] * kf[i];
            s *= c->scale;
            if (c->softcap != 0.0f)
                s = c->softcap * tanhf(s);
            s += mv;
            sc[ic - t0] = s;
            tmax = fmaxf(tmax, s);
        }
        if (tmax == -INFINITY)
            continue;
        const float Mn = fmaxf(M, tmax);
        const float ms = expf(M - Mn);
        vec_scale_f32(DV, acc, ms);
        S *= ms;
        for (int64_t ic = t0; ic < t1; ++ic) {
            if (sc[ic - t0] == -INFINITY)
                continue;
            const float p = expf(sc[ic - t0] - Mn);
            const uint8_t *vd = (const uint8_t *)a->v.data + ic * a->v.nb[1] +
                                iv2 * a->v.nb[2] + iv3 * a->v.nb[3];
            xqr_dequantize(a->v.type, vd, vf, DV);
            vec_mad_f32(DV, acc, vf, p);
            S += p;
        }
        M = Mn;
    }
    const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
    vec_scale_f32(DV, acc, S_inv);
    memcpy(a->dst + ((iq3 * c->n_q + iq1) * c->n_head + iq2) * DV, acc, (size_t)DV * 4);
}

static void fa_job_tiled(void *p, int64_t ir, int w) {
    const fa_ctx *c = (const fa_ctx *)p;
    const int64_t iq3 = ir / (c->n_head * c->n_q);
    const int64_t iq2 = (ir - iq3 * c->n_head * c->n_q) / c->n_q;
    const int64_t iq1 = ir - iq3 * c->n_head * c->n_q - iq2 * c->n_q;
    fa_row_tiled(c, iq1, iq2, iq3, c->scratch + (size_t)w * c->scratch_floats);
}

static int fa_setup(const xqr_fa_args *a, fa_ctx *c) {
    memset(c, 0, sizeof(*c));
    c->a = a;
    c->DK = a->q.ne[0];
    c->DV = a->v.ne[0];
    c->n_q = a->q.ne[1];
    c->n_head = a->q.ne[2];
    c->n_seq = a->q.ne[3];
    c->n_kv = a->k.ne[1];
    c->n_head_kv = a->k.ne[2];
    if (a->q.type != XQR_F32 || a->k.ne[0] != c->DK || a->v.ne[1] != c->n_kv || c->DK % 32 ||
        c->n_head % a->k.ne[2] || c->n_head % a->v.ne[2] || c->n_seq % a->k.ne[3] ||
        c->n_seq % a->v.ne[3])
        return -1;
    c->rk2 = c->n_head / a->k.ne[2];
    c->rk3 = c->n_seq / a->k.ne[3];
    c->rv2 = c->n_head / a->v.ne[2];
    c->rv3 = c->n_seq / a->v.ne[3];
    c->scale = a->scale;
    c->softcap = a->softcap;
    if (c->softcap != 0.0f)
        c->scale /= c->softcap;
    c->n_head_log2 = 1u << (uint32_t)floor(log2((double)c->n_head));
    c->m0 = powf(2.0f, -(a->max_bias) / (float)c->n_head_log2);
    c->m1 = powf(2.0f, -(a->max_bias / 2.0f) / (float)c->n_head_log2);
    switch (a->k.type) {
    case XQR_F16: c->q_dot_type = XQR_F16; break;
    case XQR_Q8_0:
    case XQR_Q4_0: c->q_dot_type = XQR_Q8_0; break;
    case XQR_F32: c->q_dot_type = XQR_F32; break;
    default: return -1;
    }
    c->use_f32_qk = a->policy == XQR_FA_POLICY4 && a->k.type == XQR_F16 && a->v.type == XQR_F16;
    return 0;
}

int xqr_flash_attn_ext(const xqr_fa_args *a) {
    fa_ctx c;
    if (fa_setup(a, &c))
        return -1;
    const int workers = a->n_workers > 0 ? a->n_workers : 1;
    c.scratch_floats = (size_t)(4 * c.DK + 4 * c.DV + 64);
    c.scratch = (float *)malloc(c.scratch_floats * 4 * (size_t)workers);
    if (!c.scratch)
        return -2;
    const int kv_f = a->k.type == XQR_F16 || a->k.type == XQR_F32;
    const int split = !a->no_split_kv && c.n_q == 1 && c.n_seq == 1 && kv_f &&
                      a->k.type == a->v.type && c.n_kv >= 512;
    const int tiled = a->policy == XQR_FA_NATIVE && !split && kv_f && a->k.type == a->v.type &&
                      c.n_q >= 32;
    if (split) {
        const int nth = a->nth > 0 ? a->nth : 1;
        c.n_chunks = nth;
        c.chunk_size = (c.n_kv + nth - 1) / nth;
        c.partials = (float *)malloc((size_t)c.n_head * nth * (2 + c.DV) * 4);
        if (!c.partials) {
            free(c.scratch);
            return -2;
        }
        xqr_parallel(fa_job_chunks, &c, nth, workers);
        fa_reduce_partials(&c);
        free(c.partials);
    } else if (tiled) {
        xqr_parallel(fa_job_tiled, &c, c.n_q * c.n_head * c.n_seq, workers);
    } else {
        xqr_parallel(fa_job_rows, &c, c.n_q * c.n_head * c.n_seq, workers);
    }
    free(c.scratch);
    return 0;
}

/* float64 exact-dequant softmax attention (independent check). */
typedef struct {
    fa_ctx c;
    float *lse;
} fa64_ctx;

static void fa64_job(void *p, int64_t ir, int w) {
    (void)w;
    const fa64_ctx *x = (const fa64_ctx *)p;
    const fa_ctx *c = &x->c;
    const xqr_fa_args *a = c->a;
    const int64_t iq3 = ir / (c->n_head * c->n_q);
    const int64_t iq2 = (ir - iq3 * c->n_head * c->n_q) / c->n_q;
    const int64_t iq1 = ir - iq3 * c->n_head * c->n_q - iq2 * c->n_q;
    const int64_t DK = c->DK, DV = c->DV;
    float *kf = (float *)malloc((size_t)(DK + DV) * 4);
    float *vf = kf + DK;
    double *acc = (double *)calloc((size_t)DV, 8);
    double *sc = (double *)malloc((size_t)c->n_kv * 8);
    const uint8_t *mp = NULL;
    if (a->mask.data)
        mp = (const uint8_t *)a->mask.data + iq1 * a->mask.nb[1] +
             (iq2 % a->mask.ne[2]) * a->mask.nb[2] + (iq3 % a->mask.ne[3]) * a->mask.nb[3];
    const float slope = fa_slope(c, (uint32_t)iq2);
    const int64_t ik3 = iq3 / c->rk3, ik2 = iq2 / c->rk2;
    const int64_t iv3 = iq3 / c->rv3, iv2 = iq2 / c->rv2;
    const float *pq = (const float *)((const uint8_t *)a->q.data + iq1 * a->q.nb[1] +
                                      iq2 * a->q.nb[2] + iq3 * a->q.nb[3]);
    double M = -INFINITY;
    for (int64_t ic = 0; ic < c->n_kv; ++ic) {
        const double mv = mp ? (double)slope * h2f(mp + 2 * ic) : 0.0;
        if (mv == -INFINITY) {
            sc[ic] = -INFINITY;
            continue;
        }
        xqr_dequantize(a->k.type,
                       (const uint8_t *)a->k.data + ic * a->k.nb[1] + ik2 * a->k.nb[2] +
                           ik3 * a->k.nb[3],
                       kf, DK);
        double s = 0.0;
        for (int64_t i = 0; i < DK; ++i)
            s += (double)pq[i] * kf[i];
        s *= (double)c->scale;
        if (c->softcap != 0.0f)
            s = (double)c->softcap * tanh(s);
        s += mv;
        sc[ic] = s;
        if (s > M)
            M = s;
    }
    double S = 0.0;
    if (M != -INFINITY) {
        for (int64_t ic = 0; ic < c->n_kv; ++ic) {
            if (sc[ic] == -INFINITY)
                continue;
            const double p = exp(sc[ic] - M);
            S += p;
            xqr_dequantize(a->v.type,
                           (const uint8_t *)a->v.data + ic * a->v.nb[1] + iv2 * a->v.nb[2] +
                               iv3 * a->v.nb[3],
                           vf, DV);
            for (int64_t d = 0; d < DV; ++d)
                acc[d] += p * vf[d];
        }
    }
    float *dst = a->dst + ((iq3 * c->n_q + iq1) * c->n_head + iq2) * DV;
    for (int64_t d = 0; d < DV; ++d)
        dst[d] = S > 0.0 ? (float)(acc[d] / S) : 0.0f;
    if (x->lse)
        x->lse[(iq3 * c->n_q + iq1) * c->n_head + iq2] = S > 0.0 ? (float)(M + log(S)) : -INFINITY;
    free(kf);
    free(acc);
    free(sc);
}

int xqr_flash_attn_f64(const xqr_fa_args *a, float *lse) {
    fa64_ctx x;
    if (fa_setup(a, &x.c))
        return -1;
    x.lse = lse;
    xqr_parallel(fa64_job, &x, x.c.n_q * x.c.n_head * x.c.n_seq,
                 a->n_workers > 0 ? a->n_workers : 1);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* RKVA range attention + LSE merge.                                         */

uint32_t xqr_split_k(uint32_t active, uint32_t mode) {
    if (mode == 0) {
        uint32_t k = (active + 255u) / 256u;
        return k < 1 ? 1 : (k > 32 ? 32 : k);
    }
    uint32_t target = 128, max_splits = 128;
    if (mode == 2) {
        target = 32;
        max_splits = 256;
    } else if (mode == 3) {
        target = 512;
        max_splits = 64;
    }
    uint32_t wanted = (active + target - 1) / target;
    uint32_t k = wanted < max_splits ? wanted : max_splits;
    if (k > 256)
        k = 256;
    return k < 1 ? 1 : k;
}

void xqr_lse_merge(const float *partials, uint32_t n_splits, uint32_t n_rows, uint32_t D,
                   float *out, float *lse) {
    const size_t stride = (size_t)D + 2;
    for (uint32_t r = 0; r < n_rows; ++r) {
        int invalid = 0;
        float M = -3.402823466e38f;
        for (uint32_t s = 0; s < n_splits; ++s) {
            const float *p = partials + ((size_t)s * n_rows + r) * stride;
            const float m = p[D], den = p[D + 1];
            if (den == 0.0f)
                continue;
            if (!isfinite(den) || den < 0.0f || !isfinite(m))
                invalid = 1;
            else
                M = fmaxf(M, m);
        }
        float sum = 0.0f;
        for (uint32_t s = 0; s < n_splits && !invalid; ++s) {
            const float *p = partials + ((size_t)s * n_rows + r) * stride;
            if (p[D + 1] != 0.0f)
                sum += p[D + 1] * expf(p[D] - M);
        }
        const float inv = sum == 0.0f ? 0.0f : 1.0f / sum;
        if (!invalid && (!isfinite(sum) || sum < 0.0f || !isfinite(inv)))
            invalid = 1;
        float l = sum == 0.0f ? -INFINITY : M + logf(sum);
        if (sum != 0.0f && !isfinite(l))
            invalid = 1;
        for (uint32_t d = 0; d < D && !invalid; ++d) {
            float acc = 0.0f;
            for (uint32_t s = 0; s < n_splits; ++s) {
                const float *p = partials + ((size_t)s * n_rows + r) * stride;
                if (p[D + 1] != 0.0f) {
                    if (!isfinite(p[d]))
                        invalid = 1;
                    acc += p[d] * expf(p[D] - M);
                }
            }
            const float o = acc * inv;
            if (!isfinite(o))
                invalid = 1;
            out[(size_t)r * D + d] = o;
        }
        if (invalid) {
            for (uint32_t d = 0; d < D; ++d)
                out[(size_t)r * D + d] = NAN;
            l = NAN;
        }
        if (lse)
            lse[r] = l;
    }
}

int xqr_range_attn(const xqr_range_args *a) {
    const uint32_t D = a->head_dim, H = a->n_head, Hkv = a->n_head_kv;
    if (!D || D % 32 || !Hkv || H % Hkv)
        return -1;
    const uint32_t split_k = a->split_k ? a->split_k : xqr_split_k(a->active, 0);
    const size_t rec = xqr_row_size(a->storage, D);
    const uint32_t rows = a->n_tokens * H;
    float *part = (float *)malloc((size_t)split_k * rows * (D + 2) * 4);
    float *kf = (float *)malloc((size_t)D * 8);
    if (!part || !kf) {
        free(part);
        free(kf);
        return -2;
    }
    float *vf = kf + D;
    const uint32_t split_rows = (a->active + split_k - 1) / split_k;
    for (uint32_t qi = 0; qi < a->n_tokens; ++qi) {
        const int32_t pos = a->positions[qi];
        const uint32_t causal =
            pos < (int32_t)a->origin ? 0u : (uint32_t)(pos - (int32_t)a->origin) + 1u;
        const uint32_t limit = a->active < causal ? a->active : causal;
        for (uint32_t h = 0; h < H; ++h) {
            const uint32_t kvh = h / (H / Hkv);
            const float *q = a->q + ((size_t)qi * H + h) * D;
            for (uint32_t sp = 0; sp < split_k; ++sp) {
                uint32_t b = sp * split_rows, e = (sp + 1) * split_rows;
                b = b < limit ? b : limit;
                e = e < limit ? e : limit;
                float *p = part + ((size_t)sp * rows + (size_t)qi * H + h) * (D + 2);
                float mx = -3.402823466e38f, den = 0.0f;
                memset(p, 0, (size_t)D * 4);
                for (uint32_t r = b; r < e; ++r) {
                    const size_t off = ((size_t)r * Hkv + kvh) * rec;
                    xqr_dequantize(a->storage, (const uint8_t *)a->k + off, kf, D);
                    xqr_dequantize(a->storage, (const uint8_t *)a->v + off, vf, D);
                    float dot = 0.0f;
                    for (uint32_t d = 0; d < D; ++d)
                        dot += q[d] * kf[d];
                    const float score = dot * a->kq_scale;
                    const float nm = fmaxf(mx, score);
                    const float ow = den == 0.0f ? 0.0f : expf(mx - nm);
                    const float w = expf(score - nm);
                    for (uint32_t d = 0; d < D; ++d)
                        p[d] = p[d] * ow + w * vf[d];
                    den = den * ow + w;
                    mx = nm;
                }
                p[D] = mx;
                p[D + 1] = den;
            }
        }
    }
    xqr_lse_merge(part, split_k, rows, D, a->out, a->lse);
    free(part);
    free(kf);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* GATED_DELTA_NET.                                                          */

typedef struct {
    const xqr_gdn_args *a;
    int64_t S_k, H_k, S_v, H, T, n_seq, rq3, rk3, h_off;
    float scale;
    size_t slot_floats;
} gdn_ctx;

static float reduce8(float p[8]) {
    for (int stride = 4; stride > 0; stride >>= 1)
        for (int l = 0; l < stride; ++l)
            p[l] += p[l + stride];
    return p[0];
}

#define GDN_AT(t, s, tt, hh) \
    ((const float *)((const uint8_t *)(t).data + (s) * (t).nb[3] + (tt) * (t).nb[2] + (hh) * (t).nb[1]))

static void gdn_job(void *p, int64_t unit, int w) {
    (void)w;
    const gdn_ctx *c = (const gdn_ctx *)p;
    const xqr_gdn_args *a = c->a;
    const int64_t h = unit % c->H, s = unit / c->H;
    const int64_t S_v = c->S_v, S_k = c->S_k;
    const int64_t hk = (h + c->h_off) % c->H_k;
    const int64_t sq = s / c->rq3, sk = s / c->rk3;
    float *st = (float *)malloc((size_t)S_v * S_k * 4);
    const float *init = (const float *)((const uint8_t *)a->state.data + s * a->state.nb[3] +
                                        h * a->state.nb[2]);
    for (int64_t j = 0; j < S_v; ++j)
        memcpy(st + j * S_k, (const uint8_t *)init + j * a->state.nb[1], (size_t)S_k * 4);
    float *y_base = a->dst;
    float *snap_base = a->dst + (size_t)S_v * c->H * c->T * c->n_seq;
    for (int64_t t = 0; t < c->T; ++t) {
        const float *q = GDN_AT(a->q, sq, t, hk);
        const float *k = GDN_AT(a->k, sk, t, hk);
        const float *v = GDN_AT(a->v, s, t, h);
        const float g = *GDN_AT(a->g, s, t, h);
        const float beta = *GDN_AT(a->beta, s, t, h);
        const float decay = expf(g);
        float *y = y_base + ((s * c->T + t) * c->H + h) * S_v;
        if (a->lanes8) {
            for (int64_t j = 0; j < S_v; ++j) {
                float kv[8] = {0}, at[8] = {0};
                float *row = st + j * S_k;
                for (int64_t i = 0; i < S_k; ++i) {
                    row[i] *= decay;
                    kv[i % 8] += row[i] * k[i];
                }
                const float delta = (v[j] - reduce8(kv)) * beta;
                for (int64_t i = 0; i < S_k; ++i) {
                    row[i] += k[i] * delta;
                    at[i % 8] += row[i] * q[i];
                }
                y[j] = reduce8(at) * c->scale;
            }
        } else {
            vec_scale_f32(S_v * S_k, st, decay);
            for (int64_t j = 0; j < S_v; ++j) {
                float *row = st + j * S_k;
                const float delta = (v[j] - vec_dot_f32(S_k, row, k)) * beta;
                vec_mad_f32(S_k, row, k, delta);
                y[j] = vec_dot_f32(S_k, row, q) * c->scale;
            }
        }
        const int64_t slot = c->T - 1 - t;
        const int K = a->slots;
        if ((K > 1 && slot < K) || (K == 1 && t + 1 == c->T)) {
            float *dst = snap_base + (size_t)(K == 1 ? 0 : slot) * c->slot_floats +
                         (size_t)(s * c->H + h) * S_v * S_k;
            memcpy(dst, st, (size_t)S_v * S_k * 4);
        }
    }
    free(st);
}

int xqr_gated_delta_net(const xqr_gdn_args *a) {
    gdn_ctx c;
    c.a = a;
    c.S_k = a->q.ne[0];
    c.H_k = a->q.ne[1];
    c.S_v = a->v.ne[0];
    c.H = a->v.ne[1];
    c.T = a->v.ne[2];
    c.n_seq = a->v.ne[3];
    const int64_t total = a->n_head_total > 0 ? a->n_head_total : c.H;
    if (c.S_k != c.S_v || a->k.ne[0] != c.S_k || a->k.ne[1] != c.H_k || total % c.H_k ||
        a->head_begin < 0 || a->head_begin + c.H > total || a->slots < 1 ||
        a->q.ne[2] != c.T || c.n_seq % a->q.ne[3] || c.n_seq % a->k.ne[3])
        return -1;
    c.h_off = a->head_begin % c.H_k;
    c.rq3 = c.n_seq / a->q.ne[3];
    c.rk3 = c.n_seq / a->k.ne[3];
    c.scale = 1.0f / sqrtf((float)c.S_v);
    c.slot_floats = (size_t)c.S_v * c.S_k * c.H * c.n_seq;
    xqr_parallel(gdn_job, &c, c.H * c.n_seq, a->n_workers > 0 ? a->n_workers : 1);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* std::mt19937 + std::uniform_real_distribution<float> (libstdc++), used to  */
/* regenerate the reference GDN selftest inputs (ggml_d3d12.cpp:243-258).    */
/* MT19937: Matsumoto & Nishimura 1998.  libstdc++ generate_canonical<float, */
/* 24> takes one 32-bit draw: float(u) / 2^32, clamped below 1.              */

void xqr_std_uniform(uint32_t seed, float lo, float hi, int64_t n, float *out) {
    uint32_t mt[624];
    mt[0] = seed;
    for (int i = 1; i < 624; ++i)
        mt[i] = 1812433253u * (mt[i - 1] ^ (mt[i - 1] >> 30)) + (uint32_t)i;
    int idx = 624;
    for (int64_t o = 0; o < n; ++o) {
        if (idx >= 624) {
            for (int i = 0; i < 624; ++i) {
                const uint32_t y = (mt[i] & 0x80000000u) | (mt[(i + 1) % 624] & 0x7fffffffu);
                mt[i] = mt[(i + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
            }
            idx = 0;
        }
        uint32_t y = mt[idx++];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        y ^= y >> 18;
        float r = (float)y / 4294967296.0f;
        if (r >= 1.0f)
            r = nextafterf(1.0f, 0.0f);
        out[o] = (hi - lo) * r + lo;
    }
}
