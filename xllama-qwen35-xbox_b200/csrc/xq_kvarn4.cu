// Native KVarN4 range attention (RKVA descriptor v1 resident image, head_dim
// 256): split partials over 4-bit Bee records, rotated F16 stage rows and the
// original-domain F16 precision tail, in the (acc[256], max, denom) partial
// layout the LSE merge reduces (xq_decode.cu).  Semantics as the reference's
// shaders/rkva/rkva_range_attn_kvarn4.hlsl:64-150: rows >= active - tail come
// from the tail and meet the original q; the other rows are in the rotated
// domain (WHT256 = Sylvester H256 / 16) and meet WHT(q); their value numerator
// is rotated back with WHT at the end of the split and added to the tail's,
// with one shared running max and denominator.
//
// One CTA = (split, KV head, query token), the G = n_head / n_head_kv query
// heads of that KV head, 256 threads.  Splits cover whole 128-row record
// groups.  A record group's four records (K and V, two 128-dim slices each)
// are double-buffered into shared memory with cp.async.  Scores use the
// factorised decode other_t * (sum_d (q_d scale_d) nib_dt + sum_d q_d zero_d)
// and the value numerator other_d * (sum_t (w_t scale_t) nib_td + sum_t w_t
// zero_t) are tensor-core products (mma.sync m16n8k16): the 4-bit values
// expand exactly to f16 in registers, the f32 query / weight operand is split
// into an f16 high part and remainder (two products, ~2^-22 relative), the
// accumulators stay in the mma fragment layout.  Stage and tail rows are read
// straight from global memory into the same products.
#include <cuda_fp16.h>
#include <float.h>
#include <math.h>

#include "xq_common.cuh"
#include "xq_internal.h"

namespace xq {

namespace k4 {
constexpr int NT = 256;
constexpr int GMAX = 8;         // query heads per KV head
constexpr int REC = 8960;       // bytes per record
constexpr int GROUP = 128;      // rows per record group
constexpr int SET = 4 * REC;    // K slice 0, K slice 1, V slice 0, V slice 1
// shared memory
constexpr int SM_REC = 0;                        // 2 x SET
constexpr int SM_Q = SM_REC + 2 * SET;           // q [G][256] original
constexpr int SM_QR = SM_Q + GMAX * 256 * 4;     // WHT(q) [G][256]
constexpr int SM_QS = SM_QR + GMAX * 256 * 4;    // per group: q_r * scale_k, [2][128][8]
constexpr int SM_P = SM_QS + 2 * 128 * 8 * 4;    // slice partial scores [2][8][128]
constexpr int SM_S = SM_P + 2 * 8 * 128 * 4;     // scores -> weights [8][128]
constexpr int SM_WS = SM_QS;                     // weights * scale_v, [2][128][8] (the
                                                 // value pass, after the scores)
constexpr int SM_RED = SM_S + 8 * 128 * 4;       // small vectors
constexpr int SM_BYTES = SM_RED + 4 * 64 * 4;
} // namespace k4

struct Kvarn4Args {
    const uint8_t *k, *v; // planes
    const float *q;       // [n_tokens][n_head][256]
    const int32_t *positions;
    float *partials;      // [n_splits][n_tokens * n_head][258]
    int64_t records_bytes, stage_off, tail_off;
    int origin, active, tail, n_head, n_head_kv, n_tokens, rows_per_split;
    float scale;
};

__device__ __forceinline__ float h2f(const uint8_t *p) {
    return __half2float(*reinterpret_cast<const __half *>(p));
}

// In-place WHT256 of x[G][256] in shared memory (thread = dimension): the
// reference's order, seven butterfly strides inside each 128-slice, 1/sqrt(128)
// per slice, then the (a + b, a - b) / sqrt(2) slice mix.
__device__ void wht256_smem(float *x, int G, int d) {
    for (int stride = 1; stride < 128; stride <<= 1) {
        float nv[k4::GMAX];
#pragma unroll
        for (int g = 0; g < k4::GMAX; ++g)
            if (g < G) {
                const float own = x[g * 256 + d], oth = x[g * 256 + (d ^ stride)];
                nv[g] = (d & stride) ? oth - own : own + oth;
            }
        __syncthreads();
#pragma unroll
        for (int g = 0; g < k4::GMAX; ++g)
            if (g < G)
                x[g * 256 + d] = nv[g];
        __syncthreads();
    }
    float nv[k4::GMAX];
    const int lo = d & 127;
#pragma unroll
    for (int g = 0; g < k4::GMAX; ++g)
        if (g < G) {
            const float a = x[g * 256 + lo] * 0.08838834764831845f;
            const float b = x[g * 256 + lo + 128] * 0.08838834764831845f;
            nv[g] = (d < 128 ? a + b : a - b) * 0.7071067811865475f;
        }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < k4::GMAX; ++g)
        if (g < G)
            x[g * 256 + d] = nv[g];
    __syncthreads();
}

namespace k4 {
// Per-CTA shared-memory views and indices, passed by value to the inlined
// phases (nothing of the kernel's state has its address taken).
struct Cta {
    float *q, *qr, *qs, *p, *s, *ws, *red; // red: [0,16) qz, [16,24) m, [24,32) den,
                                           // [32,40) alpha, [40,56) wz
    int tid, warp, lane, g, c, G;          // g = lane / 4, c = lane % 4 (mma fragments)
};

// D += A B, m16n8k16, f16 inputs, f32 accumulate.  Rows 8..15 of A are zero
// here (at most 8 query heads per KV head), so their registers are 0.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
// f32 pair -> f16x2 high part and f16x2 remainder: x = hi + lo to about 2^-22
// relative, so two f16 products carry an fp32 operand
__device__ __forceinline__ void split2(float x, float y, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
// two 4-bit values -> f16x2 exactly: 0x6400 | n is the f16 1024 + n
__device__ __forceinline__ uint32_t nib2(uint32_t n0, uint32_t n1) {
    const uint32_t v = n0 | (n1 << 16) | 0x64006400u;
    const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&v), __floats2half2_rn(1024.f, 1024.f));
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t h2pair(const uint8_t *p0, const uint8_t *p1) {
    return (uint32_t) * reinterpret_cast<const uint16_t *>(p0) |
           ((uint32_t) * reinterpret_cast<const uint16_t *>(p1) << 16);
}

// Online softmax over the scores in s[g][0..n): running max / denominator
// update, weights back into s, per-query rescale factor in red[32 + g].
__device__ __forceinline__ void softmax_tile(const Cta c, int n) {
    if (c.warp < c.G) {
        const int g = c.warp;
        float mx = -FLT_MAX;
        for (int t = c.lane; t < n; t += 32)
            mx = fmaxf(mx, c.s[g * 128 + t]);
#pragma unroll
        for (int o = 16; o; o >>= 1)
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float m_old = c.red[16 + g], den_old = c.red[24 + g];
        const float m_new = fmaxf(m_old, mx);
        const float alpha = den_old == 0.0f ? 0.0f : __expf(m_old - m_new);
        float sum = 0.0f;
        for (int t = c.lane; t < n; t += 32) {
            const float w = __expf(c.s[g * 128 + t] - m_new);
            c.s[g * 128 + t] = w;
            sum += w;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1)
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (c.lane == 0) {
            c.red[16 + g] = m_new;
            c.red[24 + g] = den_old * alpha + sum;
            c.red[32 + g] = alpha;
        }
    }
    __syncthreads();
}

// A fragment (rows g < G, columns k0 + 2c, +1, +8, +9) of a [8][ld] float
// matrix with row stride ld (or of a [k][8] matrix when transposed), as hi/lo
__device__ __forceinline__ void afrag(const Cta c, const float *m, int k0, int rs, int ks,
                                      uint32_t &a0h, uint32_t &a0l, uint32_t &a2h, uint32_t &a2l) {
    const int k = k0 + 2 * c.c;
    const bool on = c.g < c.G;
    const float *r = m + c.g * rs;
    split2(on ? r[k * ks] : 0.f, on ? r[(k + 1) * ks] : 0.f, a0h, a0l);
    split2(on ? r[(k + 8) * ks] : 0.f, on ? r[(k + 9) * ks] : 0.f, a2h, a2l);
}

// n <= 128 consecutive F16 rows (row stride row_bytes; this KV head's 256
// values): stage rows (rotated, meet WHT(q), accumulate into acc_r) or tail
// rows (original, meet q, accumulate into acc_t).  Accumulators are in the
// mma C layout: query head g, dims 32 warp + 8 i + 2 c + {0, 1}.
template <bool ORIGINAL>
__device__ __forceinline__ void f16_tile(const Cta c, const uint8_t *krows, const uint8_t *vrows,
                                         int64_t row_bytes, int n, float scale,
                                         float (&acc_r)[4][2], float (&acc_t)[4][2]) {
    {
        // scores: warp w takes rows 16 w .. 16 w + 15 (two 8-row n-tiles)
        float dk[2][4] = {};
        const float *qv = ORIGINAL ? c.q : c.qr;
        for (int kk = 0; kk < 16; ++kk) {
            uint32_t a0h, a0l, a2h, a2l;
            afrag(c, qv, 16 * kk, 256, 1, a0h, a0l, a2h, a2l);
#pragma unroll
            for (int ti = 0; ti < 2; ++ti) {
                const int row = 16 * c.warp + 8 * ti + c.g;
                uint32_t b0 = 0, b1 = 0;
                if (row < n) {
                    const uint8_t *kr = krows + row * row_bytes + 2 * (16 * kk + 2 * c.c);
                    b0 = __ldg(reinterpret_cast<const uint32_t *>(kr));
                    b1 = __ldg(reinterpret_cast<const uint32_t *>(kr + 16));
                }
                mma16816(dk[ti], a0h, a2h, b0, b1);
                mma16816(dk[ti], a0l, a2l, b0, b1);
            }
        }
        if (c.g < c.G)
#pragma unroll
            for (int ti = 0; ti < 2; ++ti)
#pragma unroll
                for (int x = 0; x < 2; ++x) {
                    const int t = 16 * c.warp + 8 * ti + 2 * c.c + x;
                    c.s[c.g * 128 + t] = t < n ? dk[ti][x] * scale : -FLT_MAX;
                }
    }
    __syncthreads();
    softmax_tile(c, n);
    {
        // value numerator: warp w takes dims 32 w .. 32 w + 31 (four n-tiles)
        float dv[4][4] = {};
        for (int kk = 0; kk < (n + 15) / 16; ++kk) {
            uint32_t a0h, a0l, a2h, a2l;
            const int k = 16 * kk + 2 * c.c;
            const bool on = c.g < c.G;
            const float *wr = c.s + c.g * 128;
            split2(on && k < n ? wr[k] : 0.f, on && k + 1 < n ? wr[k + 1] : 0.f, a0h, a0l);
            split2(on && k + 8 < n ? wr[k + 8] : 0.f, on && k + 9 < n ? wr[k + 9] : 0.f, a2h, a2l);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = 32 * c.warp + 8 * i + c.g;
                const uint8_t *vr = vrows + 2 * d;
                const uint32_t b0 = h2pair(k < n ? vr + k * row_bytes : vr,
                                           k + 1 < n ? vr + (k + 1) * row_bytes : vr);
                const uint32_t b1 = h2pair(k + 8 < n ? vr + (k + 8) * row_bytes : vr,
                                           k + 9 < n ? vr + (k + 9) * row_bytes : vr);
                mma16816(dv[i], a0h, a2h, b0, b1);
                mma16816(dv[i], a0l, a2l, b0, b1);
            }
        }
        if (c.g < c.G) {
            const float al = c.red[32 + c.g];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int x = 0; x < 2; ++x) {
                    if (ORIGINAL) {
                        acc_t[i][x] = acc_t[i][x] * al + dv[i][x];
                        acc_r[i][x] *= al;
                    } else {
                        acc_r[i][x] = acc_r[i][x] * al + dv[i][x];
                        acc_t[i][x] *= al;
                    }
                }
        }
    }
    __syncthreads();
}

// Rows [t0, t0 + n) of one complete record group whose four records (K slice
// 0/1, V slice 0/1) are in shared memory at rk.
__device__ __forceinline__ void record_tile(const Cta c, const uint8_t *rk, int t0, int n,
                                            float scale, float (&acc_r)[4][2],
                                            float (&acc_t)[4][2]) {
    // per-group query factors: qs[s][d][g] = WHT(q)_g[s*128 + d] * scale_k_s[d],
    // qz[s][g] = sum_d WHT(q)_g[s*128 + d] * zero_k_s[d]
    {
        const int d = c.tid & 127, sl = c.tid >> 7;
        const uint8_t *rec = rk + sl * REC;
        const float sc = h2f(rec + 8192 + 2 * d), zr = h2f(rec + 8448 + 2 * d);
        float qv[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            qv[g] = g < c.G ? c.qr[g * 256 + sl * 128 + d] : 0.0f;
        float4 *qs4 = reinterpret_cast<float4 *>(c.qs + (sl * 128 + d) * 8);
        qs4[0] = make_float4(qv[0] * sc, qv[1] * sc, qv[2] * sc, qv[3] * sc);
        qs4[1] = make_float4(qv[4] * sc, qv[5] * sc, qv[6] * sc, qv[7] * sc);
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            float z = qv[g] * zr;
#pragma unroll
            for (int o = 16; o; o >>= 1)
                z += __shfl_xor_sync(0xffffffffu, z, o);
            if (c.lane == 0)
                c.p[(sl * 8 + g) * 128 + (d >> 5)] = z; // four warp sums per (s, g)
        }
    }
    __syncthreads();
    if (c.tid < 16) {
        const float *z = c.p + c.tid * 128;
        c.red[c.tid] = (z[0] + z[1]) + (z[2] + z[3]);
    }
    __syncthreads();
    {
        // scores: warp w takes tokens 16 w .. 16 w + 15 (two 8-token n-tiles);
        // K nibbles are [dim][token]: the word (d, tn) holds tokens 8 tn .. +7
        float dk[2][2][4] = {};
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
            const uint32_t *nw = reinterpret_cast<const uint32_t *>(rk + sl * REC);
            for (int kk = 0; kk < 8; ++kk) {
                uint32_t a0h, a0l, a2h, a2l;
                afrag(c, c.qs + sl * 128 * 8, 16 * kk, 1, 8, a0h, a0l, a2h, a2l);
                const int d = 16 * kk + 2 * c.c, sh = 4 * c.g;
#pragma unroll
                for (int ti = 0; ti < 2; ++ti) {
                    const int tn = 2 * c.warp + ti;
                    const uint32_t b0 = nib2((nw[d * 16 + tn] >> sh) & 15u,
                                             (nw[(d + 1) * 16 + tn] >> sh) & 15u);
                    const uint32_t b1 = nib2((nw[(d + 8) * 16 + tn] >> sh) & 15u,
                                             (nw[(d + 9) * 16 + tn] >> sh) & 15u);
                    mma16816(dk[sl][ti], a0h, a2h, b0, b1);
                    mma16816(dk[sl][ti], a0l, a2l, b0, b1);
                }
            }
        }
        if (c.g < c.G) {
            const float z0 = c.red[c.g], z1 = c.red[8 + c.g];
#pragma unroll
            for (int ti = 0; ti < 2; ++ti)
#pragma unroll
                for (int x = 0; x < 2; ++x) {
                    const int t = 16 * c.warp + 8 * ti + 2 * c.c + x;
                    const float o0 = h2f(rk + 8704 + 2 * t), o1 = h2f(rk + REC + 8704 + 2 * t);
                    const float sc = ((dk[0][ti][x] + z0) * o0 + (dk[1][ti][x] + z1) * o1) * scale;
                    if (t >= t0 && t < t0 + n)
                        c.s[c.g * 128 + (t - t0)] = sc;
                }
        }
    }
    __syncthreads();
    softmax_tile(c, n);
    {
        // weights * scale_v (indexed by token, zero outside the range) and
        // sum_t weights * zero_v, per slice
        const int t = c.tid & 127, sl = c.tid >> 7;
        const int j = t - t0;
        const bool in = j >= 0 && j < n;
        const uint8_t *vrec = rk + (2 + sl) * REC;
        const float sc = in ? h2f(vrec + 8192 + 2 * t) : 0.0f;
        const float zr = in ? h2f(vrec + 8448 + 2 * t) : 0.0f;
        float w[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            w[g] = (g < c.G && in) ? c.s[g * 128 + j] : 0.0f;
        float4 *ws4 = reinterpret_cast<float4 *>(c.ws + (sl * 128 + t) * 8);
        ws4[0] = make_float4(w[0] * sc, w[1] * sc, w[2] * sc, w[3] * sc);
        ws4[1] = make_float4(w[4] * sc, w[5] * sc, w[6] * sc, w[7] * sc);
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            float z = w[g] * zr;
#pragma unroll
            for (int o = 16; o; o >>= 1)
                z += __shfl_xor_sync(0xffffffffu, z, o);
            if (c.lane == 0)
                c.p[(sl * 8 + g) * 128 + (t >> 5)] = z;
        }
    }
    __syncthreads();
    if (c.tid < 16) {
        const float *z = c.p + c.tid * 128;
        c.red[40 + c.tid] = (z[0] + z[1]) + (z[2] + z[3]);
    }
    __syncthreads();
    {
        // value numerator: warp w takes dims 32 w .. +31 of slice w / 4;
        // V nibbles are [token][dim]: the word (t, dn) holds dims 8 dn .. +7
        const int sl = c.warp >> 2, dl = 32 * (c.warp & 3);
        const uint32_t *vw = reinterpret_cast<const uint32_t *>(rk + (2 + sl) * REC);
        float dv[4][4] = {};
        const int k_lo = t0 >> 4, k_hi = (t0 + n + 15) >> 4;
        for (int kk = k_lo; kk < k_hi; ++kk) {
            uint32_t a0h, a0l, a2h, a2l;
            afrag(c, c.ws + sl * 128 * 8, 16 * kk, 1, 8, a0h, a0l, a2h, a2l);
            const int t = 16 * kk + 2 * c.c, sh = 4 * c.g;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int dn = (dl >> 3) + i;
                const uint32_t b0 = nib2((vw[t * 16 + dn] >> sh) & 15u,
                                         (vw[(t + 1) * 16 + dn] >> sh) & 15u);
                const uint32_t b1 = nib2((vw[(t + 8) * 16 + dn] >> sh) & 15u,
                                         (vw[(t + 9) * 16 + dn] >> sh) & 15u);
                mma16816(dv[i], a0h, a2h, b0, b1);
                mma16816(dv[i], a0l, a2l, b0, b1);
            }
        }
        if (c.g < c.G) {
            const float al = c.red[32 + c.g], wz = c.red[40 + sl * 8 + c.g];
            const uint8_t *vrec = rk + (2 + sl) * REC;
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int x = 0; x < 2; ++x) {
                    const float other = h2f(vrec + 8704 + 2 * (dl + 8 * i + 2 * c.c + x));
                    acc_r[i][x] = acc_r[i][x] * al + (dv[i][x] + wz) * other;
                    acc_t[i][x] *= al;
                }
        }
    }
    __syncthreads();
}

// cp.async of group grp's four records of KV head kv into dst
__device__ __forceinline__ void prefetch_group(const Kvarn4Args &a, uint8_t *dst, int grp,
                                               int kv, int tid) {
    const int phys = 2 * a.n_head_kv;
    for (int i = tid; i < SET / 16; i += NT) {
        const int which = i / (REC / 16), off = (i % (REC / 16)) * 16;
        const uint8_t *plane = which < 2 ? a.k : a.v;
        cp_async<16>(smem_u32(dst + which * REC + off),
                     plane + ((int64_t)grp * phys + 2 * kv + (which & 1)) * REC + off);
    }
}
} // namespace k4

__global__ void __launch_bounds__(k4::NT, 2) kvarn4_partials_kernel(const Kvarn4Args a) {
    using namespace k4;
    extern __shared__ __align__(16) uint8_t sm[];
    Cta c;
    c.q = reinterpret_cast<float *>(sm + SM_Q);
    c.qr = reinterpret_cast<float *>(sm + SM_QR);
    c.qs = reinterpret_cast<float *>(sm + SM_QS);
    c.p = reinterpret_cast<float *>(sm + SM_P);
    c.s = reinterpret_cast<float *>(sm + SM_S);
    c.ws = reinterpret_cast<float *>(sm + SM_WS);
    c.red = reinterpret_cast<float *>(sm + SM_RED);
    c.tid = threadIdx.x;
    c.warp = c.tid >> 5;
    c.lane = c.tid & 31;
    c.g = c.lane >> 2;
    c.c = c.lane & 3;
    c.G = a.n_head / a.n_head_kv;
    const int split = blockIdx.x, kv = blockIdx.y, tok = blockIdx.z;
    const int64_t row_bytes = (int64_t)a.n_head_kv * 512;

    // ---- the query rows of this KV head, original and rotated
    for (int i = c.tid; i < c.G * 256; i += NT) {
        const int g = i >> 8, d = i & 255;
        const float x = a.q[((int64_t)tok * a.n_head + kv * c.G + g) * 256 + d];
        c.q[i] = x;
        c.qr[i] = x;
    }
    if (c.tid < GMAX) {
        c.red[16 + c.tid] = -FLT_MAX;
        c.red[24 + c.tid] = 0.0f;
    }
    __syncthreads();
    wht256_smem(c.qr, c.G, c.tid);

    const int pos = a.positions[tok];
    const int limit = pos < a.origin ? 0 : min(a.active, pos - a.origin + 1);
    const int r0 = split * a.rows_per_split;
    const int r1 = min(r0 + a.rows_per_split, limit);
    const int tail_begin = a.active - min(a.active, a.tail);
    const int live = a.active ? (a.active - 1) / GROUP : 0;
    const bool live_partial = (a.active % GROUP) != 0;
    const int og = a.origin / GROUP;
    float acc_r[4][2] = {}, acc_t[4][2] = {};

    // a group is read from its records when it has rows in [r0, r1) below the
    // tail and is neither the global sink group nor the incomplete live group
    const int g0 = r0 / GROUP, g1 = r1 > r0 ? (r1 + GROUP - 1) / GROUP : g0;
    auto record_group = [=](int grp) {
        const int lo = max(r0, grp * GROUP), hi = min(min(r1, (grp + 1) * GROUP), tail_begin);
        return lo < hi && og + grp != 0 && !(grp == live && live_partial);
    };
    int next = g0;
    while (next < g1 && !record_group(next))
        ++next;
    int buf = 0;
    if (next < g1)
        prefetch_group(a, sm + SM_REC, next, kv, c.tid);
    cp_async_commit();
    for (int grp = g0; grp < g1; ++grp) {
        const int lo = max(r0, grp * GROUP), hi = min(r1, (grp + 1) * GROUP);
        const int body_hi = min(hi, tail_begin);
        if (lo < body_hi) {
            if (!record_group(grp)) {
                // staged group: rotated F16 rows in its stage slot
                const int slot = og + grp == 0 ? 0 : 1 + ((og + grp - 1) & 1);
                const int64_t first = ((int64_t)slot * GROUP + (lo - grp * GROUP)) * row_bytes +
                                      kv * 512;
                f16_tile<false>(c, a.k + a.stage_off + first, a.v + a.stage_off + first,
                                row_bytes, body_hi - lo, a.scale, acc_r, acc_t);
            } else {
                int nxt = grp + 1;
                while (nxt < g1 && !record_group(nxt))
                    ++nxt;
                if (nxt < g1)
                    prefetch_group(a, sm + SM_REC + (buf ^ 1) * SET, nxt, kv, c.tid);
                cp_async_commit();
                cp_async_wait<1>();
                __syncthreads();
                record_tile(c, sm + SM_REC + buf * SET, lo - grp * GROUP, body_hi - lo, a.scale,
                            acc_r, acc_t);
                buf ^= 1;
            }
        }
        const int tail_lo = max(lo, tail_begin);
        if (tail_lo < hi) {
            const int64_t first = (int64_t)(tail_lo % GROUP) * row_bytes + kv * 512;
            f16_tile<true>(c, a.k + a.tail_off + first, a.v + a.tail_off + first, row_bytes,
                           hi - tail_lo, a.scale, acc_r, acc_t);
        }
    }
    cp_async_wait<0>();

    // ---- numerator = WHT(rotated part) + tail part; partial record
    float *x = c.qr;  // the rotated query is no longer needed
    float *xt = c.qs; // tail part (the group factors are no longer needed)
    __syncthreads();
    if (c.g < c.G)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int d = 32 * c.warp + 8 * i + 2 * c.c + e;
                x[c.g * 256 + d] = acc_r[i][e];
                xt[c.g * 256 + d] = acc_t[i][e];
            }
    __syncthreads();
    wht256_smem(x, c.G, c.tid);
    const int64_t n_rows = (int64_t)a.n_tokens * a.n_head;
    for (int g = 0; g < c.G; ++g) {
        const int64_t row = (int64_t)tok * a.n_head + kv * c.G + g;
        float *rec = a.partials + ((int64_t)split * n_rows + row) * 258;
        rec[c.tid] = x[g * 256 + c.tid] + xt[g * 256 + c.tid];
        if (c.tid == 0) {
            rec[256] = c.red[16 + g];
            rec[257] = c.red[24 + g];
        }
    }
}

cudaError_t launch_kvarn4(const Kvarn4Launch &l, cudaStream_t st) {
    Kvarn4Args a;
    a.k = l.k;
    a.v = l.v;
    a.q = l.q;
    a.positions = l.positions;
    a.partials = l.partials;
    a.records_bytes = l.records_bytes;
    a.stage_off = l.records_bytes;
    a.tail_off = l.records_bytes + (int64_t)384 * l.n_head_kv * 512;
    a.origin = l.origin;
    a.active = l.active;
    a.tail = l.tail;
    a.n_head = l.n_head;
    a.n_head_kv = l.n_head_kv;
    a.n_tokens = l.n_tokens;
    a.rows_per_split = l.rows_per_split;
    a.scale = l.scale;
    static std::atomic<unsigned long long> attr{0};
    cudaError_t e = set_smem_limit((const void *)kvarn4_partials_kernel, k4::SM_BYTES, attr);
    if (e != cudaSuccess)
        return e;
    dim3 grid((unsigned)l.n_splits, (unsigned)l.n_head_kv, (unsigned)l.n_tokens);
    kvarn4_partials_kernel<<<grid, k4::NT, k4::SM_BYTES, st>>>(a);
    return cudaGetLastError();
}

} // namespace xq
