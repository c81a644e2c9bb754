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
// One CTA = (split, KV head, query token), the G = n_head / n_head_kv <= 8
// query heads of that KV head, 256 threads, two CTAs per SM.  Splits cover
// whole 128-row record groups.  A record group's four records (K and V, two
// 128-dim slices each) are double-buffered into shared memory by one thread:
// each record's 128 nibble rows of 64 bytes as one TMA box with the 64-byte
// swizzle (16-byte chunk c of row r lands at chunk c ^ ((r / 2) % 4), which
// makes the fragment loads below free of bank conflicts) and its 768 bytes of
// F16 axes as one bulk copy, all completing on the buffer's mbarrier.
//
// Every product is a tensor-core mma.sync m16n8k16 whose A operand is the KV
// side (16 tokens for scores, 16 dims for the value numerator) and whose B
// operand is the G query heads (n = 8):
//   scores  s_t = other_t * (sum_d (q_d scale_d) nib_dt + sum_d q_d zero_d)
//   values  n_d = other_d * (sum_t (w_t scale_t) nib_td + sum_t w_t zero_t)
// A lane's A fragment is one byte of two words: its low nibbles are rows g and
// its high nibbles rows g + 8 (the m axis is permuted so row g is token / dim
// 2g and row g + 8 is 2g + 1 of the 16), expanded exactly to f16 with one
// byte permute, one mask and one f16 multiply-add.  The fp32 query / weight
// side is split into an f16 high part and remainder (two products, ~2^-22
// relative).  Stage and tail rows are read straight from global memory into
// the same products: F16 K rows are already A fragments; F16 V pairs are
// byte-permuted into them.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <float.h>
#include <math.h>

#include "xq_common.cuh"
#include "xq_internal.h"
#include "xq_tc.cuh"

namespace xq {

namespace k4 {
constexpr int NT = 256;
constexpr int GMAX = 8;      // query heads per KV head
constexpr int REC = 8960;    // bytes per record
constexpr int NIB = 8192;    // its 128 x 128 nibbles (128 rows of 64 bytes)
constexpr int AXB = 768;     // then 128 F16 scales, zeros, factors
constexpr int GROUP = 128;   // rows per record group
// a record group in shared memory: the nibbles of K slice 0, K slice 1, V
// slice 0, V slice 1 (512-byte aligned: the swizzle's period), then their axes
constexpr int SET = 4 * REC;
__host__ __device__ constexpr int nib_off(int which) { return which * NIB; }
__host__ __device__ constexpr int ax_off(int which) { return 4 * NIB + which * AXB; }
constexpr int QLD = 264;     // padded row stride (floats) of [8][256] query / numerator rows
constexpr int SLD = 136;     // padded row stride of the [8][128] scores
// shared memory
constexpr int SM_REC = 0;                      // 2 x SET; x / xt numerators after the loop
constexpr int SM_QR = SM_REC + 2 * SET;        // WHT(q) [8][QLD]
constexpr int SM_BF = SM_QR + GMAX * QLD * 4;  // B fragments of a tile [2][8][32] uint4
constexpr int SM_FQ = SM_BF + 2 * 8 * 32 * 16; // F16-tile B fragments of q [16][32] uint4
constexpr int SM_FQR = SM_FQ + 16 * 32 * 16;   // ... of WHT(q)
constexpr int SM_S = SM_FQR + 16 * 32 * 16;    // scores -> weights [8][SLD]
constexpr int SM_MX = SM_S + GMAX * SLD * 4;   // per-warp tile max [8 warps][8]
constexpr int SM_ZP = SM_MX + 8 * 8 * 4;       // zero-point partials [2 slices][8][4]
constexpr int SM_DP = SM_ZP + 2 * 8 * 4 * 4;   // denominator partials [8][8]
constexpr int SM_ST = SM_DP + 8 * 8 * 4;       // m, den, alpha, m_new [4][8]
constexpr int SM_BAR = SM_ST + 4 * 8 * 4;      // two mbarriers (one per record buffer), a zero word
constexpr int SM_BYTES = SM_BAR + 32 + 512;    // + alignment slack
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

namespace k4 {
// Per-CTA shared-memory views and lane indices, passed by value to the
// inlined phases (nothing of the kernel's state has its address taken).
struct Cta {
    uint8_t *sm;
    float *qr, *s, *mx, *zp, *dp, *st; // st: [0,8) m, [8,16) den, [16,24) alpha, [24,32) m_new
    uint4 *bf, *fq, *fqr;
    int tid, warp, lane, g, c, G;      // g = lane / 4, c = lane % 4 (mma fragments)
    uint32_t sel;                      // byte permute: byte g % 4 of two words -> bytes 0, 2
};

// D += A B, m16n8k16, f16 inputs, f32 accumulate
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
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
__device__ __forceinline__ uint4 split4(float x0, float x1, float x8, float x9) {
    uint4 f;
    split2(x0, x1, f.x, f.z);
    split2(x8, x9, f.y, f.w);
    return f;
}
// Byte g % 4 of words x (-> row g, k pair low half) and y (high half): low
// nibbles -> f16x2 of row g, high nibbles -> row g + 8.  0x6400 | n is the f16
// 1024 + n and 0x6400 | 16 n is 1024 + 16 n; both map back to n exactly.
__device__ __forceinline__ void nib_frag(uint32_t x, uint32_t y, uint32_t sel, uint32_t &lo,
                                         uint32_t &hi) {
    const uint32_t t = __byte_perm(x, y, sel);
    const uint32_t a = (t & 0x000f000fu) | 0x64006400u, b = (t & 0x00f000f0u) | 0x64006400u;
    const __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a), __float2half2_rn(1024.f));
    const __half2 hb = __hfma2(*reinterpret_cast<const __half2 *>(&b), __float2half2_rn(0.0625f),
                               __float2half2_rn(-64.f));
    lo = *reinterpret_cast<const uint32_t *>(&ha);
    hi = *reinterpret_cast<const uint32_t *>(&hb);
}
__device__ __forceinline__ uint32_t lds32(const uint8_t *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}
// two F16 values at p (4-byte aligned) as floats
__device__ __forceinline__ float2 h2x2(const uint8_t *p) {
    return __half22float2(*reinterpret_cast<const __half2 *>(p));
}
__device__ __forceinline__ float sum4(const float *p) {
    const float4 v = *reinterpret_cast<const float4 *>(p);
    return (v.x + v.y) + (v.z + v.w);
}

// In-register WHT256 of the 256-vector held as v[i] = x[8 lane + i] by one
// warp: Sylvester butterflies (a + b, a - b) over the index bits, three inside
// the lane and five across lanes, then / 16.
__device__ __forceinline__ void wht_regs(float (&v)[8], int lane) {
#pragma unroll
    for (int s = 1; s < 8; s <<= 1)
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (!(i & s)) {
                const float a = v[i], b = v[i + s];
                v[i] = a + b;
                v[i + s] = a - b;
            }
#pragma unroll
    for (int m = 1; m < 32; m <<= 1)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float o = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = (lane & m) ? o - v[i] : v[i] + o;
        }
#pragma unroll
    for (int i = 0; i < 8; ++i)
        v[i] *= 0.0625f;
}
// F16-tile B fragments of query head g from v[i] = x[8 lane + i]: MMA step
// 2j + h covers dims 32 j + 8 c + 4 h + {0, 1} (b0) and {2, 3} (b1), matching
// a 16-byte K row load per lane.
__device__ __forceinline__ void q_frags(const float (&v)[8], uint4 *f, int g, int lane) {
    const int j = lane >> 2, cc = lane & 3;
#pragma unroll
    for (int h = 0; h < 2; ++h)
        f[(2 * j + h) * 32 + 4 * g + cc] = split4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
}

// Scores of tokens (row, row + 1) x queries (2c, 2c + 1) into s, and the warp's
// per-query max into mx.  sv = {(row, q0), (row, q1), (row + 1, q0), (row + 1, q1)}.
__device__ __forceinline__ void put_scores(const Cta c, int row, const float (&sv)[4]) {
    const int q0 = 2 * c.c;
    *reinterpret_cast<float2 *>(c.s + q0 * SLD + row) = make_float2(sv[0], sv[2]);
    *reinterpret_cast<float2 *>(c.s + (q0 + 1) * SLD + row) = make_float2(sv[1], sv[3]);
    float m0 = fmaxf(sv[0], sv[2]), m1 = fmaxf(sv[1], sv[3]);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    if (c.g == 0) {
        c.mx[c.warp * 8 + q0] = m0;
        c.mx[c.warp * 8 + q0 + 1] = m1;
    }
}
// Running max after this tile for query q (< G); thread tid < 8 also publishes
// alpha = exp(m_old - m_new) and m_new of query tid.
__device__ __forceinline__ float tile_max(const Cta c, int q) {
    float m = c.st[q];
#pragma unroll
    for (int w = 0; w < 8; ++w)
        m = fmaxf(m, c.mx[w * 8 + q]);
    return m;
}
__device__ __forceinline__ void publish_alpha(const Cta c) {
    if (c.tid < GMAX) {
        const int q = c.tid;
        if (q < c.G) {
            const float m_new = tile_max(c, q);
            c.st[16 + q] = c.st[8 + q] == 0.0f ? 0.0f : __expf(c.st[q] - m_new);
            c.st[24 + q] = m_new;
        } else {
            c.st[16 + q] = 0.0f;
        }
    }
}
// After the value pass: den = den * alpha + tile sum, m = m_new
__device__ __forceinline__ void update_state(const Cta c) {
    if (c.tid < c.G) {
        const int q = c.tid;
        c.st[8 + q] = c.st[8 + q] * c.st[16 + q] + (sum4(c.dp + q * 8) + sum4(c.dp + q * 8 + 4));
        c.st[q] = c.st[24 + q];
    }
}

// n <= 128 consecutive F16 rows (row stride row_bytes; this KV head's 256
// values): stage rows (rotated, meet WHT(q), accumulate into acc_r) or tail
// rows (original, meet q, accumulate into acc_t).  acc[mt][.] is the mma D
// layout of the value numerator: rows = dims 32 warp + 16 mt + 2 g + {0, 1},
// columns = queries 2c, 2c + 1.
template <bool ORIGINAL>
__device__ __forceinline__ void f16_tile(const Cta c, const uint8_t *krows, const uint8_t *vrows,
                                         int64_t row_bytes, int n, float scale,
                                         float (&acc_r)[2][4], float (&acc_t)[2][4]) {
    {
        // scores: warp w takes rows 16 w + 2 g (A row g) and + 1 (A row g + 8)
        const int row = 16 * c.warp + 2 * c.g;
        const bool va = row < n, vb = row + 1 < n;
        const uint8_t *pa = krows + (int64_t)row * row_bytes + 16 * c.c;
        const uint8_t *pb = pa + row_bytes;
        const uint4 *fb = ORIGINAL ? c.fq : c.fqr;
        const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
        uint4 ka[8], kb[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            ka[j] = va ? __ldg(reinterpret_cast<const uint4 *>(pa + 64 * j)) : z4;
            kb[j] = vb ? __ldg(reinterpret_cast<const uint4 *>(pb + 64 * j)) : z4;
        }
        float d[4] = {};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint4 f0 = fb[(2 * j) * 32 + c.lane], f1 = fb[(2 * j + 1) * 32 + c.lane];
            mma16816(d, ka[j].x, kb[j].x, ka[j].y, kb[j].y, f0.x, f0.y);
            mma16816(d, ka[j].x, kb[j].x, ka[j].y, kb[j].y, f0.z, f0.w);
            mma16816(d, ka[j].z, kb[j].z, ka[j].w, kb[j].w, f1.x, f1.y);
            mma16816(d, ka[j].z, kb[j].z, ka[j].w, kb[j].w, f1.z, f1.w);
        }
        const float sv[4] = {va ? d[0] * scale : -INFINITY, va ? d[1] * scale : -INFINITY,
                             vb ? d[2] * scale : -INFINITY, vb ? d[3] * scale : -INFINITY};
        put_scores(c, row, sv);
    }
    __syncthreads();
    {
        // weights: warp w takes tokens 16 w .. 16 w + 15 (B fragments of MMA step w)
        publish_alpha(c);
        float dsum = 0.0f;
        uint4 f = make_uint4(0u, 0u, 0u, 0u);
        if (c.g < c.G) {
            const float m = tile_max(c, c.g);
            const float *sr = c.s + c.g * SLD + 16 * c.warp + 2 * c.c;
            const float2 s01 = *reinterpret_cast<const float2 *>(sr);
            const float2 s89 = *reinterpret_cast<const float2 *>(sr + 8);
            const float w0 = __expf(s01.x - m), w1 = __expf(s01.y - m);
            const float w8 = __expf(s89.x - m), w9 = __expf(s89.y - m);
            f = split4(w0, w1, w8, w9);
            dsum = (w0 + w1) + (w8 + w9);
        }
        c.bf[c.warp * 32 + c.lane] = f;
        dsum += __shfl_xor_sync(0xffffffffu, dsum, 1);
        dsum += __shfl_xor_sync(0xffffffffu, dsum, 2);
        if (c.c == 0)
            c.dp[c.g * 8 + c.warp] = dsum;
    }
    __syncthreads();
    {
        // value numerator: warp w takes dims 32 w + 16 mt + 2 g (+ 1); lane
        // loads the dim pair of tokens 16 kk + 2c + {0, 1, 8, 9}
        const uint8_t *vp = vrows + 2 * (32 * c.warp + 2 * c.g);
        float dv[2][4] = {};
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const int t = 16 * kk + 2 * c.c;
            uint32_t x[2][4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int te = t + (e & 1) + 8 * (e >> 1);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
                    x[mt][e] = te < n ? __ldg(reinterpret_cast<const uint32_t *>(
                                            vp + (int64_t)te * row_bytes + 32 * mt))
                                      : 0u;
            }
            const uint4 b = c.bf[kk * 32 + c.lane];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const uint32_t a0 = __byte_perm(x[mt][0], x[mt][1], 0x5410);
                const uint32_t a1 = __byte_perm(x[mt][0], x[mt][1], 0x7632);
                const uint32_t a2 = __byte_perm(x[mt][2], x[mt][3], 0x5410);
                const uint32_t a3 = __byte_perm(x[mt][2], x[mt][3], 0x7632);
                mma16816(dv[mt], a0, a1, a2, a3, b.x, b.y);
                mma16816(dv[mt], a0, a1, a2, a3, b.z, b.w);
            }
        }
        const float al0 = c.st[16 + 2 * c.c], al1 = c.st[17 + 2 * c.c];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float al = (i & 1) ? al1 : al0;
                if (ORIGINAL) {
                    acc_t[mt][i] = acc_t[mt][i] * al + dv[mt][i];
                    acc_r[mt][i] *= al;
                } else {
                    acc_r[mt][i] = acc_r[mt][i] * al + dv[mt][i];
                    acc_t[mt][i] *= al;
                }
            }
        update_state(c);
    }
}

// Rows [t0, t0 + n) of one complete record group whose four records (K slice
// 0/1, V slice 0/1; nibble rows swizzled) are in shared memory at rk.
__device__ __forceinline__ void record_tile(const Cta c, const uint8_t *rk, int t0, int n,
                                            float scale, float (&acc_r)[2][4],
                                            float (&acc_t)[2][4]) {
    const int fsl = c.tid >> 7, qt = (c.tid >> 5) & 3; // fragment passes: slice, quarter
    {
        // B fragments qs[d][g] = WHT(q)_g[d] * scale_k[d] of MMA steps qt, qt + 4
        // of slice fsl, and the partial sums of WHT(q) . zero_k
        const uint8_t *kax = rk + ax_off(fsl);
        float z = 0.0f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int kk = qt + 4 * h, dl = 16 * kk + 2 * c.c;
            const float *qrow = c.qr + c.g * QLD + fsl * 128 + dl;
            const float2 q01 = *reinterpret_cast<const float2 *>(qrow);
            const float2 q89 = *reinterpret_cast<const float2 *>(qrow + 8);
            const float2 s01 = h2x2(kax + 2 * dl), s89 = h2x2(kax + 2 * dl + 16);
            const float2 z01 = h2x2(kax + 256 + 2 * dl), z89 = h2x2(kax + 256 + 2 * dl + 16);
            c.bf[(fsl * 8 + kk) * 32 + c.lane] =
                split4(q01.x * s01.x, q01.y * s01.y, q89.x * s89.x, q89.y * s89.y);
            z += (q01.x * z01.x + q01.y * z01.y) + (q89.x * z89.x + q89.y * z89.y);
        }
        z += __shfl_xor_sync(0xffffffffu, z, 1);
        z += __shfl_xor_sync(0xffffffffu, z, 2);
        if (c.c == 0)
            c.zp[(fsl * 8 + c.g) * 4 + qt] = z;
    }
    __syncthreads();
    {
        // scores: warp w takes tokens 16 w + 2 g (+ 1), all 256 dims; the K
        // nibble rows are dims, the lane's word holds tokens 16 w + 8 (g / 4) ..
        const int w = c.warp;
        const int lane_off = 128 * c.c + 16 * ((w >> 1) ^ c.c) + 4 * (2 * (w & 1) + (c.g >> 2));
        float d[2][4] = {};
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
            const uint8_t *base = rk + nib_off(sl) + lane_off;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint8_t *p = base + kk * 1024;
                uint32_t a0, a1, a2, a3;
                nib_frag(lds32(p), lds32(p + 64), c.sel, a0, a1);
                nib_frag(lds32(p + 512), lds32(p + 576), c.sel, a2, a3);
                const uint4 b = c.bf[(sl * 8 + kk) * 32 + c.lane];
                mma16816(d[sl], a0, a1, a2, a3, b.x, b.y);
                mma16816(d[sl], a0, a1, a2, a3, b.z, b.w);
            }
        }
        const int row = 16 * w + 2 * c.g, q0 = 2 * c.c;
        const float2 o0 = h2x2(rk + ax_off(0) + 512 + 2 * row);
        const float2 o1 = h2x2(rk + ax_off(1) + 512 + 2 * row);
        const float z00 = sum4(c.zp + q0 * 4), z01 = sum4(c.zp + q0 * 4 + 4);
        const float z10 = sum4(c.zp + 32 + q0 * 4), z11 = sum4(c.zp + 32 + q0 * 4 + 4);
        const bool va = row >= t0 && row < t0 + n, vb = row + 1 >= t0 && row + 1 < t0 + n;
        const float sv[4] = {
            va ? (o0.x * (d[0][0] + z00) + o1.x * (d[1][0] + z10)) * scale : -INFINITY,
            va ? (o0.x * (d[0][1] + z01) + o1.x * (d[1][1] + z11)) * scale : -INFINITY,
            vb ? (o0.y * (d[0][2] + z00) + o1.y * (d[1][2] + z10)) * scale : -INFINITY,
            vb ? (o0.y * (d[0][3] + z01) + o1.y * (d[1][3] + z11)) * scale : -INFINITY};
        put_scores(c, row, sv);
    }
    __syncthreads();
    {
        // B fragments ws[t][g] = w_g[t] * scale_v[t] of MMA steps qt, qt + 4 of
        // slice fsl, and the partial sums of w . zero_v and of w
        publish_alpha(c);
        const uint8_t *vax = rk + ax_off(2 + fsl);
        float z = 0.0f, dsum = 0.0f;
        const bool on = c.g < c.G;
        const float m = on ? tile_max(c, c.g) : 0.0f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int kk = qt + 4 * h, t = 16 * kk + 2 * c.c;
            uint4 f = make_uint4(0u, 0u, 0u, 0u);
            if (on) {
                const float *sr = c.s + c.g * SLD + t;
                const float2 s01 = *reinterpret_cast<const float2 *>(sr);
                const float2 s89 = *reinterpret_cast<const float2 *>(sr + 8);
                const float w0 = __expf(s01.x - m), w1 = __expf(s01.y - m);
                const float w8 = __expf(s89.x - m), w9 = __expf(s89.y - m);
                const float2 c01 = h2x2(vax + 2 * t), c89 = h2x2(vax + 2 * t + 16);
                const float2 z01 = h2x2(vax + 256 + 2 * t), z89 = h2x2(vax + 256 + 2 * t + 16);
                f = split4(w0 * c01.x, w1 * c01.y, w8 * c89.x, w9 * c89.y);
                z += (w0 * z01.x + w1 * z01.y) + (w8 * z89.x + w9 * z89.y);
                dsum += (w0 + w1) + (w8 + w9);
            }
            c.bf[(fsl * 8 + kk) * 32 + c.lane] = f;
        }
        z += __shfl_xor_sync(0xffffffffu, z, 1);
        z += __shfl_xor_sync(0xffffffffu, z, 2);
        dsum += __shfl_xor_sync(0xffffffffu, dsum, 1);
        dsum += __shfl_xor_sync(0xffffffffu, dsum, 2);
        if (c.c == 0) {
            c.zp[(fsl * 8 + c.g) * 4 + qt] = z;
            c.dp[c.g * 8 + fsl * 4 + qt] = fsl == 0 ? dsum : 0.0f;
        }
    }
    __syncthreads();
    {
        // value numerator: warp w takes dims 16 mt + 2 g (+ 1) of unit
        // 2 (w % 4) + mt of slice w / 4, all 128 tokens; the V nibble rows are
        // tokens, the lane's word holds dims 16 unit + 8 (g / 4) ..
        const int w = c.warp, sl = w >> 2;
        const uint8_t *vbase = rk + nib_off(2 + sl) + 128 * c.c + 16 * ((w & 3) ^ c.c) + 4 * (c.g >> 2);
        float dv[2][4] = {};
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const uint4 b = c.bf[(sl * 8 + kk) * 32 + c.lane];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const uint8_t *p = vbase + kk * 1024 + 8 * mt;
                uint32_t a0, a1, a2, a3;
                nib_frag(lds32(p), lds32(p + 64), c.sel, a0, a1);
                nib_frag(lds32(p + 512), lds32(p + 576), c.sel, a2, a3);
                mma16816(dv[mt], a0, a1, a2, a3, b.x, b.y);
                mma16816(dv[mt], a0, a1, a2, a3, b.z, b.w);
            }
        }
        const int q0 = 2 * c.c;
        const float al0 = c.st[16 + q0], al1 = c.st[17 + q0];
        const float wz0 = sum4(c.zp + (sl * 8 + q0) * 4), wz1 = sum4(c.zp + (sl * 8 + q0) * 4 + 4);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            const float2 o = h2x2(rk + ax_off(2 + sl) + 512 + 2 * (32 * (w & 3) + 16 * mt + 2 * c.g));
            acc_r[mt][0] = acc_r[mt][0] * al0 + o.x * (dv[mt][0] + wz0);
            acc_r[mt][1] = acc_r[mt][1] * al1 + o.x * (dv[mt][1] + wz1);
            acc_r[mt][2] = acc_r[mt][2] * al0 + o.y * (dv[mt][2] + wz0);
            acc_r[mt][3] = acc_r[mt][3] * al1 + o.y * (dv[mt][3] + wz1);
            acc_t[mt][0] *= al0;
            acc_t[mt][1] *= al1;
            acc_t[mt][2] *= al0;
            acc_t[mt][3] *= al1;
        }
        update_state(c);
    }
}

// One thread: group grp's four records of KV head kv into the buffer at dst,
// completing on bar.  The tensor maps view each plane's records as rows of 64
// bytes (a record = 140 rows, its nibbles the first 128).
__device__ __forceinline__ void issue_group(const CUtensorMap *kmap, const CUtensorMap *vmap,
                                            const Kvarn4Args &a, uint8_t *dst, uint32_t bar,
                                            int grp, int kv) {
    tc::mbar_expect_tx(bar, SET);
    const int64_t r0 = (int64_t)grp * 2 * a.n_head_kv + 2 * kv;
#pragma unroll
    for (int which = 0; which < 4; ++which) {
        const int64_t r = r0 + (which & 1);
        tc::tma_load_2d(smem_u32(dst + nib_off(which)), which < 2 ? kmap : vmap, 0,
                        (int)(r * (REC / 64)), bar);
        tc::bulk_load(smem_u32(dst + ax_off(which)), (which < 2 ? a.k : a.v) + r * REC + NIB, AXB,
                      bar);
    }
}
} // namespace k4

__global__ void __launch_bounds__(k4::NT, 2)
    kvarn4_partials_kernel(const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, const Kvarn4Args a) {
    using namespace k4;
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sm_raw) + 511) &
                                              ~uintptr_t(511));
    Cta c;
    c.sm = sm;
    c.qr = reinterpret_cast<float *>(sm + SM_QR);
    c.s = reinterpret_cast<float *>(sm + SM_S);
    c.mx = reinterpret_cast<float *>(sm + SM_MX);
    c.zp = reinterpret_cast<float *>(sm + SM_ZP);
    c.dp = reinterpret_cast<float *>(sm + SM_DP);
    c.st = reinterpret_cast<float *>(sm + SM_ST);
    c.bf = reinterpret_cast<uint4 *>(sm + SM_BF);
    c.fq = reinterpret_cast<uint4 *>(sm + SM_FQ);
    c.fqr = reinterpret_cast<uint4 *>(sm + SM_FQR);
    c.tid = threadIdx.x;
    c.warp = c.tid >> 5;
    c.lane = c.tid & 31;
    c.g = c.lane >> 2;
    c.c = c.lane & 3;
    c.G = a.n_head / a.n_head_kv;
    {
        const uint32_t b = c.g & 3;
        c.sel = b | (b << 4) | ((b + 4) << 8) | ((b + 4) << 12);
    }
    const int split = blockIdx.x, kv = blockIdx.y, tok = blockIdx.z;
    const int64_t row_bytes = (int64_t)a.n_head_kv * 512;

    const int pos = a.positions[tok];
    const int limit = pos < a.origin ? 0 : min(a.active, pos - a.origin + 1);
    const int r0 = split * a.rows_per_split;
    const int r1 = min(r0 + a.rows_per_split, limit);
    const int tail_begin = a.active - min(a.active, a.tail);
    const int live = a.active ? (a.active - 1) / GROUP : 0;
    const bool live_partial = (a.active % GROUP) != 0;
    const int og = a.origin / GROUP;

    // a group is read from its records when it has rows in [r0, r1) below the
    // tail and is neither the global sink group nor the incomplete live group
    const int g0 = r0 / GROUP, g1 = r1 > r0 ? (r1 + GROUP - 1) / GROUP : g0;
    auto record_group = [=](int grp) {
        const int lo = max(r0, grp * GROUP), hi = min(min(r1, (grp + 1) * GROUP), tail_begin);
        return lo < hi && og + grp != 0 && !(grp == live && live_partial);
    };
    const uint32_t bar0 = smem_u32(sm + SM_BAR);
    volatile int *zero = reinterpret_cast<volatile int *>(sm + SM_BAR + 16);
    if (c.tid == 0) {
        tc::mbar_init(bar0, 1);
        tc::mbar_init(bar0 + 8, 1);
        *zero = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        tc::prefetch_map(&kmap);
        tc::prefetch_map(&vmap);
        int next = g0;
        while (next < g1 && !record_group(next))
            ++next;
        if (next < g1)
            issue_group(&kmap, &vmap, a, sm + SM_REC, bar0, next, kv);
    }

    // ---- query head g = warp: q and WHT(q) as F16-tile fragments, WHT(q) rows
    {
        const int g = c.warp;
        float v[8];
        if (g < c.G) {
            const float *src = a.q + ((int64_t)tok * a.n_head + kv * c.G + g) * 256 + 8 * c.lane;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                v[i] = src[i];
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                v[i] = 0.0f;
        }
        q_frags(v, c.fq, g, c.lane);
        wht_regs(v, c.lane);
        float4 *qd = reinterpret_cast<float4 *>(c.qr + g * QLD + 8 * c.lane);
        qd[0] = make_float4(v[0], v[1], v[2], v[3]);
        qd[1] = make_float4(v[4], v[5], v[6], v[7]);
        q_frags(v, c.fqr, g, c.lane);
        if (c.tid < GMAX) {
            c.st[c.tid] = -FLT_MAX;
            c.st[8 + c.tid] = 0.0f;
        }
    }
    __syncthreads();

    float acc_r[2][4] = {}, acc_t[2][4] = {};
    int buf = 0;
    uint32_t phase = 0;   // bit b: parity of buffer b's next completion
    bool failed = false;  // a record wait ran out (CTA-uniform)
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
                const bool ok = tc::mbar_wait(bar0 + 8 * buf, (phase >> buf) & 1, zero);
                // records landed; every thread is past the previous tile
                if (__syncthreads_or(!ok)) {
                    failed = true;
                    break;
                }
                phase ^= 1u << buf;
                if (c.tid == 0) {
                    int nxt = grp + 1;
                    while (nxt < g1 && !record_group(nxt))
                        ++nxt;
                    if (nxt < g1)
                        issue_group(&kmap, &vmap, a, sm + SM_REC + (buf ^ 1) * SET,
                                    bar0 + 8 * (buf ^ 1), nxt, kv);
                }
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
    if (failed && c.tid == 0) // give the copies still in flight a bounded time to land
        tc::mbar_wait(bar0 + 8 * buf, (phase >> buf) & 1, zero, 100000000ull);
    __syncthreads();

    // ---- numerator = WHT(rotated part) + tail part; partial record
    float *x = reinterpret_cast<float *>(sm + SM_REC), *xt = x + GMAX * QLD;
    {
        const int q0 = 2 * c.c;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
            const int d = 32 * c.warp + 16 * mt + 2 * c.g;
            *reinterpret_cast<float2 *>(x + q0 * QLD + d) = make_float2(acc_r[mt][0], acc_r[mt][2]);
            *reinterpret_cast<float2 *>(x + (q0 + 1) * QLD + d) =
                make_float2(acc_r[mt][1], acc_r[mt][3]);
            *reinterpret_cast<float2 *>(xt + q0 * QLD + d) = make_float2(acc_t[mt][0], acc_t[mt][2]);
            *reinterpret_cast<float2 *>(xt + (q0 + 1) * QLD + d) =
                make_float2(acc_t[mt][1], acc_t[mt][3]);
        }
    }
    __syncthreads();
    if (c.warp < c.G) {
        const int g = c.warp;
        float v[8], t[8];
        const float4 *xs = reinterpret_cast<const float4 *>(x + g * QLD + 8 * c.lane);
        const float4 *ts = reinterpret_cast<const float4 *>(xt + g * QLD + 8 * c.lane);
        const float4 v0 = xs[0], v1 = xs[1], t0 = ts[0], t1 = ts[1];
        v[0] = v0.x, v[1] = v0.y, v[2] = v0.z, v[3] = v0.w;
        v[4] = v1.x, v[5] = v1.y, v[6] = v1.z, v[7] = v1.w;
        t[0] = t0.x, t[1] = t0.y, t[2] = t0.z, t[3] = t0.w;
        t[4] = t1.x, t[5] = t1.y, t[6] = t1.z, t[7] = t1.w;
        wht_regs(v, c.lane);
        const int64_t n_rows = (int64_t)a.n_tokens * a.n_head;
        const int64_t row = (int64_t)tok * a.n_head + kv * c.G + g;
        float *rec = a.partials + ((int64_t)split * n_rows + row) * 258;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float2 *>(rec + 8 * c.lane + 2 * i) =
                make_float2(v[2 * i] + t[2 * i], v[2 * i + 1] + t[2 * i + 1]);
        if (c.lane == 0) {
            rec[256] = c.st[g];
            rec[257] = failed ? __int_as_float(0x7fc00000) : c.st[8 + g]; // NaN poisons the row
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
    // each plane's records as a 2D byte tensor of 64-byte rows; box = one
    // record's 128 nibble rows, 64-byte swizzle
    auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
    if (!enc)
        return cudaErrorNotSupported;
    CUtensorMap maps[2];
    for (int i = 0; i < 2; ++i) {
        cuuint64_t dims[2] = {64, (cuuint64_t)(l.records_bytes / 64)};
        cuuint64_t strides[1] = {64};
        cuuint32_t box[2] = {64, 128};
        cuuint32_t es[2] = {1, 1};
        if (enc(&maps[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(i ? l.v : l.k),
                dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    static std::atomic<unsigned long long> attr{0};
    cudaError_t e = set_smem_limit((const void *)kvarn4_partials_kernel, k4::SM_BYTES, attr);
    if (e != cudaSuccess)
        return e;
    dim3 grid((unsigned)l.n_splits, (unsigned)l.n_head_kv, (unsigned)l.n_tokens);
    kvarn4_partials_kernel<<<grid, k4::NT, k4::SM_BYTES, st>>>(maps[0], maps[1], a);
    return cudaGetLastError();
}

} // namespace xq
