// Native KVarN4 range attention (RKVA descriptor v1 resident image, head_dim
// 256): split partials over 4-bit Bee records, rotated F16 stage rows and the
// original-domain F16 precision tail, in the (acc[256], max, denom) partial
// layout the LSE merge reduces (xq_decode.cu).  Semantics as the reference's
// shaders/rkva/rkva_range_attn_kvarn4.hlsl:64-150: rows >= active - tail come
// from the tail and meet the original q; the other rows are in the rotated
// domain (WHT256 = Sylvester H256 / 16) and meet WHT(q); their value numerator
// is rotated back with WHT and added to the tail's.  Here the tail rows form a
// split of their own (original domain, no rotation) and every body split
// rotates its numerator back before it writes its partial, so the merge adds
// original-domain partials only.
//
// One CTA = (split, KV head, query token), the G = n_head / n_head_kv <= 8
// query heads of that KV head, 256 threads, two CTAs per SM.  Body splits
// cover whole 128-row groups.  A record group's four records (K and V, two
// 128-dim slices each) are double-buffered into shared memory by one thread:
// each record's 128 nibble rows of 64 bytes as one TMA box with the 64-byte
// swizzle (16-byte chunk c of row r lands at chunk c ^ ((r / 2) % 4), which
// makes the fragment loads below free of bank conflicts) and its 768 bytes of
// F16 axes as one bulk copy, all completing on the buffer's mbarrier.
//
// Warps w and w + 4 form pair p = w % 4 and own tokens 32p .. 32p + 31 of
// every 128-row tile; warp w covers dims slice w / 4 (128 dims).  Each warp
// computes its slice's partial scores of the pair's tokens, the pair adds them
// through shared memory (a 64-thread barrier), and each warp then runs its own
// online softmax over the pair's tokens and accumulates the value numerator of
// its slice; pairs are combined at the end of the split.  Per record group the
// CTA meets one CTA-wide barrier (records landed), one 128-thread barrier per
// slice (query-side fragments) and one pair barrier.
//
// Every product is a tensor-core mma.sync m16n8k16: A = the G query heads'
// fp32 operand split into an f16 high part (rows g) and remainder (rows g + 8),
// B = the KV side expanded exactly to f16 in registers (4-bit values: one byte
// permute, one mask and one f16 multiply-add give two n-tiles, the byte's low
// and high nibble):
//   scores  s_t = other_t * (sum_d (q_d scale_d) nib_dt + sum_d q_d zero_d)
//   values  n_d = other_d * (sum_t (w_t scale_t) nib_td + sum_t w_t zero_t)
// The n axis is permuted so that a lane's score columns are exactly the token
// k-slots of its value-product A fragment (tokens 2c, 2c + 1, 2c + 8, 2c + 9 of
// each 16), so the softmax weights never leave the lane.  Stage and tail rows
// (F16) are read straight from global memory into the same products.
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
constexpr int QLD = 264;     // padded row stride (floats) of [8][256] rows
// shared memory
constexpr int SM_REC = 0;                      // 2 x SET; x [4 pairs][8][QLD] after the loop
constexpr int SM_QR = SM_REC + 2 * SET;        // WHT(q) [8][QLD] (body splits)
constexpr int SM_KF = SM_QR + GMAX * QLD * 4;  // record-tile A fragments [2 slices][8][32] uint4
constexpr int SM_FQ = SM_KF + 2 * 8 * 32 * 16; // F16-tile A fragments [2][8][32] uint4
constexpr int SM_XS = SM_FQ + 2 * 8 * 32 * 16; // partial scores [2 parities][2][4 pairs][32][8]
constexpr int SM_ZP = SM_XS + 2 * 2 * 4 * 32 * 8 * 4; // q . zero_k partials [2][8][4]
constexpr int SM_MP = SM_ZP + 2 * 8 * 4 * 4;   // per-pair max and denominator [2][4][8]
constexpr int SM_BAR = SM_MP + 2 * 4 * 8 * 4;  // two mbarriers (one per record buffer), a zero word
constexpr int SM_BYTES = SM_BAR + 32 + 512;    // + alignment slack
} // namespace k4

struct Kvarn4Args {
    const uint8_t *k, *v; // planes
    const float *q;       // [n_tokens][n_head][256]
    const int32_t *positions;
    float *partials;      // [n_splits][n_tokens * n_head][258]
    int64_t records_bytes, stage_off, tail_off;
    int origin, active, tail, n_head, n_head_kv, n_tokens, rows_per_split, n_body;
    float scale;
};

namespace k4 {
// Per-CTA shared-memory views and lane indices, passed by value to the
// inlined phases (nothing of the kernel's state has its address taken).
struct Cta {
    float *qr, *xs, *zp;
    uint4 *kf, *fq;
    int tid, warp, lane, g, c, s, p, G; // g = lane / 4, c = lane % 4; s = slice, p = pair
    uint32_t sel; // byte permute: byte g / 2 of two words -> bytes 0 and 2
};
// Online-softmax state of one lane (query head g; replicated over c) and the
// value numerator of its slice: acc[u][i] = dim 16u + {2c, 2c+1, 2c+8, 2c+9}[i].
struct Run {
    float m, den;
    float acc[8][4];
};

// D += A B, m16n8k16, f16 inputs, f32 accumulate
__device__ __forceinline__ void mma16816(float (&d)[4], const uint4 &a, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}
// f32 pair -> f16x2 high part and f16x2 remainder: x = hi + lo to about 2^-22
// relative, so the two A rows g (hi) and g + 8 (lo) carry an fp32 operand
__device__ __forceinline__ void split2(float x, float y, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x, y);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}
// A fragment of k-slots (2c, 2c+1) = (x0, x1) and (2c+8, 2c+9) = (x8, x9)
__device__ __forceinline__ uint4 afrag(float x0, float x1, float x8, float x9) {
    uint4 f;
    split2(x0, x1, f.x, f.y);
    split2(x8, x9, f.z, f.w);
    return f;
}
// Byte g / 2 of words x (k-slot 2c) and y (k-slot 2c + 1): the low nibbles as
// the B register of n-tile parity 0, the high nibbles of parity 1.  0x6400 | n
// is the f16 1024 + n and 0x6400 | 16 n is 1024 + 16 n; both map back to n
// exactly.
__device__ __forceinline__ void nib_frag(uint32_t x, uint32_t y, uint32_t sel, uint32_t &lo,
                                         uint32_t &hi) {
    const uint32_t t = __byte_perm(x, y, sel);
    const uint32_t a = (t & 0x000f000fu) | 0x64006400u, b = (t & 0x00f000f0u) | 0x64006400u;
    const uint32_t k1024 = 0x64006400u, k16th = 0x2c002c00u, km64 = 0xd400d400u;
    const __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a),
                               *reinterpret_cast<const __half2 *>(&k1024));
    const __half2 hb = __hfma2(*reinterpret_cast<const __half2 *>(&b),
                               *reinterpret_cast<const __half2 *>(&k16th),
                               *reinterpret_cast<const __half2 *>(&km64));
    lo = *reinterpret_cast<const uint32_t *>(&ha);
    hi = *reinterpret_cast<const uint32_t *>(&hb);
}
__device__ __forceinline__ uint32_t lds32(const uint8_t *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}
__device__ __forceinline__ uint32_t ldg32(const uint8_t *p) {
    return __ldg(reinterpret_cast<const uint32_t *>(p));
}
// two F16 values at p (4-byte aligned) as floats
__device__ __forceinline__ float2 h2x2(const uint8_t *p) {
    return __half22float2(*reinterpret_cast<const __half2 *>(p));
}
__device__ __forceinline__ float sum4(const float *p) {
    const float4 v = *reinterpret_cast<const float4 *>(p);
    return (v.x + v.y) + (v.z + v.w);
}
// Named barriers with constant ids: 1 + s for the 128 threads of slice s,
// 3 + p for the 64 threads of pair p (0 is __syncthreads)
template <int ID, int COUNT>
__device__ __forceinline__ void bar_sync_c() {
    asm volatile("bar.sync %0, %1;\n" ::"n"(ID), "n"(COUNT) : "memory");
}
__device__ __forceinline__ void slice_sync(int s) {
    if (s == 0)
        bar_sync_c<1, 128>();
    else
        bar_sync_c<2, 128>();
}
__device__ __forceinline__ void pair_sync(int p) {
    switch (p) {
    case 0: bar_sync_c<3, 64>(); break;
    case 1: bar_sync_c<4, 64>(); break;
    case 2: bar_sync_c<5, 64>(); break;
    default: bar_sync_c<6, 64>(); break;
    }
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

// Sum the pair's partial scores (part: this warp's slice, part[u'][e] for
// tokens 32p + 16u' + {2c, 2c+1, 2c+8, 2c+9}[e] of the tile), scale, mask
// tokens outside [t0, t0 + n) and query heads >= G, and run the lane's
// online-softmax step.  Returns the weights in w and the accumulators'
// rescale factor.  The exchange buffer alternates with the tile parity, so a
// partner still reading the previous tile's scores is never overwritten.
__device__ __forceinline__ float pair_softmax(const Cta c, const float (&part)[2][4], int t0,
                                              int n, float scale, int parity, Run &r,
                                              float (&w)[2][4]) {
    float *own = c.xs + (((parity * 2 + c.s) * 4 + c.p) * 32 + c.lane) * 8;
    const float *oth = c.xs + (((parity * 2 + (c.s ^ 1)) * 4 + c.p) * 32 + c.lane) * 8;
    reinterpret_cast<float4 *>(own)[0] = make_float4(part[0][0], part[0][1], part[0][2], part[0][3]);
    reinterpret_cast<float4 *>(own)[1] = make_float4(part[1][0], part[1][1], part[1][2], part[1][3]);
    pair_sync(c.p);
    const float4 o0 = reinterpret_cast<const float4 *>(oth)[0];
    const float4 o1 = reinterpret_cast<const float4 *>(oth)[1];
    const float other[2][4] = {{o0.x, o0.y, o0.z, o0.w}, {o1.x, o1.y, o1.z, o1.w}};
    const bool on = c.g < c.G;
    float sc[2][4], mt = -INFINITY;
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int t = 32 * c.p + 16 * u + 2 * c.c + (e & 1) + 8 * (e >> 1);
            // slice 0 + slice 1 in the same order in both warps of the pair
            const float v = (c.s == 0 ? part[u][e] + other[u][e] : other[u][e] + part[u][e]) * scale;
            sc[u][e] = (on && t >= t0 && t < t0 + n) ? v : -INFINITY;
            mt = fmaxf(mt, sc[u][e]);
        }
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    const float m_new = fmaxf(r.m, mt);
    const float alpha = r.den == 0.0f ? 0.0f : __expf(r.m - m_new);
    float sum = 0.0f;
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            w[u][e] = __expf(sc[u][e] - m_new); // masked: exp(-inf) = 0
            sum += w[u][e];
        }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (on) {
        r.den = r.den * alpha + sum;
        r.m = m_new;
    }
    return alpha;
}

// Scores D of n-tiles (u', parity) -> part[u'][e] in token order {2c, 2c+1,
// 2c+8, 2c+9}: column 2c is token 2c + parity, column 2c + 1 is 2c + 8 + parity;
// rows g (hi) and g + 8 (lo) add up.
__device__ __forceinline__ void gather_scores(const float (&d)[2][2][4], float (&part)[2][4]) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        part[u][0] = d[u][0][0] + d[u][0][2];
        part[u][1] = d[u][1][0] + d[u][1][2];
        part[u][2] = d[u][0][1] + d[u][0][3];
        part[u][3] = d[u][1][1] + d[u][1][3];
    }
}

// n <= 128 consecutive F16 rows (row stride row_bytes; this KV head's 256
// values at krows / vrows): stage rows of a body split (rotated; A = WHT(q)
// fragments) or tail rows of the tail split (original; A = q fragments).
__device__ __forceinline__ void f16_tile(const Cta c, const uint8_t *krows, const uint8_t *vrows,
                                         int64_t row_bytes, int n, float scale, int parity, Run &r) {
    float part[2][4];
    {
        // B: lane g' = g takes token 2 (g / 2) + 8 (g % 2) + parity of unit
        // 2p + u', dims 16 kk + 2c (+ 8) of slice s
        float d[2][2][4] = {};
        const uint8_t *kb = krows + 2 * (128 * c.s + 2 * c.c);
        const int jb = 32 * c.p + 2 * (c.g >> 1) + 8 * (c.g & 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const uint4 a = c.fq[(c.s * 8 + kk) * 32 + c.lane];
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int par = 0; par < 2; ++par) {
                    const int j = jb + 16 * u + par;
                    const uint8_t *kr = kb + (int64_t)j * row_bytes + 32 * kk;
                    const uint32_t b0 = j < n ? ldg32(kr) : 0u, b1 = j < n ? ldg32(kr + 16) : 0u;
                    mma16816(d[u][par], a, b0, b1);
                }
        }
        gather_scores(d, part);
    }
    float w[2][4];
    const float alpha = pair_softmax(c, part, 0, n, scale, parity, r, w);
    {
        uint4 av[2];
#pragma unroll
        for (int u = 0; u < 2; ++u)
            av[u] = afrag(w[u][0], w[u][1], w[u][2], w[u][3]);
        // B: lane g takes dims 16 u + 8 (g % 2) + 2 (g / 2) + {0, 1} (the two
        // parities) of tokens 32p + 16u' + 2c + {0, 1, 8, 9}
        const uint8_t *vb = vrows + 2 * (128 * c.s + 8 * (c.g & 1) + 2 * (c.g >> 1));
        const int tb = 32 * c.p + 2 * c.c;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            float dv[2][4] = {};
#pragma unroll
            for (int uu = 0; uu < 2; ++uu) {
                uint32_t x[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = tb + 16 * uu + (e & 1) + 8 * (e >> 1);
                    x[e] = t < n ? ldg32(vb + (int64_t)t * row_bytes + 32 * u) : 0u;
                }
                mma16816(dv[0], av[uu], __byte_perm(x[0], x[1], 0x5410),
                         __byte_perm(x[2], x[3], 0x5410));
                mma16816(dv[1], av[uu], __byte_perm(x[0], x[1], 0x7632),
                         __byte_perm(x[2], x[3], 0x7632));
            }
            r.acc[u][0] = r.acc[u][0] * alpha + (dv[0][0] + dv[0][2]);
            r.acc[u][1] = r.acc[u][1] * alpha + (dv[1][0] + dv[1][2]);
            r.acc[u][2] = r.acc[u][2] * alpha + (dv[0][1] + dv[0][3]);
            r.acc[u][3] = r.acc[u][3] * alpha + (dv[1][1] + dv[1][3]);
        }
    }
}

// Rows [t0, t0 + n) of one complete record group whose four records are in
// shared memory at rk (nibble rows swizzled).
__device__ __forceinline__ void record_tile(const Cta c, const uint8_t *rk, int t0, int n,
                                            float scale, int parity, Run &r) {
    {
        // A fragments of slice s: qs[d] = WHT(q)_g[128 s + d] * scale_k[d] for
        // MMA steps p and p + 4, and this thread's part of WHT(q) . zero_k
        const uint8_t *kax = rk + ax_off(c.s);
        float z = 0.0f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int kk = c.p + 4 * h, dl = 16 * kk + 2 * c.c;
            const float *qrow = c.qr + c.g * QLD + 128 * c.s + dl;
            const float2 q01 = *reinterpret_cast<const float2 *>(qrow);
            const float2 q89 = *reinterpret_cast<const float2 *>(qrow + 8);
            const float2 s01 = h2x2(kax + 2 * dl), s89 = h2x2(kax + 2 * dl + 16);
            const float2 z01 = h2x2(kax + 256 + 2 * dl), z89 = h2x2(kax + 256 + 2 * dl + 16);
            c.kf[(c.s * 8 + kk) * 32 + c.lane] =
                afrag(q01.x * s01.x, q01.y * s01.y, q89.x * s89.x, q89.y * s89.y);
            z += (q01.x * z01.x + q01.y * z01.y) + (q89.x * z89.x + q89.y * z89.y);
        }
        z += __shfl_xor_sync(0xffffffffu, z, 1);
        z += __shfl_xor_sync(0xffffffffu, z, 2);
        if (c.c == 0)
            c.zp[(c.s * 8 + c.g) * 4 + c.p] = z;
        slice_sync(c.s);
    }
    float part[2][4];
    {
        // scores of tokens 32p + 16u' + ..., all 128 dims of slice s; the K
        // nibble rows are dims, lane g' reads byte g' / 2 of word 2 (2p + u') +
        // g' % 2 (tokens 2 (g' / 2) + 8 (g' % 2) + {0, 1} of the unit)
        float d[2][2][4] = {};
        const uint8_t *kb = rk + nib_off(c.s) + 128 * c.c + 16 * (c.p ^ c.c) + 4 * (c.g & 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const uint4 a = c.kf[(c.s * 8 + kk) * 32 + c.lane];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const uint8_t *pp = kb + kk * 1024 + 8 * u;
                uint32_t b0p0, b0p1, b1p0, b1p1;
                nib_frag(lds32(pp), lds32(pp + 64), c.sel, b0p0, b0p1);
                nib_frag(lds32(pp + 512), lds32(pp + 576), c.sel, b1p0, b1p1);
                mma16816(d[u][0], a, b0p0, b1p0);
                mma16816(d[u][1], a, b0p1, b1p1);
            }
        }
        gather_scores(d, part);
        const float qz = sum4(c.zp + (c.s * 8 + c.g) * 4);
        const uint8_t *oax = rk + ax_off(c.s) + 512;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int t = 32 * c.p + 16 * u + 2 * c.c;
            const float2 o01 = h2x2(oax + 2 * t), o89 = h2x2(oax + 2 * t + 16);
            part[u][0] = o01.x * (part[u][0] + qz);
            part[u][1] = o01.y * (part[u][1] + qz);
            part[u][2] = o89.x * (part[u][2] + qz);
            part[u][3] = o89.y * (part[u][3] + qz);
        }
    }
    float w[2][4];
    const float alpha = pair_softmax(c, part, t0, n, scale, parity, r, w);
    {
        // A = w * scale_v of slice s's V record, and sum_t w_t zero_v[t]
        const uint8_t *vax = rk + ax_off(2 + c.s);
        uint4 av[2];
        float wz = 0.0f;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int t = 32 * c.p + 16 * u + 2 * c.c;
            const float2 c01 = h2x2(vax + 2 * t), c89 = h2x2(vax + 2 * t + 16);
            const float2 z01 = h2x2(vax + 256 + 2 * t), z89 = h2x2(vax + 256 + 2 * t + 16);
            av[u] = afrag(w[u][0] * c01.x, w[u][1] * c01.y, w[u][2] * c89.x, w[u][3] * c89.y);
            wz += (w[u][0] * z01.x + w[u][1] * z01.y) + (w[u][2] * z89.x + w[u][3] * z89.y);
        }
        wz += __shfl_xor_sync(0xffffffffu, wz, 1);
        wz += __shfl_xor_sync(0xffffffffu, wz, 2);
        // value numerator: the V nibble rows are tokens 32p + 16u' + 2c + {0,
        // 1, 8, 9}; lane g reads byte g / 2 of word 2u + g % 2 (dims 16u + 8 (g
        // % 2) + 2 (g / 2) + {0, 1})
        const uint8_t *vb = rk + nib_off(2 + c.s) + 2048 * c.p + 128 * c.c + 4 * (c.g & 1);
        const uint8_t *oax = vax + 512 + 4 * c.c;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            float dv[2][4] = {};
            const int off = 16 * ((u >> 1) ^ c.c) + 8 * (u & 1);
#pragma unroll
            for (int uu = 0; uu < 2; ++uu) {
                const uint8_t *pp = vb + 1024 * uu + off;
                uint32_t b0p0, b0p1, b1p0, b1p1;
                nib_frag(lds32(pp), lds32(pp + 64), c.sel, b0p0, b0p1);
                nib_frag(lds32(pp + 512), lds32(pp + 576), c.sel, b1p0, b1p1);
                mma16816(dv[0], av[uu], b0p0, b1p0);
                mma16816(dv[1], av[uu], b0p1, b1p1);
            }
            const float2 o01 = h2x2(oax + 32 * u), o89 = h2x2(oax + 32 * u + 16);
            r.acc[u][0] = r.acc[u][0] * alpha + o01.x * ((dv[0][0] + dv[0][2]) + wz);
            r.acc[u][1] = r.acc[u][1] * alpha + o01.y * ((dv[1][0] + dv[1][2]) + wz);
            r.acc[u][2] = r.acc[u][2] * alpha + o89.x * ((dv[0][1] + dv[0][3]) + wz);
            r.acc[u][3] = r.acc[u][3] * alpha + o89.y * ((dv[1][1] + dv[1][3]) + wz);
        }
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
    c.qr = reinterpret_cast<float *>(sm + SM_QR);
    c.xs = reinterpret_cast<float *>(sm + SM_XS);
    c.zp = reinterpret_cast<float *>(sm + SM_ZP);
    c.kf = reinterpret_cast<uint4 *>(sm + SM_KF);
    c.fq = reinterpret_cast<uint4 *>(sm + SM_FQ);
    c.tid = threadIdx.x;
    c.warp = c.tid >> 5;
    c.lane = c.tid & 31;
    c.g = c.lane >> 2;
    c.c = c.lane & 3;
    c.s = c.warp >> 2;
    c.p = c.warp & 3;
    c.G = a.n_head / a.n_head_kv;
    {
        const uint32_t b = c.g >> 1;
        c.sel = b | (b << 4) | ((b + 4) << 8) | ((b + 4) << 12);
    }
    const int split = blockIdx.x, kv = blockIdx.y, tok = blockIdx.z;
    const int64_t row_bytes = (int64_t)a.n_head_kv * 512;

    const int pos = a.positions[tok];
    const int limit = pos < a.origin ? 0 : min(a.active, pos - a.origin + 1);
    const int tail_begin = a.active - min(a.active, a.tail);
    const bool tail_split = split >= a.n_body; // rows [tail_begin, active), original domain
    const int r0 = tail_split ? tail_begin : split * a.rows_per_split;
    const int r1 = tail_split ? limit : min(min(r0 + a.rows_per_split, tail_begin), limit);
    const int live = a.active ? (a.active - 1) / GROUP : 0;
    const bool live_partial = (a.active % GROUP) != 0;
    const int og = a.origin / GROUP;

    // a body group is read from its records unless it is the global sink group
    // or the incomplete live group (stage rows)
    const int g0 = r0 / GROUP, g1 = (!tail_split && r1 > r0) ? (r1 + GROUP - 1) / GROUP : g0;
    auto record_group = [=](int grp) { return og + grp != 0 && !(grp == live && live_partial); };
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

    // ---- query head g = warp: WHT(q) rows (body splits) and the F16-tile A
    // fragments of the split's domain; lane l holds dims 8l .. 8l + 7 = half
    // l % 2 of MMA step l / 2
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
        if (!tail_split) {
            wht_regs(v, c.lane);
            float4 *qd = reinterpret_cast<float4 *>(c.qr + g * QLD + 8 * c.lane);
            qd[0] = make_float4(v[0], v[1], v[2], v[3]);
            qd[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
        uint2 *fq2 = reinterpret_cast<uint2 *>(c.fq);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            uint2 hl;
            split2(v[2 * cc], v[2 * cc + 1], hl.x, hl.y);
            fq2[((c.lane >> 1) * 32 + 4 * g + cc) * 2 + (c.lane & 1)] = hl;
        }
    }
    __syncthreads();

    Run run;
    run.m = -FLT_MAX;
    run.den = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int i = 0; i < 4; ++i)
            run.acc[u][i] = 0.0f;
    int parity = 0;       // score-exchange buffer of the next tile
    bool failed = false;  // a record wait ran out (CTA-uniform)
    int buf = 0;
    uint32_t phase = 0;   // bit b: parity of buffer b's next completion
    if (tail_split) {
        // the tail buffer is a ring of 128 rows: row r at r % 128
        for (int rr = r0; rr < r1;) {
            const int n = min(r1 - rr, GROUP - rr % GROUP);
            const int64_t first = (int64_t)(rr % GROUP) * row_bytes + kv * 512;
            f16_tile(c, a.k + a.tail_off + first, a.v + a.tail_off + first, row_bytes, n, a.scale,
                     parity, run);
            parity ^= 1;
            rr += n;
        }
    } else {
        for (int grp = g0; grp < g1; ++grp) {
            const int lo = max(r0, grp * GROUP), hi = min(r1, (grp + 1) * GROUP);
            if (!record_group(grp)) {
                // staged group: rotated F16 rows in its stage slot
                const int slot = og + grp == 0 ? 0 : 1 + ((og + grp - 1) & 1);
                const int64_t first =
                    ((int64_t)slot * GROUP + (lo - grp * GROUP)) * row_bytes + kv * 512;
                f16_tile(c, a.k + a.stage_off + first, a.v + a.stage_off + first, row_bytes,
                         hi - lo, a.scale, parity, run);
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
                record_tile(c, sm + SM_REC + buf * SET, lo - grp * GROUP, hi - lo, a.scale,
                            parity, run);
                buf ^= 1;
            }
            parity ^= 1;
        }
    }
    if (failed && c.tid == 0) // give the copies still in flight a bounded time to land
        tc::mbar_wait(bar0 + 8 * buf, (phase >> buf) & 1, zero, 100000000ull);

    // ---- combine the four pairs: per query head the max over pairs, each
    // pair's numerator and denominator rescaled to it
    float *mp = reinterpret_cast<float *>(sm + SM_MP); // [0, 32) max, [32, 64) den per (p, q)
    if (c.s == 0 && c.c == 0)
        mp[c.p * 8 + c.g] = run.m;
    __syncthreads();
    float *x = reinterpret_cast<float *>(sm + SM_REC); // [4 pairs][8][QLD]
    {
        float mx = mp[c.g];
#pragma unroll
        for (int pp = 1; pp < 4; ++pp)
            mx = fmaxf(mx, mp[pp * 8 + c.g]);
        const float f = run.den == 0.0f ? 0.0f : __expf(run.m - mx);
        float *xr = x + (c.p * 8 + c.g) * QLD + 128 * c.s + 2 * c.c;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            *reinterpret_cast<float2 *>(xr + 16 * u) =
                make_float2(run.acc[u][0] * f, run.acc[u][1] * f);
            *reinterpret_cast<float2 *>(xr + 16 * u + 8) =
                make_float2(run.acc[u][2] * f, run.acc[u][3] * f);
        }
        if (c.s == 0 && c.c == 0)
            mp[32 + c.p * 8 + c.g] = run.den * f;
    }
    __syncthreads();
    if (c.warp < c.G) {
        const int g = c.warp;
        float v[8] = {};
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
            const float4 *xs = reinterpret_cast<const float4 *>(x + (pp * 8 + g) * QLD + 8 * c.lane);
            const float4 v0 = xs[0], v1 = xs[1];
            v[0] += v0.x, v[1] += v0.y, v[2] += v0.z, v[3] += v0.w;
            v[4] += v1.x, v[5] += v1.y, v[6] += v1.z, v[7] += v1.w;
        }
        if (!tail_split)
            wht_regs(v, c.lane); // back to the original domain
        const int64_t n_rows = (int64_t)a.n_tokens * a.n_head;
        const int64_t row = (int64_t)tok * a.n_head + kv * c.G + g;
        float *rec = a.partials + ((int64_t)split * n_rows + row) * 258;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float2 *>(rec + 8 * c.lane + 2 * i) =
                make_float2(v[2 * i], v[2 * i + 1]);
        if (c.lane == 0) {
            float mx = mp[g], den = 0.0f;
#pragma unroll
            for (int pp = 0; pp < 4; ++pp) {
                mx = fmaxf(mx, mp[pp * 8 + g]);
                den += mp[32 + pp * 8 + g];
            }
            rec[256] = mx;
            rec[257] = failed ? __int_as_float(0x7fc00000) : den; // NaN poisons the row
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
    a.n_body = l.n_body;
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
