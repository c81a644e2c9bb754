// Native KVarN4 range attention (RKVA descriptor v1 resident image, head_dim
// 256) on the tcgen05 tensor cores: split partials over 4-bit Bee records,
// rotated F16 stage rows and the original-domain F16 precision tail, in the
// (acc[256], max, denom) partial layout the LSE merge reduces (xq_decode.cu).
// Semantics as the reference's shaders/rkva/rkva_range_attn_kvarn4.hlsl:64-150:
// rows >= active - tail come from the tail and meet the original q; the other
// rows are in the rotated domain (WHT256 = Sylvester H256 / 16) and meet
// WHT(q); their value numerator is rotated back with WHT and added to the
// tail's.  Here the tail rows form a split of their own (original domain) and
// every body split rotates its numerator back before it writes its partial,
// so the merge adds original-domain partials only.
//
// One CTA = (split, KV head, query token), the G = n_head / n_head_kv <= 8
// query heads of that KV head, 256 threads, two CTAs per SM, 64 TMEM columns.
// Per 128-row record group (four records: K and V, two 128-dim slices each):
//
//   1. the K records' 4-bit values are widened to bytes in shared memory as
//      the MN-major UMMA A operand (one 128-byte row per dim: the low nibbles
//      of the row's 64 bytes, then the high nibbles, i.e. tokens 0, 2, .., 126,
//      1, 3, .., 127; 128-byte swizzle); the query side q_d scale_d of each
//      slice is written as the K-major B operand in three balanced int8 limbs
//      (x = 2^-E (l0 + 2^8 l1 + 2^16 l2), one power-of-two exponent per query
//      head and slice, |x 2^E| < 2^22);
//   2. scores: eight tcgen05.mma kind::i8 (M = 128 tokens, N = 32 = 8 heads x 3
//      limbs + 8 unused, K = 32) accumulate exact int32 sums in TMEM;
//      s_t = scale * sum_slices other_t (2^-E (D0 + 2^8 D1 + 2^16 D2) +
//      sum_d q_d zero_d);
//   3. the V records are widened the same way (rows = tokens, bytes = dims);
//   4. one warp per query head runs the online-softmax step over the 128
//      tokens and writes w_t scale_v[t] as three int8 limbs (the V B operand),
//      with sum_t w_t zero_v[t];
//   5. values: eight more kind::i8 MMAs (M = 128 dims, N = 32, K = 32); each
//      thread owns one dim of one slice for all eight heads:
//      acc = acc * alpha + other_d (2^-E (D0 + 2^8 D1 + 2^16 D2) +
//      sum_t w_t zero_v[t]).
//
// The int8 products are exact; the only rounding on the tensor-core side is
// the 22-bit limb quantisation of the fp32 query / weight operands (relative
// 2^-22 of each head's largest value) and fp32 when the limbs are combined.
// F16 stage / tail rows run the same five steps with kind::f16 MMAs: F16 K rows
// (K-major) and V rows (MN-major, even dims then odd dims so that a thread
// owns the same dim in both kinds of tile) staged into shared memory, and the
// query / weights as an f16 high part plus remainder (N = 16 = 8 heads x 2).
// TMEM: scores of slice s at column 32 s, values at 64 + 32 s.
// A record group's raw bytes arrive one group ahead by bulk copies: the 4-bit
// rows into the upper halves of the operand slots they are widened into (read
// into registers before a barrier, so the widening can overwrite them), the
// F16 scales / zeros / factors into a 3 KB area; K is requested once the
// previous group's score MMAs are done, V once its value MMAs are done.
// Every mbarrier wait is bounded; on timeout the CTA poisons its partial (NaN
// denominator), waits a bounded time for its MMAs and copies, frees TMEM and
// returns.
#include <cuda.h>
#include <cuda_fp16.h>
#include <float.h>
#include <math.h>

#include "xq_common.cuh"
#include "xq_internal.h"
#include "xq_tc.cuh"

namespace xq {

namespace k4 {
constexpr int NT = 256;
constexpr int GMAX = 8;    // query heads per KV head
constexpr int REC = 8960;  // bytes per record: 8192 of nibbles (128 rows x 64 B), then
constexpr int NIB = 8192;  // 128 F16 scales, 128 zeros (per row), 128 factors (per column)
constexpr int GROUP = 128; // rows per record group
constexpr int QLD = 264;   // padded fp32 row stride of [8][256] rows
constexpr int PLD = 132;   // padded row stride of the partial scores [2][8][128]
// shared memory (1024-byte aligned base; every operand tile 1024-aligned)
constexpr int SM_A0 = 0;     // 32 KB: K operand (records: slice s at 16 KB s; F16: K or V slice 0)
constexpr int SM_A1 = 32768; // 32 KB: V operand (records: slice s at 16 KB s; F16: K or V slice 1)
constexpr int SM_BQ = 65536; // 8 KB: query operand (slice s at 4 KB s: int8 32 rows, f16 16 x 2)
constexpr int SM_BW = 73728; // 8 KB: weight operand (same)
constexpr int SM_QV = 81920; // q (tail split) or WHT(q) (body splits) [8][QLD] fp32
constexpr int SM_PS = SM_QV + GMAX * QLD * 4;   // partial scores [2 slices][8][PLD]
constexpr int SM_VEC = SM_PS + 2 * 8 * PLD * 4; // per-head vectors [16][8]
constexpr int SM_AX = SM_VEC + 16 * 8 * 4;      // F16 axes: K slice 0, 1, V slice 0, 1 (768 B each)
constexpr int SM_BAR = SM_AX + 4 * 768;         // bar_S, bar_V, bar_RK, bar_RV, TMEM slot, zero word
constexpr int SM_BYTES = SM_BAR + 64 + 1024;    // + alignment slack
// rows of the per-head vectors
constexpr int V_M = 0, V_DEN = 1, V_ALPHA = 2, V_EQ = 3, V_QZ = 5, V_EW = 7, V_WZ = 9;
constexpr uint32_t TMEM_COLS = 128; // scores slice 0 / 1 at 0 / 32, values at 64 / 96

// tcgen05.mma kind::i8, A s8 MN-major (the 4-bit values 0..15), B s8 K-major,
// s32 accumulator
constexpr uint32_t ID_I8 = (2u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (0u << 16) |
                           ((32u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t ID_F16_S = tc::idesc(128, 16, 0, 0); // K rows K-major
constexpr uint32_t ID_F16_V = tc::idesc(128, 16, 1, 0); // V rows MN-major
} // namespace k4

struct Kvarn4Args {
    const uint8_t *k, *v; // planes
    const float *q;       // [n_tokens][n_head][256]
    const int32_t *positions;
    float *partials;      // [n_splits][n_tokens * n_head][258]
    int64_t stage_off, tail_off;
    int origin, active, tail, n_head, n_head_kv, n_tokens, rows_per_split, n_body;
    float scale;
};

namespace k4 {
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
    asm volatile(
        "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(ID_I8), "r"(acc));
}
__device__ __forceinline__ uint4 ldg128(const uint8_t *p) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
}
__device__ __forceinline__ float h2f(const uint8_t *p) {
    return __half2float(*reinterpret_cast<const __half *>(p));
}
__device__ __forceinline__ void h8(const uint8_t *p, float (&x)[8]) { // 8 F16 at p (16 B)
    const uint4 u = *reinterpret_cast<const uint4 *>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void h4(const uint8_t *p, float (&x)[4]) { // 4 F16 at p (8 B)
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    x[0] = a.x, x[1] = a.y, x[2] = b.x, x[3] = b.y;
}
// Byte offset of 16-byte chunk c of row r in a tile of 128-byte rows with the
// 128-byte swizzle
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
    return r * 128u + ((c ^ (r & 7u)) << 4);
}
// Widen one 16-byte chunk (32 nibbles, low nibble first) of row r, chunk c4 of
// the row's four: low nibbles to chunk c4, high nibbles to chunk 4 + c4.
__device__ __forceinline__ void widen(uint8_t *tile, int r, int c4, uint4 w) {
    const uint32_t m = 0x0f0f0f0fu;
    *reinterpret_cast<uint4 *>(tile + swz(r, c4)) = make_uint4(w.x & m, w.y & m, w.z & m, w.w & m);
    *reinterpret_cast<uint4 *>(tile + swz(r, 4 + c4)) =
        make_uint4((w.x >> 4) & m, (w.y >> 4) & m, (w.z >> 4) & m, (w.w >> 4) & m);
}
// Position p of a widened row -> token / dim index (low nibbles are the even
// ones)
__device__ __forceinline__ int unperm(int p) { return p < 64 ? 2 * p : 2 * (p - 64) + 1; }
// Three balanced int8 limbs of v = rint(x * 2^E), |v| < 2^22:
// v = l0 + 2^8 l1 + 2^16 l2 with l0, l1 in [-128, 127], |l2| <= 64
__device__ __forceinline__ void limbs(float x, float mul, int &l0, int &l1, int &l2) {
    const int v = __float2int_rn(x * mul);
    l0 = ((v + 128) & 255) - 128;
    const int v1 = (v - l0) >> 8;
    l1 = ((v1 + 128) & 255) - 128;
    l2 = (v1 - l1) >> 8;
}
// 2^E with E = 21 - ilogb(mx): the largest |x| maps below 2^22; 1 when mx = 0
__device__ __forceinline__ float limb_scale(float mx) {
    return mx > 0.0f ? ldexpf(1.0f, 21 - ilogbf(mx)) : 1.0f;
}
// D0 + 2^8 D1 + 2^16 D2 of the int32 sums held as float bit patterns
__device__ __forceinline__ float combine(float d0, float d1, float d2) {
    return fmaf((float)__float_as_int(d2), 65536.0f,
                fmaf((float)__float_as_int(d1), 256.0f, (float)__float_as_int(d0)));
}
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
    return (uint32_t)(a & 255) | ((uint32_t)(b & 255) << 8) | ((uint32_t)(c & 255) << 16) |
           ((uint32_t)(d & 255) << 24);
}
__device__ __forceinline__ uint32_t f16x2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// f32 x -> f16 high part, remainder
__device__ __forceinline__ void hilo(float x, float &hi, float &lo) {
    hi = __half2float(__float2half_rn(x));
    lo = x - hi;
}

struct Cta {
    uint8_t *sm;
    float *qv, *ps, *vec;
    uint32_t tmem, bar_s, bar_v, bar_rk, bar_rv;
    volatile int *zero;
    int tid, warp, lane, G;
};

// ---- step 4: the online-softmax step of the tile (warp q = query head q;
// lane l holds tokens 4l .. 4l + 3) over scores = scale * (slice 0 + slice 1
// partials), masked to [t0, t0 + n).  Writes the weight operand: int8 limbs
// of w * scale_v (records) or f16 high / remainder of w (F16 rows).
template <bool REC_TILE>
__device__ __forceinline__ void softmax_step(const Cta c, int t0, int n, float scale) {
    const int q = c.warp, t = 4 * c.lane;
    float *vec = c.vec;
    if (q >= c.G) {
        if (c.lane == 0) {
            vec[V_ALPHA * 8 + q] = 0.0f;
            vec[V_EW * 8 + q] = vec[(V_EW + 1) * 8 + q] = 0.0f;
            vec[V_WZ * 8 + q] = vec[(V_WZ + 1) * 8 + q] = 0.0f;
        }
        return;
    }
    const float4 p0 = *reinterpret_cast<const float4 *>(c.ps + q * PLD + t);
    const float4 p1 = *reinterpret_cast<const float4 *>(c.ps + (8 + q) * PLD + t);
    const float sp[4] = {p0.x + p1.x, p0.y + p1.y, p0.z + p1.z, p0.w + p1.w};
    float sc[4], mt = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sc[i] = (t + i >= t0 && t + i < t0 + n) ? sp[i] * scale : -INFINITY;
        mt = fmaxf(mt, sc[i]);
    }
    mt = warp_max(mt);
    const float m_old = vec[V_M * 8 + q], den_old = vec[V_DEN * 8 + q];
    const float m_new = fmaxf(m_old, mt);
    const float alpha = den_old == 0.0f ? 0.0f : __expf(m_old - m_new);
    float w[4], sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w[i] = __expf(sc[i] - m_new);
        sum += w[i];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        uint8_t *bw = c.sm + SM_BW + s * 4096;
        if (REC_TILE) {
            const uint8_t *vax = c.sm + SM_AX + (2 + s) * 768;
            float sv[4], zv[4], ws[4], mx = 0.0f, wz = 0.0f;
            h4(vax + 2 * t, sv);
            h4(vax + 256 + 2 * t, zv);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                ws[i] = w[i] * sv[i];
                mx = fmaxf(mx, fabsf(ws[i]));
                wz = fmaf(w[i], zv[i], wz);
            }
            mx = warp_max(mx);
            wz = warp_sum(wz);
            const float mul = limb_scale(mx);
            int l[3][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                limbs(ws[i], mul, l[0][i], l[1][i], l[2][i]);
            // K-major B: row 8 j + q = limb j; k = token
#pragma unroll
            for (int j = 0; j < 3; ++j)
                *reinterpret_cast<uint32_t *>(bw + swz(8 * j + q, t >> 4) + (t & 15)) =
                    pack4(l[j][0], l[j][1], l[j][2], l[j][3]);
            if (c.lane == 0) {
                vec[(V_EW + s) * 8 + q] = 1.0f / mul;
                vec[(V_WZ + s) * 8 + q] = wz;
            }
        } else if (s == 0) {
            // F16 rows: both slices' products use the same weights; rows q (f16
            // high part) and 8 + q (remainder), two 64-token atom columns
            float h[4], l[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                hilo(w[i], h[i], l[i]);
#pragma unroll
            for (int ss = 0; ss < 2; ++ss) {
                uint8_t *b = c.sm + SM_BW + ss * 4096 + (t >> 6) * 2048;
                const int tc = t & 63;
                *reinterpret_cast<uint2 *>(b + swz(q, tc >> 3) + 2 * (tc & 7)) =
                    make_uint2(f16x2(h[0], h[1]), f16x2(h[2], h[3]));
                *reinterpret_cast<uint2 *>(b + swz(8 + q, tc >> 3) + 2 * (tc & 7)) =
                    make_uint2(f16x2(l[0], l[1]), f16x2(l[2], l[3]));
            }
            if (c.lane == 0) {
                vec[V_EW * 8 + q] = vec[(V_EW + 1) * 8 + q] = 1.0f;
                vec[V_WZ * 8 + q] = vec[(V_WZ + 1) * 8 + q] = 0.0f;
            }
        }
    }
    if (c.lane == 0) {
        vec[V_M * 8 + q] = m_new;
        vec[V_DEN * 8 + q] = den_old * alpha + sum;
        vec[V_ALPHA * 8 + q] = alpha;
    }
}

// ---- step 5 epilogue: this thread's value-numerator dim (slice s = warp / 4,
// TMEM lane L = 32 (warp % 4) + lane, dim position unperm(L)) for all heads
template <bool REC_TILE>
__device__ __forceinline__ void value_epilogue(const Cta c, float (&acc)[8]) {
    const int s = c.warp >> 2, L = 32 * (c.warp & 3) + c.lane;
    const uint32_t ta = c.tmem + ((uint32_t)(32 * (c.warp & 3)) << 16) + 64 + 32 * s;
    if (REC_TILE) {
        float d[32];
        tc::tmem_ld32(ta, d);
        const float o = h2f(c.sm + SM_AX + (2 + s) * 768 + 512 + 2 * unperm(L));
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float val = fmaf(combine(d[q], d[8 + q], d[16 + q]), c.vec[(V_EW + s) * 8 + q],
                                   c.vec[(V_WZ + s) * 8 + q]);
            acc[q] = fmaf(o, val, acc[q] * c.vec[V_ALPHA * 8 + q]);
        }
    } else {
        float d[16];
        tc::tmem_ld16(ta, d);
#pragma unroll
        for (int q = 0; q < 8; ++q)
            acc[q] = fmaf(acc[q], c.vec[V_ALPHA * 8 + q], d[q] + d[8 + q]);
    }
}

// ---- step 2 epilogue: this thread's token (slice s, TMEM lane L, token
// position pos(L)) partial scores for all heads into ps[s][q][token]
template <bool REC_TILE>
__device__ __forceinline__ void score_epilogue(const Cta c) {
    const int s = c.warp >> 2, L = 32 * (c.warp & 3) + c.lane;
    const uint32_t ta = c.tmem + ((uint32_t)(32 * (c.warp & 3)) << 16) + 32 * s;
    const int tok = REC_TILE ? unperm(L) : L;
    float *ps = c.ps + s * 8 * PLD + tok;
    if (REC_TILE) {
        float d[32];
        tc::tmem_ld32(ta, d);
        const float o = h2f(c.sm + SM_AX + s * 768 + 512 + 2 * tok);
#pragma unroll
        for (int q = 0; q < 8; ++q)
            ps[q * PLD] = o * fmaf(combine(d[q], d[8 + q], d[16 + q]), c.vec[(V_EQ + s) * 8 + q],
                                   c.vec[(V_QZ + s) * 8 + q]);
    } else {
        float d[16];
        tc::tmem_ld16(ta, d);
#pragma unroll
        for (int q = 0; q < 8; ++q)
            ps[q * PLD] = d[q] + d[8 + q];
    }
}

// Bounded wait on an MMA barrier by every thread; false on timeout.
__device__ __forceinline__ bool wait_mma(const Cta c, uint32_t bar, uint32_t &phase) {
    const bool ok = tc::mbar_wait(bar, phase, c.zero);
    phase ^= 1u;
    tc::tc_fence_after();
    return ok;
}

// Raw 4-bit rows of the K (A0) or V (A1) records of a group, waited for and
// read into registers: thread chunks i = tid + 256 j -> slice i / 512, row
// (i / 4) % 128, 16-byte chunk i % 4, at the upper half of the slice's slot.
__device__ __forceinline__ bool fetch_raw(const Cta c, int region, uint32_t bar, uint32_t &phase,
                                          uint4 (&w)[4]) {
    const bool ok = tc::mbar_wait(bar, phase, c.zero);
    phase ^= 1u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = c.tid + NT * j, s = i >> 9, r = (i >> 2) & 127, c4 = i & 3;
        w[j] = *reinterpret_cast<const uint4 *>(c.sm + region + s * 16384 + 8192 + r * 64 + c4 * 16);
    }
    return ok;
}
// One thread: bulk copies of group grp's K (or V) records of KV head kv: the
// 4-bit rows to the upper halves of the slots, the axes to the axes area.
__device__ __forceinline__ void issue_raw(const Cta c, const Kvarn4Args &a, bool value, int grp,
                                          int kv) {
    const uint8_t *plane = value ? a.v : a.k;
    const uint32_t bar = value ? c.bar_rv : c.bar_rk;
    const int64_t r = ((int64_t)grp * a.n_head_kv + kv) * 2 * REC;
    tc::fence_async_smem(); // earlier generic reads of these bytes come first
    tc::mbar_expect_tx(bar, 2 * REC);
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        tc::bulk_load(smem_u32(c.sm + (value ? SM_A1 : SM_A0) + s * 16384 + 8192),
                      plane + r + s * REC, NIB, bar);
        tc::bulk_load(smem_u32(c.sm + SM_AX + ((value ? 2 : 0) + s) * 768), plane + r + s * REC + NIB,
                      768, bar);
    }
}

// Per-CTA pipeline state: MMA and copy barrier phases, copies in flight
struct Pipe {
    uint32_t ph_s, ph_v, ph_rk, ph_rv;
    bool rk_pend, rv_pend;
};

// One record group, rows [t0, t0 + n) of it; its raw K rows are in kw, its V
// rows and all axes landed (or land) in shared memory.  When next >= 0 the
// next record group's K is requested once the score MMAs are done and read
// into kw at the end, and its V requested after the final barrier.  Returns
// false if a wait ran out (CTA-uniform).
__device__ __forceinline__ bool record_tile(const Cta c, const Kvarn4Args &a, uint4 (&kw)[4],
                                            int t0, int n, int next, int kv, Pipe &pp,
                                            float (&acc)[8]) {
    // 1. K widened into A0 (slice s at 16 KB s); the query operand
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = c.tid + NT * j, s = i >> 9, r = (i >> 2) & 127, c4 = i & 3;
        widen(c.sm + SM_A0 + s * 16384, r, c4, kw[j]);
    }
    {
        // thread (slice s, head q, dims 8 ch .. 8 ch + 7); the 16 threads of a
        // (s, q) are one half-warp
        const int s = c.tid >> 7, q = (c.tid >> 4) & 7, ch = c.tid & 15;
        const uint8_t *kax = c.sm + SM_AX + s * 768;
        float sk[8], zk[8];
        h8(kax + 16 * ch, sk);
        h8(kax + 256 + 16 * ch, zk);
        const float *qr = c.qv + q * QLD + 128 * s + 8 * ch;
        const float4 qa = *reinterpret_cast<const float4 *>(qr);
        const float4 qb = *reinterpret_cast<const float4 *>(qr + 4);
        const float qx[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        float qs[8], mx = 0.0f, z = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qs[i] = qx[i] * sk[i];
            mx = fmaxf(mx, fabsf(qs[i]));
            z = fmaf(qx[i], zk[i], z);
        }
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            z += __shfl_xor_sync(0xffffffffu, z, o);
        }
        const float mul = limb_scale(mx);
        int l[3][8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            limbs(qs[i], mul, l[0][i], l[1][i], l[2][i]);
        uint8_t *bq = c.sm + SM_BQ + s * 4096;
        const uint32_t off = 8 * (ch & 1);
#pragma unroll
        for (int j = 0; j < 3; ++j)
            *reinterpret_cast<uint2 *>(bq + swz(8 * j + q, ch >> 1) + off) =
                make_uint2(pack4(l[j][0], l[j][1], l[j][2], l[j][3]),
                           pack4(l[j][4], l[j][5], l[j][6], l[j][7]));
        if (ch == 0) {
            c.vec[(V_EQ + s) * 8 + q] = 1.0f / mul;
            c.vec[(V_QZ + s) * 8 + q] = z;
        }
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    // 2. scores: D[token][limb x head] per slice, K = 128 dims in 4 steps
    if (c.tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t ad = tc::sdesc(smem_u32(c.sm + SM_A0 + s * 16384 + kk * 4096),
                                              16384, 1024);
                const uint64_t bd =
                    tc::sdesc(smem_u32(c.sm + SM_BQ + s * 4096) + kk * 32, 16, 1024);
                mma_i8(c.tmem + 32 * s, ad, bd, kk > 0);
            }
        tc::mma_commit(c.bar_s);
    }
    // 3. the V rows into registers (widened after the next barrier)
    uint4 vw[4];
    bool ok = fetch_raw(c, SM_A1, c.bar_rv, pp.ph_rv, vw);
    pp.rv_pend = false;
    ok &= wait_mma(c, c.bar_s, pp.ph_s);
    score_epilogue<true>(c);
    tc::tc_fence_before();
    if (__syncthreads_or(!ok))
        return false;
    if (next >= 0) {
        // A0 and the K axes are free: the score MMAs are done, the epilogue read
        if (c.tid == 0)
            issue_raw(c, a, false, next, kv);
        pp.rk_pend = true;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int i = c.tid + NT * j, s = i >> 9, r = (i >> 2) & 127, c4 = i & 3;
        widen(c.sm + SM_A1 + s * 16384, r, c4, vw[j]);
    }
    // 4. softmax step, weight operand
    softmax_step<true>(c, t0, n, a.scale);
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    // 5. values: D[dim][limb x head] per slice, K = 128 tokens in 4 steps
    if (c.tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint64_t ad = tc::sdesc(smem_u32(c.sm + SM_A1 + s * 16384 + kk * 4096),
                                              16384, 1024);
                const uint64_t bd =
                    tc::sdesc(smem_u32(c.sm + SM_BW + s * 4096) + kk * 32, 16, 1024);
                mma_i8(c.tmem + 64 + 32 * s, ad, bd, kk > 0);
            }
        tc::mma_commit(c.bar_v);
    }
    ok = wait_mma(c, c.bar_v, pp.ph_v);
    value_epilogue<true>(c, acc);
    if (next >= 0) {
        ok &= fetch_raw(c, SM_A0, c.bar_rk, pp.ph_rk, kw);
        pp.rk_pend = false;
    }
    tc::tc_fence_before();
    if (__syncthreads_or(!ok))
        return false;
    if (next >= 0) {
        // A1 and the V axes are free: the value MMAs are done, the epilogue read
        if (c.tid == 0)
            issue_raw(c, a, true, next, kv);
        pp.rv_pend = true;
    }
    return true;
}

// Stage n <= 128 F16 rows (row stride row_bytes, this head's 256 values at
// rows) into A0 (slice 0) and A1 (slice 1): K rows as K-major tiles (two
// 64-dim atom columns of 128 rows), V rows MN-major with the even dims of each
// 8 in the first 64-dim block and the odd dims in the second (the order of the
// widened records).  Rows >= n are zero.
template <bool VALUE>
__device__ __forceinline__ void stage_f16(const Cta c, const uint8_t *rows, int64_t row_bytes,
                                          int n) {
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
        const int i = c.tid + NT * j, s = i >> 11, r = (i >> 4) & 127, ch = i & 15;
        const uint4 w = r < n ? ldg128(rows + r * row_bytes + 256 * s + 16 * ch)
                              : make_uint4(0u, 0u, 0u, 0u);
        uint8_t *tile = c.sm + (s ? SM_A1 : SM_A0);
        if (!VALUE) {
            *reinterpret_cast<uint4 *>(tile + (ch >> 3) * 16384 + swz(r, ch & 7)) = w;
        } else {
            // dims 8 ch .. 8 ch + 7: even ones -> positions 4 ch .. (block 0),
            // odd ones -> 64 + 4 ch .. (block 1)
            const uint2 ev = make_uint2(__byte_perm(w.x, w.y, 0x5410), __byte_perm(w.z, w.w, 0x5410));
            const uint2 od = make_uint2(__byte_perm(w.x, w.y, 0x7632), __byte_perm(w.z, w.w, 0x7632));
            const uint32_t off = swz(r, ch >> 1) + 8 * (ch & 1);
            *reinterpret_cast<uint2 *>(tile + off) = ev;
            *reinterpret_cast<uint2 *>(tile + 16384 + off) = od;
        }
    }
}

// n <= 128 F16 rows: stage rows of a body split (rotated, meet WHT(q)) or
// tail rows of the tail split (original, meet q); qv holds the right one.
__device__ __forceinline__ bool f16_tile(const Cta c, const uint8_t *krows, const uint8_t *vrows,
                                         int64_t row_bytes, int n, float scale, Pipe &pp,
                                         float (&acc)[8]) {
    stage_f16<false>(c, krows, row_bytes, n);
    {
        // query operand: rows q (f16 of qv) and 8 + q (remainder); thread
        // (slice s, head q, dims 8 ch .. 8 ch + 7)
        const int s = c.tid >> 7, q = (c.tid >> 4) & 7, ch = c.tid & 15;
        const float *qr = c.qv + q * QLD + 128 * s + 8 * ch;
        float h[8], l[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            hilo(qr[i], h[i], l[i]);
        uint8_t *b = c.sm + SM_BQ + s * 4096 + (ch >> 3) * 2048;
        *reinterpret_cast<uint4 *>(b + swz(q, ch & 7)) =
            make_uint4(f16x2(h[0], h[1]), f16x2(h[2], h[3]), f16x2(h[4], h[5]), f16x2(h[6], h[7]));
        *reinterpret_cast<uint4 *>(b + swz(8 + q, ch & 7)) =
            make_uint4(f16x2(l[0], l[1]), f16x2(l[2], l[3]), f16x2(l[4], l[5]), f16x2(l[6], l[7]));
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    if (c.tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t a = smem_u32(c.sm + (s ? SM_A1 : SM_A0)) + (kk >> 2) * 16384 +
                                   (kk & 3) * 32;
                const uint32_t b =
                    smem_u32(c.sm + SM_BQ + s * 4096) + (kk >> 2) * 2048 + (kk & 3) * 32;
                tc::mma_ss(c.tmem + 32 * s, tc::sdesc(a, 16, 1024), tc::sdesc(b, 16, 1024),
                           ID_F16_S, kk > 0);
            }
        tc::mma_commit(c.bar_s);
    }
    bool ok = wait_mma(c, c.bar_s, pp.ph_s);
    score_epilogue<false>(c);
    tc::tc_fence_before();
    if (__syncthreads_or(!ok))
        return false;
    stage_f16<true>(c, vrows, row_bytes, n); // A0 / A1 free: the score MMAs are done
    softmax_step<false>(c, 0, n, scale);
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    if (c.tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const uint32_t a = smem_u32(c.sm + (s ? SM_A1 : SM_A0)) + kk * 2048;
                const uint32_t b =
                    smem_u32(c.sm + SM_BW + s * 4096) + (kk >> 2) * 2048 + (kk & 3) * 32;
                tc::mma_ss(c.tmem + 64 + 32 * s, tc::sdesc(a, 16384, 1024),
                           tc::sdesc(b, 16, 1024), ID_F16_V, kk > 0);
            }
        tc::mma_commit(c.bar_v);
    }
    ok = wait_mma(c, c.bar_v, pp.ph_v);
    value_epilogue<false>(c, acc);
    tc::tc_fence_before();
    return __syncthreads_or(!ok) == 0;
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

} // namespace k4

__global__ void __launch_bounds__(k4::NT, 2) kvarn4_partials_kernel(const Kvarn4Args a) {
    using namespace k4;
    extern __shared__ __align__(1024) uint8_t sm_raw[];
    // aligned by an offset on the shared array itself, so that every access
    // through sm stays a shared-memory access (a round trip through an integer
    // would leave the compiler only generic addresses)
    uint8_t *sm = sm_raw + ((1024u - (smem_u32(sm_raw) & 1023u)) & 1023u);
    Cta c;
    c.sm = sm;
    c.qv = reinterpret_cast<float *>(sm + SM_QV);
    c.ps = reinterpret_cast<float *>(sm + SM_PS);
    c.vec = reinterpret_cast<float *>(sm + SM_VEC);
    c.bar_s = smem_u32(sm + SM_BAR);
    c.bar_v = c.bar_s + 8;
    c.bar_rk = c.bar_s + 16;
    c.bar_rv = c.bar_s + 24;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + SM_BAR + 32);
    c.zero = reinterpret_cast<volatile int *>(sm + SM_BAR + 36);
    c.tid = threadIdx.x;
    c.warp = c.tid >> 5;
    c.lane = c.tid & 31;
    c.G = a.n_head / a.n_head_kv;
    const int split = blockIdx.x, kv = blockIdx.y, tok = blockIdx.z;
    const int64_t row_bytes = (int64_t)a.n_head_kv * 512;
    const int live = a.active ? (a.active - 1) / GROUP : 0;
    const bool live_partial = (a.active % GROUP) != 0;
    const int og = a.origin / GROUP;
    // a body group is read from its records unless it is the global sink group
    // or the incomplete live group (stage rows)
    auto record_group = [=](int grp) { return og + grp != 0 && !(grp == live && live_partial); };

    // Launched as a programmatic dependent: until griddepcontrol.wait the
    // kernel before this one may still be writing q, the positions or the
    // planes, and reading the partials this kernel writes, so only set-up and
    // an L2 prefetch of the split's first group (no data consumed) come first.
    // The merge after this kernel may launch at once; it waits for this grid.
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    if (c.tid == 0) {
        tc::mbar_init(c.bar_s, 1);
        tc::mbar_init(c.bar_v, 1);
        tc::mbar_init(c.bar_rk, 1);
        tc::mbar_init(c.bar_rv, 1);
        *c.zero = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        const int gp = split * a.rows_per_split / GROUP;
        if (split < a.n_body && record_group(gp)) {
            const int64_t r = ((int64_t)gp * a.n_head_kv + kv) * 2 * REC;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a.k + r), "r"(2 * REC)
                         : "memory");
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a.v + r), "r"(2 * REC)
                         : "memory");
        }
    }
    if (c.warp == 0)
        tc::tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    asm volatile("griddepcontrol.wait;\n" ::: "memory");

    const int pos = a.positions[tok];
    const int limit = pos < a.origin ? 0 : min(a.active, pos - a.origin + 1);
    const int tail_begin = a.active - min(a.active, a.tail);
    const bool tail_split = split >= a.n_body; // rows [tail_begin, active), original domain
    const int r0 = tail_split ? tail_begin : split * a.rows_per_split;
    const int r1 = tail_split ? limit : min(min(r0 + a.rows_per_split, tail_begin), limit);
    const int g0 = r0 / GROUP, g1 = (!tail_split && r1 > r0) ? (r1 + GROUP - 1) / GROUP : g0;

    // the next record group after grp, if the tile after grp is one (else -1)
    auto next_record = [=](int grp) { return grp + 1 < g1 && record_group(grp + 1) ? grp + 1 : -1; };
    Pipe pp = {0u, 0u, 0u, 0u, false, false};
    const bool first_rec = g0 < g1 && record_group(g0);
    if (c.tid == 0 && first_rec) {
        issue_raw(c, a, false, g0, kv);
        issue_raw(c, a, true, g0, kv);
    }
    pp.rk_pend = pp.rv_pend = first_rec;
    {
        // query head g = warp: q or WHT(q) rows; running max / denominator
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
        if (!tail_split)
            wht_regs(v, c.lane);
        float4 *qd = reinterpret_cast<float4 *>(c.qv + g * QLD + 8 * c.lane);
        qd[0] = make_float4(v[0], v[1], v[2], v[3]);
        qd[1] = make_float4(v[4], v[5], v[6], v[7]);
        if (c.tid < GMAX) {
            c.vec[V_M * 8 + c.tid] = -FLT_MAX;
            c.vec[V_DEN * 8 + c.tid] = 0.0f;
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    c.tmem = *tmem_slot;

    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    uint4 kw[4];          // raw K rows of the coming record group
    bool have_kw = false; // kw holds them (read at the end of the previous record tile)
    bool ok = true;
    if (tail_split) {
        // the tail buffer is a ring of 128 rows: row r at r % 128
        for (int rr = r0; rr < r1 && ok;) {
            const int n = min(r1 - rr, GROUP - rr % GROUP);
            const int64_t first = (int64_t)(rr % GROUP) * row_bytes + kv * 512;
            ok = f16_tile(c, a.k + a.tail_off + first, a.v + a.tail_off + first, row_bytes, n,
                          a.scale, pp, acc);
            rr += n;
        }
    } else {
        for (int grp = g0; grp < g1 && ok; ++grp) {
            const int lo = max(r0, grp * GROUP), hi = min(r1, (grp + 1) * GROUP);
            const int next = next_record(grp);
            if (!record_group(grp)) {
                // staged group: rotated F16 rows in its stage slot
                const int slot = og + grp == 0 ? 0 : 1 + ((og + grp - 1) & 1);
                const int64_t first =
                    ((int64_t)slot * GROUP + (lo - grp * GROUP)) * row_bytes + kv * 512;
                ok = f16_tile(c, a.k + a.stage_off + first, a.v + a.stage_off + first,
                              row_bytes, hi - lo, a.scale, pp, acc);
                if (ok && next >= 0) {
                    // A0, A1 and the axes are free again after the tile's last barrier
                    if (c.tid == 0) {
                        issue_raw(c, a, false, next, kv);
                        issue_raw(c, a, true, next, kv);
                    }
                    pp.rk_pend = pp.rv_pend = true;
                }
                have_kw = false;
            } else {
                if (!have_kw) {
                    ok = fetch_raw(c, SM_A0, c.bar_rk, pp.ph_rk, kw);
                    pp.rk_pend = false;
                    if (__syncthreads_or(!ok)) // every raw read is done before the widening
                        break;
                }
                ok = record_tile(c, a, kw, lo - grp * GROUP, hi - lo, next, kv, pp, acc);
                have_kw = next >= 0;
            }
        }
    }
    if (!ok && c.tid == 0) {
        // give the MMAs and copies still in flight a bounded time to finish
        // before TMEM and shared memory go (MMA barriers: parity of the last
        // expected phase, immediate if it completed)
        tc::mbar_wait(c.bar_s, pp.ph_s ^ 1u, c.zero, 100000000ull);
        tc::mbar_wait(c.bar_v, pp.ph_v ^ 1u, c.zero, 100000000ull);
        if (pp.rk_pend)
            tc::mbar_wait(c.bar_rk, pp.ph_rk, c.zero, 100000000ull);
        if (pp.rv_pend)
            tc::mbar_wait(c.bar_rv, pp.ph_rv, c.zero, 100000000ull);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (c.warp == 0)
        tc::tmem_dealloc(c.tmem, TMEM_COLS);

    // ---- numerator rows x[q][dim] (A0 is free now), rotated back in body splits
    float *x = reinterpret_cast<float *>(sm + SM_A0);
    {
        const int s = c.warp >> 2, L = 32 * (c.warp & 3) + c.lane;
        const int d = 128 * s + unperm(L);
#pragma unroll
        for (int q = 0; q < 8; ++q)
            x[q * QLD + d] = acc[q];
    }
    __syncthreads();
    if (c.warp < c.G) {
        const int g = c.warp;
        float v[8];
        const float4 *xs = reinterpret_cast<const float4 *>(x + g * QLD + 8 * c.lane);
        const float4 v0 = xs[0], v1 = xs[1];
        v[0] = v0.x, v[1] = v0.y, v[2] = v0.z, v[3] = v0.w;
        v[4] = v1.x, v[5] = v1.y, v[6] = v1.z, v[7] = v1.w;
        if (!tail_split)
            wht_regs(v, c.lane);
        const int64_t n_rows = (int64_t)a.n_tokens * a.n_head;
        const int64_t row = (int64_t)tok * a.n_head + kv * c.G + g;
        float *rec = a.partials + ((int64_t)split * n_rows + row) * 258;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float2 *>(rec + 8 * c.lane + 2 * i) =
                make_float2(v[2 * i], v[2 * i + 1]);
        if (c.lane == 0) {
            rec[256] = c.vec[V_M * 8 + g];
            rec[257] = ok ? c.vec[V_DEN * 8 + g] : __int_as_float(0x7fc00000); // NaN poisons
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
    static std::atomic<unsigned long long> attr{0};
    cudaError_t e = set_smem_limit((const void *)kvarn4_partials_kernel, k4::SM_BYTES, attr);
    if (e != cudaSuccess)
        return e;
    // programmatic dependent of the previous kernel on the stream (see the
    // kernel's griddepcontrol.wait)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)l.n_splits, (unsigned)l.n_head_kv, (unsigned)l.n_tokens);
    cfg.blockDim = dim3(k4::NT, 1, 1);
    cfg.dynamicSmemBytes = k4::SM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kvarn4_partials_kernel, a);
}

} // namespace xq
