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
// (thread = token x slice); the value numerator is accumulated per dimension
// in registers, other_d * (sum_t (w_t scale_t) nib_td + sum_t w_t zero_t)
// (thread = dimension).  Stage and tail rows are read straight from global
// memory with the same thread mapping.
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
    int tid, warp, lane, G;
};

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

// n <= 128 consecutive F16 rows (row stride row_bytes; this KV head's 256
// values at +kv*512): stage rows (rotated, meet WHT(q), accumulate into
// acc_r) or tail rows (original, meet q, accumulate into acc_t).
template <bool ORIGINAL>
__device__ __forceinline__ void f16_tile(const Cta c, const uint8_t *krows, const uint8_t *vrows,
                                         int64_t row_bytes, int n, float scale,
                                         float (&acc_r)[GMAX], float (&acc_t)[GMAX]) {
    {
        // scores: thread = (row, slice); the slice's 8 + 8 loads in flight
        const int t = c.tid & 127, sl = c.tid >> 7;
        float acc[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            acc[g] = 0.0f;
        if (t < n) {
            const uint4 *krow = reinterpret_cast<const uint4 *>(krows + t * row_bytes + sl * 256);
            const float *qv = (ORIGINAL ? c.q : c.qr) + sl * 128;
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                uint4 raw[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    raw[i] = __ldg(krow + 8 * hlf + i);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const __half2 *hp = reinterpret_cast<const __half2 *>(&raw[i]);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 kf = __half22float2(hp[j]);
                        const int d = 8 * (8 * hlf + i) + 2 * j;
#pragma unroll
                        for (int g = 0; g < GMAX; ++g)
                            if (g < c.G)
                                acc[g] = fmaf(qv[g * 256 + d], kf.x,
                                              fmaf(qv[g * 256 + d + 1], kf.y, acc[g]));
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            if (g < c.G)
                c.p[(sl * 8 + g) * 128 + t] = acc[g];
    }
    __syncthreads();
    for (int i = c.tid; i < c.G * 128; i += NT) {
        const int g = i >> 7, t = i & 127;
        c.s[g * 128 + t] = t < n ? (c.p[g * 128 + t] + c.p[(8 + g) * 128 + t]) * scale : -FLT_MAX;
    }
    __syncthreads();
    softmax_tile(c, n);
    {
        // value numerator: thread = dimension, 16 rows' loads in flight
        const int d = c.tid;
        float add[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            add[g] = 0.0f;
        for (int t0 = 0; t0 < n; t0 += 16) {
            float vf[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                vf[j] = t0 + j < n ? __half2float(__ldg(reinterpret_cast<const __half *>(
                                         vrows + (t0 + j) * row_bytes + 2 * d)))
                                   : 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
#pragma unroll
                for (int g = 0; g < GMAX; ++g)
                    if (g < c.G)
                        add[g] = fmaf(t0 + j < n ? c.s[g * 128 + t0 + j] : 0.0f, vf[j], add[g]);
        }
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            if (g < c.G) {
                const float al = c.red[32 + g];
                if (ORIGINAL) {
                    acc_t[g] = acc_t[g] * al + add[g];
                    acc_r[g] *= al;
                } else {
                    acc_r[g] = acc_r[g] * al + add[g];
                    acc_t[g] *= al;
                }
            }
    }
    __syncthreads();
}

// Rows [t0, t0 + n) of one complete record group whose four records (K slice
// 0/1, V slice 0/1) are in shared memory at rk.
__device__ __forceinline__ void record_tile(const Cta c, const uint8_t *rk, int t0, int n,
                                            float scale, float (&acc_r)[GMAX],
                                            float (&acc_t)[GMAX]) {
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
        // scores: thread = (token, slice)
        const int t = c.tid & 127, sl = c.tid >> 7;
        const uint8_t *nib = rk + sl * REC; // [d][token] nibbles
        const float4 *qs4 = reinterpret_cast<const float4 *>(c.qs + sl * 128 * 8);
        float acc[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            acc[g] = 0.0f;
        for (int d = 0; d < 128; ++d) {
            const uint32_t b = nib[d * 64 + (t >> 1)];
            const float nv = (float)((b >> ((t & 1) * 4)) & 15u);
            const float4 qa = qs4[d * 2], qb = qs4[d * 2 + 1];
            acc[0] = fmaf(qa.x, nv, acc[0]);
            acc[1] = fmaf(qa.y, nv, acc[1]);
            acc[2] = fmaf(qa.z, nv, acc[2]);
            acc[3] = fmaf(qa.w, nv, acc[3]);
            acc[4] = fmaf(qb.x, nv, acc[4]);
            acc[5] = fmaf(qb.y, nv, acc[5]);
            acc[6] = fmaf(qb.z, nv, acc[6]);
            acc[7] = fmaf(qb.w, nv, acc[7]);
        }
        const float other = h2f(nib + 8704 + 2 * t);
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            c.p[(sl * 8 + g) * 128 + t] = (acc[g] + c.red[sl * 8 + g]) * other;
    }
    __syncthreads();
    for (int i = c.tid; i < c.G * 128; i += NT) {
        const int g = i >> 7, j = i & 127, t = t0 + j;
        c.s[g * 128 + j] =
            j < n ? (c.p[g * 128 + t] + c.p[(8 + g) * 128 + t]) * scale : -FLT_MAX;
    }
    __syncthreads();
    softmax_tile(c, n);
    {
        // weights * scale_v and sum_t weights * zero_v, per slice
        const int j = c.tid & 127, sl = c.tid >> 7;
        const uint8_t *vrec = rk + (2 + sl) * REC;
        const float sc = j < n ? h2f(vrec + 8192 + 2 * (t0 + j)) : 0.0f;
        const float zr = j < n ? h2f(vrec + 8448 + 2 * (t0 + j)) : 0.0f;
        float w[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            w[g] = (g < c.G && j < n) ? c.s[g * 128 + j] : 0.0f;
        float4 *ws4 = reinterpret_cast<float4 *>(c.ws + (sl * 128 + j) * 8);
        ws4[0] = make_float4(w[0] * sc, w[1] * sc, w[2] * sc, w[3] * sc);
        ws4[1] = make_float4(w[4] * sc, w[5] * sc, w[6] * sc, w[7] * sc);
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            float z = w[g] * zr;
#pragma unroll
            for (int o = 16; o; o >>= 1)
                z += __shfl_xor_sync(0xffffffffu, z, o);
            if (c.lane == 0)
                c.p[(sl * 8 + g) * 128 + (j >> 5)] = z;
        }
    }
    __syncthreads();
    if (c.tid < 16) {
        const float *z = c.p + c.tid * 128;
        c.red[40 + c.tid] = (z[0] + z[1]) + (z[2] + z[3]);
    }
    __syncthreads();
    {
        // value numerator: thread = dimension (slice sl, dim cc)
        const int d = c.tid, sl = d >> 7, cc = d & 127;
        const uint8_t *vrec = rk + (2 + sl) * REC; // [token][dim] nibbles
        const float4 *ws4 = reinterpret_cast<const float4 *>(c.ws + sl * 128 * 8);
        float add[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            add[g] = 0.0f;
        for (int j = 0; j < n; ++j) {
            const uint32_t b = vrec[(t0 + j) * 64 + (cc >> 1)];
            const float nv = (float)((b >> ((cc & 1) * 4)) & 15u);
            const float4 wa = ws4[j * 2], wb = ws4[j * 2 + 1];
            add[0] = fmaf(wa.x, nv, add[0]);
            add[1] = fmaf(wa.y, nv, add[1]);
            add[2] = fmaf(wa.z, nv, add[2]);
            add[3] = fmaf(wa.w, nv, add[3]);
            add[4] = fmaf(wb.x, nv, add[4]);
            add[5] = fmaf(wb.y, nv, add[5]);
            add[6] = fmaf(wb.z, nv, add[6]);
            add[7] = fmaf(wb.w, nv, add[7]);
        }
        const float other = h2f(vrec + 8704 + 2 * cc);
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
            if (g < c.G) {
                const float al = c.red[32 + g];
                acc_r[g] = acc_r[g] * al + (add[g] + c.red[40 + sl * 8 + g]) * other;
                acc_t[g] *= al;
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
    float acc_r[GMAX], acc_t[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
        acc_r[g] = acc_t[g] = 0.0f;

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
    float *x = c.qr; // the rotated query is no longer needed
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
        if (g < c.G)
            x[g * 256 + c.tid] = acc_r[g];
    __syncthreads();
    wht256_smem(x, c.G, c.tid);
    const int64_t n_rows = (int64_t)a.n_tokens * a.n_head;
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
        if (g >= c.G)
            break;
        const int64_t row = (int64_t)tok * a.n_head + kv * c.G + g;
        float *rec = a.partials + ((int64_t)split * n_rows + row) * 258;
        rec[c.tid] = x[g * 256 + c.tid] + acc_t[g];
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
