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

__global__ void __launch_bounds__(k4::NT, 2) kvarn4_partials_kernel(const Kvarn4Args a) {
    using namespace k4;
    extern __shared__ __align__(16) uint8_t sm[];
    float *q_s = reinterpret_cast<float *>(sm + SM_Q);
    float *qr_s = reinterpret_cast<float *>(sm + SM_QR);
    float *qs_s = reinterpret_cast<float *>(sm + SM_QS);
    float *p_s = reinterpret_cast<float *>(sm + SM_P);
    float *s_s = reinterpret_cast<float *>(sm + SM_S);
    float *ws_s = reinterpret_cast<float *>(sm + SM_WS);
    float *red = reinterpret_cast<float *>(sm + SM_RED); // [0,16) qz, [16,24) m, [24,32) den,
                                                         // [32,40) alpha, [40,56) wz
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, kv = blockIdx.y, tok = blockIdx.z;
    const int G = a.n_head / a.n_head_kv;
    const int phys = 2 * a.n_head_kv;
    const int64_t row_bytes = (int64_t)a.n_head_kv * 512;

    // ---- the query rows of this KV head, original and rotated
    for (int i = tid; i < G * 256; i += NT) {
        const int g = i >> 8, d = i & 255;
        const float x = a.q[((int64_t)tok * a.n_head + kv * G + g) * 256 + d];
        q_s[i] = x;
        qr_s[i] = x;
    }
    if (tid < GMAX) {
        red[16 + tid] = -FLT_MAX;
        red[24 + tid] = 0.0f;
    }
    __syncthreads();
    wht256_smem(qr_s, G, tid);

    const int pos = a.positions[tok];
    const int limit = pos < a.origin ? 0 : min(a.active, pos - a.origin + 1);
    const int r0 = split * a.rows_per_split;
    const int r1 = min(r0 + a.rows_per_split, limit);
    const int tail_begin = a.active - min(a.active, a.tail);
    const int live = a.active ? (a.active - 1) / GROUP : 0;
    float acc_r[GMAX], acc_t[GMAX];
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
        acc_r[g] = acc_t[g] = 0.0f;

    auto is_staged = [&](int grp) {
        return a.origin / GROUP + grp == 0 || (grp == live && (a.active % GROUP) != 0);
    };
    // a record group is read from its records when some of its rows in
    // [r0, r1) are below the tail and the group is not staged
    auto uses_records = [&](int grp) {
        const int lo = max(r0, grp * GROUP), hi = min(min(r1, (grp + 1) * GROUP), tail_begin);
        return lo < hi && !is_staged(grp);
    };
    auto prefetch = [&](int grp, int buf) {
        uint8_t *dst = sm + SM_REC + buf * SET;
        for (int i = tid; i < SET / 16; i += NT) {
            const int which = i / (REC / 16), off = (i % (REC / 16)) * 16;
            const uint8_t *plane = which < 2 ? a.k : a.v;
            const int ph = 2 * kv + (which & 1);
            cp_async<16>(smem_u32(dst + which * REC + off),
                         plane + ((int64_t)grp * phys + ph) * REC + off);
        }
    };

    // online softmax over the scores in s_s[g][0..n): running max/denominator
    // update, weights back into s_s, per-query rescale factor in red[32 + g]
    auto softmax_tile = [&](int n) {
        if (warp < G) {
            const int g = warp;
            float mx = -FLT_MAX;
            for (int t = lane; t < n; t += 32)
                mx = fmaxf(mx, s_s[g * 128 + t]);
#pragma unroll
            for (int o = 16; o; o >>= 1)
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_old = red[16 + g], den_old = red[24 + g];
            const float m_new = fmaxf(m_old, mx);
            const float alpha = den_old == 0.0f ? 0.0f : expf(m_old - m_new);
            float sum = 0.0f;
            for (int t = lane; t < n; t += 32) {
                const float w = expf(s_s[g * 128 + t] - m_new);
                s_s[g * 128 + t] = w;
                sum += w;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1)
                sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) {
                red[16 + g] = m_new;
                red[24 + g] = den_old * alpha + sum;
                red[32 + g] = alpha;
            }
        }
        __syncthreads();
    };

    // rows [lo, hi) of F16 rows (stage: rotated, tail: original), straight
    // from global memory; rows_base addresses row 0 of this plane region and
    // row(i) maps a compact row to its region row
    auto f16_rows = [&](int lo, int hi, bool original, auto region_row) {
        for (int c0 = lo; c0 < hi; c0 += 128) {
            const int n = min(128, hi - c0);
            // scores: thread = (row, slice)
            {
                const int t = tid & 127, s = tid >> 7;
                float acc[GMAX];
#pragma unroll
                for (int g = 0; g < GMAX; ++g)
                    acc[g] = 0.0f;
                if (t < n) {
                    const uint8_t *krow = region_row(a.k, c0 + t) + kv * 512 + s * 256;
                    const float *qv = (original ? q_s : qr_s) + s * 128;
                    for (int d8 = 0; d8 < 16; ++d8) {
                        const uint4 raw = *reinterpret_cast<const uint4 *>(krow + 16 * d8);
                        const __half2 *hp = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 kf = __half22float2(hp[j]);
                            const int d = 8 * d8 + 2 * j;
#pragma unroll
                            for (int g = 0; g < GMAX; ++g)
                                if (g < G)
                                    acc[g] = fmaf(qv[g * 256 + d], kf.x,
                                                  fmaf(qv[g * 256 + d + 1], kf.y, acc[g]));
                        }
                    }
                }
#pragma unroll
                for (int g = 0; g < GMAX; ++g)
                    if (g < G)
                        p_s[(s * 8 + g) * 128 + t] = acc[g];
            }
            __syncthreads();
            for (int i = tid; i < G * 128; i += NT) {
                const int g = i >> 7, t = i & 127;
                s_s[g * 128 + t] =
                    t < n ? (p_s[g * 128 + t] + p_s[(8 + g) * 128 + t]) * a.scale : -FLT_MAX;
            }
            __syncthreads();
            softmax_tile(n);
            // value numerator: thread = dimension
            {
                const int d = tid;
                float add[GMAX];
#pragma unroll
                for (int g = 0; g < GMAX; ++g)
                    add[g] = 0.0f;
                for (int t = 0; t < n; ++t) {
                    const float vf = h2f(region_row(a.v, c0 + t) + kv * 512 + 2 * d);
#pragma unroll
                    for (int g = 0; g < GMAX; ++g)
                        if (g < G)
                            add[g] = fmaf(s_s[g * 128 + t], vf, add[g]);
                }
#pragma unroll
                for (int g = 0; g < GMAX; ++g)
                    if (g < G) {
                        const float al = red[32 + g];
                        if (original) {
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
    };

    // ---- walk the split's record groups
    const int g0 = r0 / GROUP, g1 = r1 > r0 ? (r1 + GROUP - 1) / GROUP : g0;
    int next_rec = g0; // next group whose records are prefetched
    while (next_rec < g1 && !uses_records(next_rec))
        ++next_rec;
    int buf = 0;
    if (next_rec < g1)
        prefetch(next_rec, 0);
    cp_async_commit();
    for (int grp = g0; grp < g1; ++grp) {
        const int lo = max(r0, grp * GROUP), hi = min(r1, (grp + 1) * GROUP);
        const int body_hi = min(hi, tail_begin);
        if (lo < body_hi) {
            if (is_staged(grp)) {
                const int slot = (a.origin / GROUP + grp) == 0
                                     ? 0
                                     : 1 + ((a.origin / GROUP + grp - 1) & 1);
                f16_rows(lo, body_hi, false, [&](const uint8_t *plane, int row) {
                    return plane + a.stage_off +
                           ((int64_t)slot * GROUP + (row - grp * GROUP)) * row_bytes;
                });
            } else {
                // records of this group are in buffer `buf`; prefetch the next
                int nxt = grp + 1;
                while (nxt < g1 && !uses_records(nxt))
                    ++nxt;
                if (nxt < g1)
                    prefetch(nxt, buf ^ 1);
                cp_async_commit();
                cp_async_wait<1>();
                __syncthreads();
                const uint8_t *rk0 = sm + SM_REC + buf * SET;
                const int t0 = lo - grp * GROUP, n = body_hi - lo; // rows t0 .. t0 + n
                // per-group query factors: qs[s][d][g] = WHT(q)_g[s*128 + d] * scale_k_s[d],
                // qz[s][g] = sum_d WHT(q)_g[s*128 + d] * zero_k_s[d]
                {
                    const int d = tid & 127, s = tid >> 7;
                    const uint8_t *rec = rk0 + s * REC;
                    const float sc = h2f(rec + 8192 + 2 * d), zr = h2f(rec + 8448 + 2 * d);
#pragma unroll
                    for (int g = 0; g < GMAX; ++g) {
                        const float qv = g < G ? qr_s[g * 256 + s * 128 + d] : 0.0f;
                        qs_s[(s * 128 + d) * 8 + g] = qv * sc;
                        float z = qv * zr;
#pragma unroll
                        for (int o = 16; o; o >>= 1)
                            z += __shfl_xor_sync(0xffffffffu, z, o);
                        if (lane == 0)
                            p_s[(s * 8 + g) * 128 + (d >> 5)] = z; // 4 warp sums per (s, g)
                    }
                }
                __syncthreads();
                if (tid < 16) {
                    const int s = tid >> 3, g = tid & 7;
                    const float *z = p_s + (s * 8 + g) * 128;
                    red[s * 8 + g] = (z[0] + z[1]) + (z[2] + z[3]);
                }
                __syncthreads();
                // scores: thread = (token, slice)
                {
                    const int t = tid & 127, s = tid >> 7;
                    const uint8_t *nib = rk0 + s * REC; // [d][token] nibbles
                    float acc[GMAX];
#pragma unroll
                    for (int g = 0; g < GMAX; ++g)
                        acc[g] = 0.0f;
                    const float4 *qs4 = reinterpret_cast<const float4 *>(qs_s + s * 128 * 8);
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
                        p_s[(s * 8 + g) * 128 + t] = (acc[g] + red[s * 8 + g]) * other;
                }
                __syncthreads();
                for (int i = tid; i < G * 128; i += NT) {
                    const int g = i >> 7, j = i & 127; // j-th row of the range
                    const int t = t0 + j;
                    s_s[g * 128 + j] = j < n ? (p_s[g * 128 + t] + p_s[(8 + g) * 128 + t]) * a.scale
                                             : -FLT_MAX;
                }
                __syncthreads();
                softmax_tile(n);
                // weights * scale_v and sum_t weights * zero_v, per slice
                {
                    const int j = tid & 127, s = tid >> 7;
                    const uint8_t *vrec = rk0 + (2 + s) * REC;
                    const float sc = j < n ? h2f(vrec + 8192 + 2 * (t0 + j)) : 0.0f;
                    const float zr = j < n ? h2f(vrec + 8448 + 2 * (t0 + j)) : 0.0f;
#pragma unroll
                    for (int g = 0; g < GMAX; ++g) {
                        const float w = (g < G && j < n) ? s_s[g * 128 + j] : 0.0f;
                        ws_s[(s * 128 + j) * 8 + g] = w * sc;
                        float z = w * zr;
#pragma unroll
                        for (int o = 16; o; o >>= 1)
                            z += __shfl_xor_sync(0xffffffffu, z, o);
                        if (lane == 0)
                            p_s[(s * 8 + g) * 128 + (j >> 5)] = z;
                    }
                }
                __syncthreads();
                if (tid < 16) {
                    const int s = tid >> 3, g = tid & 7;
                    const float *z = p_s + (s * 8 + g) * 128;
                    red[40 + s * 8 + g] = (z[0] + z[1]) + (z[2] + z[3]);
                }
                __syncthreads();
                // value numerator: thread = dimension (slice s, dim c)
                {
                    const int d = tid, s = d >> 7, c = d & 127;
                    const uint8_t *vrec = rk0 + (2 + s) * REC; // [token][dim] nibbles
                    const float4 *ws4 = reinterpret_cast<const float4 *>(ws_s + s * 128 * 8);
                    float add[GMAX];
#pragma unroll
                    for (int g = 0; g < GMAX; ++g)
                        add[g] = 0.0f;
                    for (int j = 0; j < n; ++j) {
                        const uint32_t b = vrec[(t0 + j) * 64 + (c >> 1)];
                        const float nv = (float)((b >> ((c & 1) * 4)) & 15u);
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
                    const float other = h2f(vrec + 8704 + 2 * c);
#pragma unroll
                    for (int g = 0; g < GMAX; ++g)
                        if (g < G) {
                            const float al = red[32 + g];
                            acc_r[g] = acc_r[g] * al + (add[g] + red[40 + s * 8 + g]) * other;
                            acc_t[g] *= al;
                        }
                }
                __syncthreads();
                buf ^= 1;
            }
        }
        const int tail_lo = max(lo, tail_begin);
        if (tail_lo < hi)
            f16_rows(tail_lo, hi, true, [&](const uint8_t *plane, int row) {
                return plane + a.tail_off + (int64_t)(row % GROUP) * row_bytes;
            });
    }
    cp_async_wait<0>();

    // ---- numerator = WHT(rotated part) + tail part; partial record
    float *x = qr_s; // reuse: the rotated query is no longer needed
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GMAX; ++g)
        if (g < G)
            x[g * 256 + tid] = acc_r[g];
    __syncthreads();
    wht256_smem(x, G, tid);
    const int64_t n_rows = (int64_t)a.n_tokens * a.n_head;
    for (int g = 0; g < G; ++g) {
        const int64_t row = (int64_t)tok * a.n_head + kv * G + g;
        float *rec = a.partials + ((int64_t)split * n_rows + row) * 258;
        rec[tid] = x[g * 256 + tid] + acc_t[g];
        if (tid == 0) {
            rec[256] = red[16 + g];
            rec[257] = red[24 + g];
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
