// Split-KV flash decode over F16 / Q8_0 / Q4_0 KV caches, and the fixed-order
// log-sum-exp merge of split partials.
//
// Semantics (ggml-cpu FLASH_ATTN_EXT, patches/0008 context lines 4-35 and the
// split-KV branch of patches/0006 lines 7-14; RKVA range partials
// shaders/rkva/rkva_range_attn.hlsl:59-106 and reducer
// rkva_range_reduce_opt.hlsl:26-133):
//   * q is first converted to K's dot type (F16 for F16 K, Q8_0 for Q8_0/Q4_0
//     K) when q_convert is set; the RKVA entry uses raw F32 q;
//   * s = (q . k) * scale, softcap, + slope * mask; masked (-inf) rows skip;
//   * GQA: q head h reads kv head h / (n_head / n_head_kv);
//   * KV values are dequantised exactly in registers; products and sums are
//     fp32 (the float accumulation the target tolerance is written for).
//
// Layout of work: one CTA = (split of KV rows, kv head, block of NR q-rows,
// sequence).  The NR q-rows are the (query, head) pairs that share the kv
// head, so every K/V byte is read once for all of them.  K/V tiles of R rows
// stream into shared memory through a 2-stage cp.async pipeline; scores use
// LPR lanes per row (dims interleaved in 4-dim chunks) and warp shuffles; the
// PV product gives each thread 4 dims x NR q-rows over a group of rows.
#include <atomic>
#include <float.h>
#include <math.h>

#include "xq_common.cuh"
#include "xq_internal.h"

namespace xq {

constexpr int kThreads = 256;

template <int T, int D, int NR, int R, int VW>
__global__ void __launch_bounds__(kThreads, 2) fa_decode_kernel(const DecodeArgs a) {
    constexpr int REC = rec_bytes(T, D);
    constexpr int SS = smem_stride(REC);
    constexpr int NCH = D / 4;          // 4-dim chunks per row
    constexpr int LPR = kThreads / R;   // score lanes per row
    constexpr int NRG = kThreads / NCH; // PV row groups
    constexpr int RPG = R / NRG;        // rows per PV group
    constexpr int VPR = REC / VW;       // copy vectors per row
    constexpr int NW = kThreads / 32;
    static_assert(REC % VW == 0, "row bytes must split into copy vectors");
    static_assert(NCH % LPR == 0 && R % NRG == 0, "tile shape");

    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t *kbuf = smem;                                      // [2][R][SS]
    uint8_t *vbuf = kbuf + 2 * R * SS;                         // [2][R][SS]
    float *q_s = reinterpret_cast<float *>(vbuf + 2 * R * SS); // [NR][D]
    float *p_s = q_s + NR * D;                                 // [R][NR]
    float *red = p_s + R * NR;                                 // [NW][NR]
    float *m_s = red + NW * NR;                                // [NR]
    float *l_s = m_s + NR;                                     // [NR]
    float *al_s = l_s + NR;                                    // [NR]
    float *slope_s = al_s + NR;                                // [NR]
    int64_t *moff_s = reinterpret_cast<int64_t *>(slope_s + NR); // [NR]
    int *lim_s = reinterpret_cast<int *>(moff_s + NR);         // [NR]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = blockIdx.y % a.n_head_kv;
    const int qb = blockIdx.y / a.n_head_kv;
    const int s = blockIdx.z;
    const int64_t split = a.split_begin + blockIdx.x;
    const int64_t r0 = split * a.rows_per_split;
    const int64_t r1 = min((int64_t)a.n_kv, r0 + a.rows_per_split);
    const int jbase = qb * NR;
    const int nj = min(NR, a.n_qrows - jbase);

    const uint8_t *kbase = a.k + (int64_t)kvh * a.k_nb2 + (int64_t)(s / a.rk3) * a.k_nb3;
    const uint8_t *vbase = a.v + (int64_t)kvh * a.v_nb2 + (int64_t)(s / a.rv3) * a.v_nb3;

    auto load_tile = [&](int stage, int64_t t0) {
        const int nrows = (int)min((int64_t)R, r1 - t0);
        uint8_t *kd = kbuf + stage * R * SS;
        uint8_t *vd = vbuf + stage * R * SS;
        for (int idx = tid; idx < nrows * VPR; idx += kThreads) {
            const int r = idx / VPR, c = idx - r * VPR;
            cp_async<VW>(smem_u32(kd + r * SS + c * VW), kbase + (t0 + r) * a.k_nb1 + c * VW);
            cp_async<VW>(smem_u32(vd + r * SS + c * VW), vbase + (t0 + r) * a.v_nb1 + c * VW);
        }
    };

    if (r0 < r1)
        load_tile(0, r0);
    cp_async_commit();

    // ---- prologue: q rows (converted to K's dot type), per-row constants ----
    for (int j = tid; j < NR; j += kThreads) {
        m_s[j] = -INFINITY;
        l_s[j] = 0.0f;
        float slope = 1.0f;
        int64_t moff = 0;
        int lim = a.n_kv;
        if (j < nj) {
            const int jj = jbase + j, iq1 = jj / a.G, h = kvh * a.G + jj % a.G;
            if (a.alibi)
                slope = h < a.n_head_log2 ? powf(a.m0, (float)(h + 1))
                                          : powf(a.m1, (float)(2 * (h - a.n_head_log2) + 1));
            moff = (int64_t)iq1 * a.m_nb1 + (int64_t)(h % a.m_ne2) * a.m_nb2 +
                   (int64_t)(s % a.m_ne3) * a.m_nb3;
            if (a.positions) {
                const int pos = a.positions[iq1];
                lim = pos < a.origin ? 0 : min(a.active, pos - a.origin + 1);
            }
        }
        slope_s[j] = slope;
        moff_s[j] = moff;
        lim_s[j] = lim;
    }
    if (!a.q_convert || T == kF16) {
        for (int idx = tid; idx < NR * D; idx += kThreads) {
            const int j = idx / D, d = idx - j * D;
            float x = 0.0f;
            if (j < nj) {
                const int jj = jbase + j, iq1 = jj / a.G, h = kvh * a.G + jj % a.G;
                x = *reinterpret_cast<const float *>(a.q + (int64_t)iq1 * a.q_nb1 +
                                                     (int64_t)h * a.q_nb2 +
                                                     (int64_t)s * a.q_nb3 + 4 * d);
                if (a.q_convert)
                    x = __half2float(__float2half_rn(x));
            }
            q_s[idx] = x;
        }
    } else {
        // ggml quantize_row_q8_0 reference arithmetic, one warp per 32-block.
        for (int blk = warp; blk < NR * (D / 32); blk += NW) {
            const int j = blk / (D / 32), b = blk - j * (D / 32);
            float x = 0.0f;
            if (j < nj) {
                const int jj = jbase + j, iq1 = jj / a.G, h = kvh * a.G + jj % a.G;
                x = *reinterpret_cast<const float *>(a.q + (int64_t)iq1 * a.q_nb1 +
                                                     (int64_t)h * a.q_nb2 +
                                                     (int64_t)s * a.q_nb3 + 4 * (b * 32 + lane));
            }
            const float amax = warp_max(fabsf(x));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            const float qi = roundf(x * id);
            q_s[j * D + b * 32 + lane] = qi * __half2float(__float2half_rn(d));
        }
    }
    __syncthreads();

    // ---- main loop over R-row tiles ----
    const int row = tid / LPR, ql = tid % LPR;      // score mapping
    const int pc = tid % NCH, rg = tid / NCH;        // PV mapping
    float acc[NR][4];
#pragma unroll
    for (int j = 0; j < NR; ++j)
        acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;

    int stage = 0;
    for (int64_t t0 = r0; t0 < r1; t0 += R, stage ^= 1) {
        if (t0 + R < r1)
            load_tile(stage ^ 1, t0 + R);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();

        const uint8_t *ktile = kbuf + stage * R * SS;
        const uint8_t *vtile = vbuf + stage * R * SS;
        const int64_t grow = t0 + row;
        const bool rvalid = grow < r1;

        float sc[NR];
#pragma unroll
        for (int j = 0; j < NR; ++j)
            sc[j] = 0.0f;
        if (rvalid) {
            const uint8_t *krow = ktile + row * SS;
#pragma unroll 4
            for (int cc = 0; cc < NCH / LPR; ++cc) {
                const int c = cc * LPR + ql;
                float kx[4];
                load4<T>(krow, c, kx);
#pragma unroll
                for (int j = 0; j < NR; ++j) {
                    const float4 qq = *reinterpret_cast<const float4 *>(q_s + j * D + 4 * c);
                    sc[j] = fmaf(qq.x, kx[0], sc[j]);
                    sc[j] = fmaf(qq.y, kx[1], sc[j]);
                    sc[j] = fmaf(qq.z, kx[2], sc[j]);
                    sc[j] = fmaf(qq.w, kx[3], sc[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < NR; ++j) {
#pragma unroll
            for (int o = 1; o < LPR; o <<= 1)
                sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], o);
            float x = sc[j] * a.scale;
            if (a.softcap != 0.0f)
                x = a.softcap * tanhf(x);
            if (a.mask && rvalid) {
                const float mv = slope_s[j] * __half2float(*reinterpret_cast<const __half *>(
                                                  a.mask + moff_s[j] + 2 * grow));
                x = mv == -INFINITY ? -INFINITY : x + mv;
            }
            if (!rvalid || j >= nj || grow >= lim_s[j])
                x = -INFINITY;
            sc[j] = x;
        }
        // tile max per q-row: over the rows of this warp, then across warps
#pragma unroll
        for (int j = 0; j < NR; ++j) {
            float mx = sc[j];
#pragma unroll
            for (int o = LPR; o < 32; o <<= 1)
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0)
                red[warp * NR + j] = mx;
        }
        __syncthreads();
        if (tid < NR) {
            float mt = red[tid];
#pragma unroll
            for (int w = 1; w < NW; ++w)
                mt = fmaxf(mt, red[w * NR + tid]);
            const float mo = m_s[tid];
            const float mn = fmaxf(mo, mt);
            al_s[tid] = mo == -INFINITY ? (mn == -INFINITY ? 1.0f : 0.0f) : expf(mo - mn);
            m_s[tid] = mn;
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < NR; ++j) {
            const float p = sc[j] == -INFINITY ? 0.0f : expf(sc[j] - m_s[j]);
            if (ql == (j % LPR))
                p_s[row * NR + j] = p;
            float sum = p;
#pragma unroll
            for (int o = LPR; o < 32; o <<= 1)
                sum += __shfl_xor_sync(0xffffffffu, sum, o);
            sc[j] = sum;
        }
        __syncthreads(); // red (max) fully consumed before reuse as sums
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < NR; ++j)
                red[warp * NR + j] = sc[j];
        }
        __syncthreads();
        if (tid < NR) {
            float lt = red[tid];
#pragma unroll
            for (int w = 1; w < NW; ++w)
                lt += red[w * NR + tid];
            l_s[tid] = l_s[tid] * al_s[tid] + lt;
        }
        // PV
#pragma unroll
        for (int j = 0; j < NR; ++j) {
            const float al = al_s[j];
            acc[j][0] *= al;
            acc[j][1] *= al;
            acc[j][2] *= al;
            acc[j][3] *= al;
        }
        const int nrows = (int)min((int64_t)R, r1 - t0);
#pragma unroll 2
        for (int rr = 0; rr < RPG; ++rr) {
            const int r = rg * RPG + rr;
            if (r < nrows) {
                float vx[4];
                load4<T>(vtile + r * SS, pc, vx);
#pragma unroll
                for (int j = 0; j < NR; ++j) {
                    const float p = p_s[r * NR + j];
                    acc[j][0] = fmaf(p, vx[0], acc[j][0]);
                    acc[j][1] = fmaf(p, vx[1], acc[j][1]);
                    acc[j][2] = fmaf(p, vx[2], acc[j][2]);
                    acc[j][3] = fmaf(p, vx[3], acc[j][3]);
                }
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---- epilogue: combine PV row groups in a fixed order ----
    float *obuf = reinterpret_cast<float *>(kbuf); // [NR][D], aliases stage buffers
    for (int g = NRG - 1; g >= 1; --g) {
        if (rg == g) {
#pragma unroll
            for (int j = 0; j < NR; ++j) {
                float4 *o = reinterpret_cast<float4 *>(obuf + j * D + 4 * pc);
                if (g == NRG - 1) {
                    *o = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
                } else {
                    float4 t = *o;
                    *o = make_float4(t.x + acc[j][0], t.y + acc[j][1], t.z + acc[j][2],
                                     t.w + acc[j][3]);
                }
            }
        }
        __syncthreads();
    }
    if (rg != 0)
        return;
#pragma unroll
    for (int j = 0; j < NR; ++j) {
        if (j >= nj)
            break;
        float o[4];
        if (NRG > 1) {
            const float4 t = *reinterpret_cast<const float4 *>(obuf + j * D + 4 * pc);
            o[0] = t.x + acc[j][0];
            o[1] = t.y + acc[j][1];
            o[2] = t.z + acc[j][2];
            o[3] = t.w + acc[j][3];
        } else {
            o[0] = acc[j][0];
            o[1] = acc[j][1];
            o[2] = acc[j][2];
            o[3] = acc[j][3];
        }
        const int jj = jbase + j, iq1 = jj / a.G, h = kvh * a.G + jj % a.G;
        const int64_t orow = ((int64_t)s * a.n_q + iq1) * a.n_head + h;
        float m = m_s[j], l = l_s[j];
        if (a.direct) {
            if (a.sinks) {
                const float sk = a.sinks[h];
                if (sk > m) {
                    const float ms = expf(m - sk);
                    o[0] *= ms;
                    o[1] *= ms;
                    o[2] *= ms;
                    o[3] *= ms;
                    l = l * ms + 1.0f;
                    m = sk;
                } else {
                    l += expf(sk - m);
                }
            }
            const float inv = l == 0.0f ? 0.0f : 1.0f / l;
            *reinterpret_cast<float4 *>(a.dst + orow * D + 4 * pc) =
                make_float4(o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv);
            if (a.lse && pc == 0)
                a.lse[orow] = l == 0.0f ? -INFINITY : m + logf(l);
        } else {
            float *rec = a.partials + ((split - a.split_begin) * (int64_t)a.n_seq * a.n_q *
                                           a.n_head + orow) * (D + 2);
            rec[4 * pc + 0] = o[0];
            rec[4 * pc + 1] = o[1];
            rec[4 * pc + 2] = o[2];
            rec[4 * pc + 3] = o[3];
            if (pc == 0) {
                rec[D] = l == 0.0f ? -FLT_MAX : m;
                rec[D + 1] = l;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// LSE merge: one thread-block cluster per output row, one CTA per 32 dims.
// Every CTA reads all splits' (m, l), forms the global max M, the weights
// w_s = exp(m_s - M) and L = sum l_s w_s (fixed order: thread-strided, then
// the warp tree, then warps in order); its 8 warps own contiguous runs of
// splits for its 32 dims (lane = dim, one 128-byte line per split) and their
// sums are added in warp order.  The numerators are requested together with
// (m, l), so the merge costs one memory latency.  Any non-finite input of a
// live split or a non-finite result poisons the whole row (NaN out, NaN lse):
// each CTA pushes its flag into every peer's shared memory and one cluster
// barrier later reads them all.  The order of every sum depends only on the
// number of splits, never on which GPU or launch produced each split.
namespace mg {
constexpr int NT = 256, NW = NT / 32, CACHE = 2048, XR = 24;
constexpr size_t STG_CAP = 64 * 1024; // staged numerators per CTA at most
constexpr size_t STG_PAD = 96 * 1024; // dynamic shared memory of a D = 256 staged CTA

__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void st_peer(int *local, uint32_t rank, int v) {
    uint32_t addr = (uint32_t)__cvta_generic_to_shared(local), peer;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(peer) : "r"(addr), "r"(rank));
    asm volatile("st.shared::cluster.u32 [%0], %1;\n" ::"r"(peer), "r"(v) : "memory");
}
} // namespace mg

// Rows are (group, row) pairs: group g merges splits [g * n_splits, (g + 1) *
// n_splits) of the partials.  With `records` set, each merged row is written
// as a partial record itself -- (O normalised, lse, 1), or (0, -FLT_MAX, 0)
// when empty, NaN when poisoned -- so merged groups merge again exactly like
// splits (sinks are applied only by a final, non-record merge).  A lane owns
// DL adjacent dims (DL = 2: 8-byte loads, half the CTAs per row).  With STG
// the CTA's numerators are first copied into shared memory (8-byte cp.async,
// dynamic shared memory of n_splits x 32 DL floats) instead of being held in
// registers.  Every dim is summed over the same split ranges in the same
// order in all variants.
template <int D, int DL, bool STG>
__global__ void __launch_bounds__(mg::NT) lse_merge_kernel(const float *__restrict__ part,
                                                           int64_t n_splits, int64_t n_rows,
                                                           float *__restrict__ out,
                                                           float *__restrict__ lse,
                                                           const float *__restrict__ sinks,
                                                           int n_head, int records,
                                                           int xchg) {
    using namespace mg;
    constexpr int NC = D / (32 * DL); // CTAs per row (the cluster)
    constexpr int CD = 32 * DL;       // dims per CTA
    __shared__ float2 wd_s[CACHE]; // (m, l), then (w, l) of each split
    __shared__ float red[NW];
    __shared__ float accw[NW][CD];
    __shared__ int flags_s[NC]; // slot r: CTA r's poison flag (written by CTA r)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int chunk = blockIdx.x % NC; // == rank in the cluster
    const int64_t row = blockIdx.x / NC; // group * n_rows + row in the group
    const int64_t grp = row / n_rows, grow = row - grp * n_rows;
    const int64_t stride = (int64_t)n_rows * (D + 2);
    const float *base = part + grp * n_splits * stride + grow * (D + 2);
    const bool cached = n_splits <= CACHE;
    auto md = [&](int64_t s) {
        return make_float2(base[s * stride + D], base[s * stride + D + 1]);
    };
    auto ld = [&](const float *p, float (&v)[DL]) {
        if constexpr (DL == 2) {
            const float2 t = *reinterpret_cast<const float2 *>(p);
            v[0] = t.x;
            v[1] = t.y;
        } else {
            v[0] = *p;
        }
    };
    // xchg: a numerator's poison reaches the row's other CTAs through the
    // cluster; without it (records of the decode kernels, which mark a
    // non-finite numerator with a NaN denominator) the (m, l) pass below sees
    // every row's poison in every CTA, and no cluster is launched
    if (xchg)
        cluster_arrive_relaxed(); // every peer has started before any DSMEM store below
    // the next decode may launch now; it waits for this grid before it writes
    // the partials read here
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    grid_dep_wait(); // partials come from the preceding kernel
    // this warp's splits [s0, s1), lane = dims d .. d + DL - 1; first XR
    // numerators in flight now
    const int d = chunk * CD + DL * lane;
    const int64_t s0 = n_splits * warp / NW, s1 = n_splits * (warp + 1) / NW;
    const float *xb = base + d;
    constexpr int XRR = STG ? 1 : XR;
    float x[XRR][DL];
    extern __shared__ __align__(16) float xs_s[]; // STG: [n_splits][CD] numerators
    if constexpr (STG) {
        // every numerator of this CTA's dims copied to shared memory (8-byte
        // copies, no registers held); read back in the same order below
        const float *cb = base + chunk * CD;
        for (int64_t k = tid; k < n_splits * (CD / 2); k += NT) {
            const int64_t sp = k / (CD / 2), j = k - sp * (CD / 2);
            cp_async<8>(smem_u32(xs_s + sp * CD + 2 * j), cb + sp * stride + 2 * j);
        }
        cp_async_commit();
    } else {
#pragma unroll
        for (int i = 0; i < XR; ++i) {
            if (s0 + i < s1) {
                ld(xb + (s0 + i) * stride, x[i]);
            } else {
#pragma unroll
                for (int c = 0; c < DL; ++c)
                    x[i][c] = 0.0f;
            }
        }
    }

    float mx = -FLT_MAX;
    int bad = 0;
    for (int64_t s = tid; s < n_splits; s += NT) {
        const float2 v = md(s);
        if (cached)
            wd_s[s] = v;
        if (v.y == 0.0f)
            continue;
        if (!isfinite(v.y) || v.y < 0.0f || !isfinite(v.x))
            bad = 1;
        else
            mx = fmaxf(mx, v.x);
    }
    mx = warp_max(mx);
    if (lane == 0)
        red[warp] = mx;
    bad = __syncthreads_or(bad);
    float M = red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w)
        M = fmaxf(M, red[w]);
    __syncthreads();

    float lsum = 0.0f;
    for (int64_t s = tid; s < n_splits; s += NT) {
        const float2 v = cached ? wd_s[s] : md(s);
        const float w = v.y != 0.0f ? expf(v.x - M) : 0.0f;
        if (cached)
            wd_s[s] = make_float2(w, v.y);
        if (v.y != 0.0f)
            lsum += v.y * w;
    }
    lsum = warp_sum(lsum);
    if (lane == 0)
        red[warp] = lsum;
    if constexpr (STG)
        cp_async_wait<0>();
    __syncthreads();
    float L = red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w)
        L += red[w];

    // chk: NaN iff some live numerator is not finite
    float acc[DL], chk[DL];
#pragma unroll
    for (int c = 0; c < DL; ++c)
        acc[c] = chk[c] = 0.0f;
    if constexpr (STG) {
        for (int64_t cs = s0; cs < s1; ++cs) {
            const float2 v = wd_s[cs];
#pragma unroll
            for (int c = 0; c < DL; ++c) {
                const float y = v.y != 0.0f ? xs_s[cs * CD + DL * lane + c] : 0.0f;
                acc[c] = fmaf(y, v.x, acc[c]);
                chk[c] = fmaf(y, 0.0f, chk[c]);
            }
        }
    } else if (cached) {
        for (int64_t cs = s0; cs < s1; cs += XR) {
            if (cs != s0) {
#pragma unroll
                for (int i = 0; i < XR; ++i) {
                    if (cs + i < s1) {
                        ld(xb + (cs + i) * stride, x[i]);
                    } else {
#pragma unroll
                        for (int c = 0; c < DL; ++c)
                            x[i][c] = 0.0f;
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < XR; ++i) {
                if (cs + i < s1) {
                    const float2 v = wd_s[cs + i];
#pragma unroll
                    for (int c = 0; c < DL; ++c) {
                        const float y = v.y != 0.0f ? x[i][c] : 0.0f;
                        acc[c] = fmaf(y, v.x, acc[c]);
                        chk[c] = fmaf(y, 0.0f, chk[c]);
                    }
                }
            }
        }
    } else {
        // more splits than the shared-memory cache: weights recomputed per split
        for (int64_t cs = s0; cs < s1; ++cs) {
            const float2 v = md(cs);
            const float w = v.y != 0.0f ? expf(v.x - M) : 0.0f;
            float xv[DL];
            ld(xb + cs * stride, xv);
#pragma unroll
            for (int c = 0; c < DL; ++c) {
                const float y = v.y != 0.0f ? xv[c] : 0.0f;
                acc[c] = fmaf(y, w, acc[c]);
                chk[c] = fmaf(y, 0.0f, chk[c]);
            }
        }
    }
    bool nonfinite = false;
#pragma unroll
    for (int c = 0; c < DL; ++c) {
        accw[warp][DL * lane + c] = acc[c];
        nonfinite = nonfinite || !isfinite(chk[c]);
    }
    bad |= __syncthreads_or(nonfinite);

    float o[DL], l = 0.0f;
#pragma unroll
    for (int c = 0; c < DL; ++c)
        o[c] = 0.0f;
    if (warp == 0) {
#pragma unroll
        for (int c = 0; c < DL; ++c) {
            o[c] = accw[0][DL * lane + c];
#pragma unroll
            for (int w = 1; w < NW; ++w)
                o[c] += accw[w][DL * lane + c];
        }
        // the sink joins as one more split of weight exp(sink - M)
        if (sinks) {
            const float sk = sinks[row % n_head];
            if (L == 0.0f || sk > M) {
                const float ms = L == 0.0f ? 0.0f : expf(M - sk);
#pragma unroll
                for (int c = 0; c < DL; ++c)
                    o[c] *= ms;
                L = L * ms + 1.0f;
                M = sk;
            } else {
                L += expf(sk - M);
            }
        }
        const float inv = L == 0.0f ? 0.0f : 1.0f / L;
        l = L == 0.0f ? -INFINITY : M + logf(L);
        bool rowbad = !isfinite(L) || L < 0.0f || !isfinite(inv) || (L != 0.0f && !isfinite(l));
#pragma unroll
        for (int c = 0; c < DL; ++c) {
            o[c] *= inv;
            rowbad = rowbad || !isfinite(o[c]);
        }
        bad |= __any_sync(0xffffffffu, rowbad);
    }
    // push this CTA's flag into slot `chunk` of every CTA of the row
    if (xchg) {
        cluster_wait();
        if (warp == 0 && lane < NC)
            st_peer(&flags_s[chunk], (uint32_t)lane, bad);
        cluster_sync();
    }
    if (warp == 0) {
        int poison = bad;
        if (xchg)
#pragma unroll
            for (int r = 0; r < NC; ++r)
                poison |= flags_s[r];
        float *dst = records ? out + row * (D + 2) : out + row * D;
#pragma unroll
        for (int c = 0; c < DL; ++c)
            dst[d + c] = poison ? NAN : o[c];
        if (chunk == 0 && lane == 0) {
            if (records) {
                dst[D] = poison ? NAN : (L == 0.0f ? -FLT_MAX : l);
                dst[D + 1] = poison ? NAN : (L == 0.0f ? 0.0f : 1.0f);
            } else if (lse) {
                lse[row] = poison ? NAN : l;
            }
        }
    }
}


// Merge for many rows with few splits each (e.g. the per-group merges of a
// KV-sharded step): one warp per merged row, lane l owning dims l + 32 j, and
// the splits taken 32 at a time (lane s holds split c + s's max and
// denominator and broadcasts its weight).  Numerators are added in split order
// per dim; the row's poison flag stays inside the warp.  Same inputs, outputs
// and record mode as lse_merge_kernel.
template <int D>
__global__ void __launch_bounds__(256) lse_merge_rows_kernel(const float *__restrict__ part,
                                                             int64_t n_splits, int64_t n_rows,
                                                             int64_t n_total,
                                                             float *__restrict__ out,
                                                             float *__restrict__ lse,
                                                             const float *__restrict__ sinks,
                                                             int n_head, int records) {
    constexpr int J = D / 32, SB = 8;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); // warp-uniform
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    mg::grid_dep_wait();
    if (row >= n_total)
        return;
    const int64_t grp = row / n_rows, grow = row - grp * n_rows;
    const int64_t stride = (int64_t)n_rows * (D + 2);
    const float *base = part + grp * n_splits * stride + grow * (D + 2);

    float M = -FLT_MAX;
    int bad = 0;
    for (int64_t c = 0; c < n_splits; c += 32) {
        const int64_t sp = c + lane;
        if (sp < n_splits) {
            const float m = base[sp * stride + D], den = base[sp * stride + D + 1];
            if (den != 0.0f) {
                if (!isfinite(den) || den < 0.0f || !isfinite(m))
                    bad = 1;
                else
                    M = fmaxf(M, m);
            }
        }
    }
    M = warp_max(M);
    float lp = 0.0f;
    for (int64_t c = 0; c < n_splits; c += 32) {
        const int64_t sp = c + lane;
        if (sp < n_splits) {
            const float m = base[sp * stride + D], den = base[sp * stride + D + 1];
            if (den != 0.0f)
                lp += den * expf(m - M);
        }
    }
    float L = warp_sum(lp);

    float acc[J], chk = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
        acc[j] = 0.0f;
    for (int64_t c = 0; c < n_splits; c += 32) {
        const int64_t sp = c + lane;
        float wl = 0.0f, dl = 0.0f;
        if (sp < n_splits) {
            dl = base[sp * stride + D + 1];
            wl = dl != 0.0f ? expf(base[sp * stride + D] - M) : 0.0f;
        }
        const int nc = (int)min((int64_t)32, n_splits - c);
        for (int s0 = 0; s0 < nc; s0 += SB) {
            float x[SB][J];
#pragma unroll
            for (int i = 0; i < SB; ++i)
#pragma unroll
                for (int j = 0; j < J; ++j)
                    x[i][j] = s0 + i < nc ? base[(c + s0 + i) * stride + lane + 32 * j] : 0.0f;
#pragma unroll
            for (int i = 0; i < SB; ++i) {
                const float w = __shfl_sync(0xffffffffu, wl, (s0 + i) & 31);
                const float dn = __shfl_sync(0xffffffffu, dl, (s0 + i) & 31);
                if (s0 + i < nc && dn != 0.0f) {
#pragma unroll
                    for (int j = 0; j < J; ++j) {
                        acc[j] = fmaf(x[i][j], w, acc[j]);
                        chk = fmaf(x[i][j], 0.0f, chk);
                    }
                }
            }
        }
    }
    if (!records && sinks) {
        const float sk = sinks[grow % n_head];
        if (L == 0.0f || sk > M) {
            const float ms = L == 0.0f ? 0.0f : expf(M - sk);
#pragma unroll
            for (int j = 0; j < J; ++j)
                acc[j] *= ms;
            L = L * ms + 1.0f;
            M = sk;
        } else {
            L += expf(sk - M);
        }
    }
    const float inv = L == 0.0f ? 0.0f : 1.0f / L;
    const float l = L == 0.0f ? -INFINITY : M + logf(L);
    bool rowbad = bad || !isfinite(chk) || !isfinite(L) || L < 0.0f || !isfinite(inv) ||
                  (L != 0.0f && !isfinite(l));
#pragma unroll
    for (int j = 0; j < J; ++j) {
        acc[j] *= inv;
        rowbad |= !isfinite(acc[j]);
    }
    const bool poison = __any_sync(0xffffffffu, rowbad);
    if (records) {
        float *rec = out + row * (D + 2);
#pragma unroll
        for (int j = 0; j < J; ++j)
            rec[lane + 32 * j] = poison ? NAN : acc[j];
        if (lane == 0) {
            rec[D] = poison ? NAN : (L == 0.0f ? -FLT_MAX : l);
            rec[D + 1] = poison ? NAN : (L == 0.0f ? 0.0f : 1.0f);
        }
    } else {
#pragma unroll
        for (int j = 0; j < J; ++j)
            out[row * D + lane + 32 * j] = poison ? NAN : acc[j];
        if (lse && lane == 0)
            lse[row] = poison ? NAN : l;
    }
}

// The same merge with four warps per row (two rows per CTA): warp w of a row
// owns dims [w D/4, (w+1) D/4), D/128 adjacent dims per lane, and requests
// the numerators of 32 splits at once before adding them.  Every warp forms
// the row's max, denominator and weights itself in the same order as the
// one-warp kernel, and every dim is added over the splits in split order, so
// the outputs are bit-identical to lse_merge_rows_kernel's; the row's poison
// flag is OR-ed across its four warps in shared memory.  D = 128 or 256
// (D = 256 loads 8-byte pairs: partials 8-byte aligned).
template <int D>
__global__ void __launch_bounds__(256) lse_merge_rows4_kernel(const float *__restrict__ part,
                                                              int64_t n_splits, int64_t n_rows,
                                                              int64_t n_total,
                                                              float *__restrict__ out,
                                                              float *__restrict__ lse,
                                                              const float *__restrict__ sinks,
                                                              int n_head, int records) {
    constexpr int DPL = D / 128; // dims per lane
    static_assert(DPL == 1 || DPL == 2, "D = 128 or 256");
    __shared__ int bad_s[2];
    const int lane = threadIdx.x & 31, wr = (threadIdx.x >> 5) & 3, rs = threadIdx.x >> 7;
    const int64_t row = (int64_t)blockIdx.x * 2 + rs;
    const bool live = row < n_total;
    if (threadIdx.x < 2)
        bad_s[threadIdx.x] = 0;
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    mg::grid_dep_wait();
    const int64_t grp = live ? row / n_rows : 0, grow = live ? row - grp * n_rows : 0;
    const int64_t stride = (int64_t)n_rows * (D + 2);
    const float *base = part + grp * n_splits * stride + grow * (D + 2);
    const int d0 = wr * (D / 4) + DPL * lane;

    float M = -FLT_MAX;
    int bad = 0;
    float L = 0.0f;
    float acc[DPL], chk = 0.0f;
#pragma unroll
    for (int j = 0; j < DPL; ++j)
        acc[j] = 0.0f;
    if (live) {
        for (int64_t c = 0; c < n_splits; c += 32) {
            const int64_t sp = c + lane;
            if (sp < n_splits) {
                const float m = base[sp * stride + D], den = base[sp * stride + D + 1];
                if (den != 0.0f) {
                    if (!isfinite(den) || den < 0.0f || !isfinite(m))
                        bad = 1;
                    else
                        M = fmaxf(M, m);
                }
            }
        }
        M = warp_max(M);
        float lp = 0.0f;
        for (int64_t c = 0; c < n_splits; c += 32) {
            const int64_t sp = c + lane;
            if (sp < n_splits) {
                const float m = base[sp * stride + D], den = base[sp * stride + D + 1];
                if (den != 0.0f)
                    lp += den * expf(m - M);
            }
        }
        L = warp_sum(lp);
        for (int64_t c = 0; c < n_splits; c += 32) {
            const int64_t sp = c + lane;
            float wl = 0.0f, dl = 0.0f;
            if (sp < n_splits) {
                dl = base[sp * stride + D + 1];
                wl = dl != 0.0f ? expf(base[sp * stride + D] - M) : 0.0f;
            }
            const int nc = (int)min((int64_t)32, n_splits - c);
            // this lane's numerators of the chunk's splits, all in flight
            float x[32][DPL];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float *p = base + (c + i) * stride + d0;
                if (i < nc) {
                    if constexpr (DPL == 2) {
                        const float2 t = *reinterpret_cast<const float2 *>(p);
                        x[i][0] = t.x;
                        x[i][1] = t.y;
                    } else {
                        x[i][0] = *p;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < DPL; ++j)
                        x[i][j] = 0.0f;
                }
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float w = __shfl_sync(0xffffffffu, wl, i);
                const float dn = __shfl_sync(0xffffffffu, dl, i);
                if (i < nc && dn != 0.0f) {
#pragma unroll
                    for (int j = 0; j < DPL; ++j) {
                        acc[j] = fmaf(x[i][j], w, acc[j]);
                        chk = fmaf(x[i][j], 0.0f, chk);
                    }
                }
            }
        }
        if (!records && sinks) {
            const float sk = sinks[grow % n_head];
            if (L == 0.0f || sk > M) {
                const float ms = L == 0.0f ? 0.0f : expf(M - sk);
#pragma unroll
                for (int j = 0; j < DPL; ++j)
                    acc[j] *= ms;
                L = L * ms + 1.0f;
                M = sk;
            } else {
                L += expf(sk - M);
            }
        }
    }
    const float inv = L == 0.0f ? 0.0f : 1.0f / L;
    const float l = L == 0.0f ? -INFINITY : M + logf(L);
    bool rowbad = bad || !isfinite(chk) || !isfinite(L) || L < 0.0f || !isfinite(inv) ||
                  (L != 0.0f && !isfinite(l));
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
        acc[j] *= inv;
        rowbad |= !isfinite(acc[j]);
    }
    if (__any_sync(0xffffffffu, rowbad) && lane == 0)
        atomicOr(&bad_s[rs], 1);
    __syncthreads();
    if (!live)
        return;
    const bool poison = bad_s[rs] != 0;
    if (records) {
        float *rec = out + row * (D + 2);
#pragma unroll
        for (int j = 0; j < DPL; ++j)
            rec[d0 + j] = poison ? NAN : acc[j];
        if (wr == 0 && lane == 0) {
            rec[D] = poison ? NAN : (L == 0.0f ? -FLT_MAX : l);
            rec[D + 1] = poison ? NAN : (L == 0.0f ? 0.0f : 1.0f);
        }
    } else {
#pragma unroll
        for (int j = 0; j < DPL; ++j)
            out[row * D + d0 + j] = poison ? NAN : acc[j];
        if (lse && wr == 0 && lane == 0)
            lse[row] = poison ? NAN : l;
    }
}

// ---------------------------------------------------------------------------
// Host side: configuration and launch.

template <int T, int D, int NR, int R, int VW>
static cudaError_t launch_one(const DecodeArgs &a, size_t smem, dim3 grid, cudaStream_t st) {
    auto kern = fa_decode_kernel<T, D, NR, R, VW>;
    static std::atomic<unsigned long long> attr_done{0};
    cudaError_t e = set_smem_limit((const void *)kern, smem, attr_done);
    if (e != cudaSuccess)
        return e;
    kern<<<grid, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

static size_t decode_smem(int type, int D, int NR, int R) {
    const int SS = smem_stride(rec_bytes(type, D));
    size_t b = (size_t)4 * R * SS;                   // K, V x 2 stages
    b += (size_t)NR * D * 4 + (size_t)R * NR * 4;     // q, p
    b += (size_t)(kThreads / 32) * NR * 4 + 4 * NR * 4; // red, m, l, alpha, slope
    b += (size_t)NR * 8 + (size_t)NR * 4;             // mask offsets, limits
    const size_t ob = (size_t)NR * D * 4;             // epilogue aliases K stages
    if (ob > (size_t)2 * R * SS)
        b += ob;
    return b;
}

bool decode_config(int type, int D, int n_qrows, const DecodeArgs &a, DecodeConfig *cfg) {
    if (type != kF16 && type != kQ8 && type != kQ4)
        return false;
    if (D != 64 && D != 128 && D != 256)
        return false;
    cfg->type = type;
    cfg->D = D;
    cfg->NR = n_qrows <= 4 ? 4 : n_qrows <= 8 ? 8 : 16;
    cfg->R = smem_stride(rec_bytes(type, D)) > 288 ? 32 : 64;
    // widest cp.async that every row start and the row length allow
    const uint64_t rec = (uint64_t)rec_bytes(type, D);
    const uint64_t align = (uint64_t)(uintptr_t)a.k | (uint64_t)(uintptr_t)a.v |
                           (uint64_t)a.k_nb1 | (uint64_t)a.k_nb2 | (uint64_t)a.k_nb3 |
                           (uint64_t)a.v_nb1 | (uint64_t)a.v_nb2 | (uint64_t)a.v_nb3 | rec;
    cfg->VW = (align % 16 == 0) ? 16 : (align % 8 == 0) ? 8 : (align % 4 == 0) ? 4 : 0;
    if (!cfg->VW)
        return false;
    cfg->smem = decode_smem(type, D, cfg->NR, cfg->R);
    return true;
}

template <int T, int D, int NR, int R>
static cudaError_t dispatch_vw(const DecodeArgs &a, const DecodeConfig &c, dim3 g,
                               cudaStream_t st) {
    if constexpr (rec_bytes(T, D) % 16 == 0)
        if (c.VW == 16)
            return launch_one<T, D, NR, R, 16>(a, c.smem, g, st);
    if constexpr (rec_bytes(T, D) % 8 == 0)
        if (c.VW >= 8)
            return launch_one<T, D, NR, R, 8>(a, c.smem, g, st);
    return launch_one<T, D, NR, R, 4>(a, c.smem, g, st);
}

template <int T, int D>
static cudaError_t dispatch_nr(const DecodeArgs &a, const DecodeConfig &c, dim3 g,
                               cudaStream_t st) {
    constexpr int R = smem_stride(rec_bytes(T, D)) > 288 ? 32 : 64;
    switch (c.NR) {
    case 4: return dispatch_vw<T, D, 4, R>(a, c, g, st);
    case 8: return dispatch_vw<T, D, 8, R>(a, c, g, st);
    default: return dispatch_vw<T, D, 16, R>(a, c, g, st);
    }
}

template <int T>
static cudaError_t dispatch_d(const DecodeArgs &a, const DecodeConfig &c, dim3 g,
                              cudaStream_t st) {
    switch (c.D) {
    case 64: return dispatch_nr<T, 64>(a, c, g, st);
    case 128: return dispatch_nr<T, 128>(a, c, g, st);
    default: return dispatch_nr<T, 256>(a, c, g, st);
    }
}

cudaError_t launch_decode(const DecodeArgs &a, const DecodeConfig &c, dim3 grid,
                          cudaStream_t st) {
    switch (c.type) {
    case kF16: return dispatch_d<kF16>(a, c, grid, st);
    case kQ8: return dispatch_d<kQ8>(a, c, grid, st);
    default: return dispatch_d<kQ4>(a, c, grid, st);
    }
}

// SM count of the current device, queried once per device (0 if unknown).
static int merge_sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return 0;
    if (dev >= 0 && dev < 64 && (n = cache[dev].load(std::memory_order_relaxed)) > 0)
        return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return 0;
    if (dev >= 0 && dev < 64)
        cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

cudaError_t launch_merge(const float *partials, int64_t n_splits, int64_t n_rows, int D,
                         float *out, float *lse, const float *sinks, int n_head,
                         cudaStream_t st, int64_t n_groups, bool records, bool flagged) {
    if (n_rows <= 0 || n_groups <= 0)
        return cudaSuccess;
    if (n_groups * n_rows * (D / 32) > 0x7fffffff)
        return cudaErrorInvalidValue;
    const int64_t total = n_groups * n_rows;
    if (total >= 128 || records) {
        // enough rows to fill the GPU with one warp each -- and every record
        // merge, whatever its row count: a record must come out of the same
        // kernel (the same summation order) however the groups are spread
        // over GPUs, or the merged result would depend on the GPU count
        void (*rk)(const float *, int64_t, int64_t, int64_t, float *, float *, const float *,
                   int, int);
        // four warps per row (every numerator of 32 splits in flight at once)
        // when the rows fit one wave at one CTA per SM: the per-GPU group
        // merge of an 8-GPU config-5 step (32 splits x 192 rows) 7.3 -> 4.2
        // us; for more rows the memory traffic sets the time and one warp per
        // row at higher occupancy is faster (all 8 groups on one GPU: 10.9
        // against 20.8 us).  The same sums either way.
        const int sms = merge_sm_count();
        const bool four = (D == 128 || (D == 256 && ((uintptr_t)partials & 7) == 0)) &&
                          (total + 1) / 2 <= sms;
        switch (D) {
        case 64: rk = lse_merge_rows_kernel<64>; break;
        case 128: rk = four ? lse_merge_rows4_kernel<128> : lse_merge_rows_kernel<128>; break;
        case 256: rk = four ? lse_merge_rows4_kernel<256> : lse_merge_rows_kernel<256>; break;
        default: return cudaErrorInvalidValue;
        }
        cudaLaunchConfig_t rc = {};
        rc.gridDim = dim3((unsigned)(four ? (total + 1) / 2 : (total + 7) / 8), 1, 1);
        rc.blockDim = dim3(256, 1, 1);
        rc.stream = st;
        cudaLaunchAttribute ra[1];
        ra[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        ra[0].val.programmaticStreamSerializationAllowed = 1;
        rc.attrs = ra;
        rc.numAttrs = 1;
        return cudaLaunchKernelEx(&rc, rk, partials, n_splits, n_rows, total, out, lse, sinks,
                                  n_head, records ? 1 : 0);
    }
    void (*kern)(const float *, int64_t, int64_t, float *, float *, const float *, int, int,
                 int);
    // two dims per lane (8-byte loads) where the records allow it: half the
    // CTAs per row, the same sums (config 2: 15.8 -> 14.9 us a step, while
    // the merge timed on its own did not change)
    const int dl = D >= 128 && ((uintptr_t)partials & 7) == 0 ? 2 : 1;
    // numerators staged in shared memory (32 registers, no array in flight):
    // config 1 11.3 -> 10.1 us a step, kv4 28.6 -> 26.9 us.  At D = 256 the
    // CTA reserves mg::STG_PAD bytes so that it never shares an SM with two
    // Q8_0 / Q4_0 decode CTAs (77-81 KB each): sharing made config 2's step
    // slower (14.9 -> 16.4 us) although the merge alone was faster.  Same sums
    // in every variant.
    const size_t stg_bytes = (size_t)n_splits * 64 * sizeof(float);
    bool stg = dl == 2 && stg_bytes <= mg::STG_CAP;
    if (stg && D == 256) {
        // the reservation leaves one merge CTA per SM: staged only where the
        // whole grid fits in one wave (the register path holds two per SM)
        stg = n_groups * n_rows * (D / 64) <= merge_sm_count();
    }
    const size_t stg_dyn = D == 256 ? mg::STG_PAD : stg_bytes;
    switch (D * 4 + dl) {
    case 64 * 4 + 1: kern = lse_merge_kernel<64, 1, false>; break;
    case 128 * 4 + 1: kern = lse_merge_kernel<128, 1, false>; break;
    case 256 * 4 + 1: kern = lse_merge_kernel<256, 1, false>; break;
    case 128 * 4 + 2:
        kern = stg ? lse_merge_kernel<128, 2, true> : lse_merge_kernel<128, 2, false>;
        break;
    case 256 * 4 + 2:
        kern = stg ? lse_merge_kernel<256, 2, true> : lse_merge_kernel<256, 2, false>;
        break;
    default: return cudaErrorInvalidValue;
    }
    if (stg) {
        static std::atomic<unsigned long long> stg_attr[2];
        const cudaError_t e = set_smem_limit((const void *)kern, mg::STG_PAD, stg_attr[D == 256]);
        if (e != cudaSuccess)
            return e;
    }
    const int nc = D / (32 * dl);
    // one cluster of nc CTAs per row (exchanging the row's poison flag), or,
    // for records whose producer marks poisoned numerators in their
    // denominators (`flagged`), nc independent CTAs; launched as a
    // programmatic dependent of the kernel before it on the stream (the merge
    // waits for it in-kernel)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n_groups * n_rows * nc), 1, 1);
    cfg.blockDim = dim3(mg::NT, 1, 1);
    cfg.dynamicSmemBytes = stg ? stg_dyn : 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)nc;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = flagged ? 1 : 2;
    return cudaLaunchKernelEx(&cfg, kern, partials, n_splits, n_rows, out, lse, sinks, n_head,
                              records ? 1 : 0, flagged ? 0 : 1);
}

} // namespace xq
