// GATED_DELTA_NET, recurrent form (any T, K rollback slots, n_seq >= 1).
//
// Per (sequence, value head h) with state S[col][i] (col = value dim, i = key
// dim), for each token t (ggml-cpu GATED_DELTA_NET; the fork's host mirror
// src/bridge/ggml_d3d12.cpp:113-158 and shaders/ggml_d3d12_gated_delta_net.hlsl:40-86):
//   S   <- exp(g_t) * S
//   d   =  (v_t[col] - sum_i S[col][i] k_t[i]) * beta_t
//   S[col][:] += k_t * d
//   y_t[col] = (sum_i S[col][i] q_t[i]) / sqrt(S_k)
// with key head h % H_k.  Columns are independent, so a CTA owns CB columns
// of one (sequence, head) and keeps them in registers for all T tokens.  This
// bit-comparable kernel serves short sequences (decode, T <= 8); longer ones
// go to gdn_stream_kernel below.  Eight
// lanes share a column; lane l holds elements i = l + 8e, accumulates its
// partial dot in increasing i and the eight partials meet in the tree
// (l, l+4), (l, l+2), (l, l+1) -- the order of the reference mirror's
// eight-lane reduction -- with explicit round-to-nearest multiplies and adds
// (no FMA contraction).  exp(g) is evaluated in double and rounded once.
#include "xq_common.cuh"
#include "xq_internal.h"

namespace xq {

template <int S, int CB>
__global__ void __launch_bounds__(CB * 8) gdn_recurrent_kernel(const GdnArgs a) {
    constexpr int TPC = 8;       // lanes per column
    constexpr int EPT = S / TPC; // elements per lane
    const int unit = blockIdx.x;
    const int h = unit % a.H, seq = unit / a.H;
    const int col = blockIdx.y * CB + threadIdx.x / TPC;
    const int l = threadIdx.x % TPC;
    const int hk = (h + a.h_off) % a.H_k;
    const int sq = seq / a.rq3, sk = seq / a.rk3;

    const char *st_row = reinterpret_cast<const char *>(a.state) + seq * a.s_nb3 +
                         (int64_t)h * a.s_nb2 + (int64_t)col * a.s_nb1;
    // Launched as a programmatic dependent: the next kernel may launch now (it
    // waits for this grid before it reads what this one writes); until
    // griddepcontrol.wait the kernel before this one may still be writing the
    // state and the token inputs, so only an L2 prefetch of this CTA's state
    // rows (contiguous, no data consumed) comes first.
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    if (threadIdx.x == 0) {
        const char *rows = st_row - (int64_t)(threadIdx.x / TPC) * a.s_nb1;
        if (a.s_nb1 == 4 * S && ((reinterpret_cast<uintptr_t>(rows)) & 15) == 0)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(rows),
                         "r"((uint32_t)(CB * 4 * S))
                         : "memory");
    }
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    float st[EPT];
#pragma unroll
    for (int e = 0; e < EPT; ++e)
        st[e] = reinterpret_cast<const float *>(st_row)[l + TPC * e];

    const size_t slot_elems = (size_t)S * S * a.H * a.n_seq;
    float *snap = a.dst + (size_t)S * a.H * a.T * a.n_seq;
    const size_t snap_off = ((size_t)(seq * a.H + h) * S + col) * S;

    auto ptr = [](const float *base, int64_t o) {
        return reinterpret_cast<const float *>(reinterpret_cast<const char *>(base) + o);
    };
    const float *qb = ptr(a.q, sq * a.q_nb3 + hk * a.q_nb1);
    const float *kb = ptr(a.k, sk * a.k_nb3 + hk * a.k_nb1);
    const float *vb = ptr(a.v, seq * a.v_nb3 + h * a.v_nb1);
    const float *gb = ptr(a.g, seq * a.g_nb3 + h * a.g_nb1);
    const float *bb = ptr(a.beta, seq * a.b_nb3 + h * a.b_nb1);

    for (int t = a.t_begin; t < a.T; ++t) {
        const float *qt = ptr(qb, (int64_t)t * a.q_nb2);
        const float *kt = ptr(kb, (int64_t)t * a.k_nb2);
        float kx[EPT], qx[EPT];
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            kx[e] = __ldg(kt + l + TPC * e);
            qx[e] = __ldg(qt + l + TPC * e);
        }
        const float vv = __ldg(ptr(vb, (int64_t)t * a.v_nb2) + col);
        const float beta = __ldg(ptr(bb, (int64_t)t * a.b_nb2));
        const float decay = (float)exp((double)__ldg(ptr(gb, (int64_t)t * a.g_nb2)));

        float kv = 0.0f;
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            st[e] = __fmul_rn(st[e], decay);
            kv = __fadd_rn(kv, __fmul_rn(st[e], kx[e]));
        }
        kv = __fadd_rn(kv, __shfl_xor_sync(0xffffffffu, kv, 4));
        kv = __fadd_rn(kv, __shfl_xor_sync(0xffffffffu, kv, 2));
        kv = __fadd_rn(kv, __shfl_xor_sync(0xffffffffu, kv, 1));
        const float delta = __fmul_rn(__fsub_rn(vv, kv), beta);
        float at = 0.0f;
#pragma unroll
        for (int e = 0; e < EPT; ++e) {
            st[e] = __fadd_rn(st[e], __fmul_rn(kx[e], delta));
            at = __fadd_rn(at, __fmul_rn(st[e], qx[e]));
        }
        at = __fadd_rn(at, __shfl_xor_sync(0xffffffffu, at, 4));
        at = __fadd_rn(at, __shfl_xor_sync(0xffffffffu, at, 2));
        at = __fadd_rn(at, __shfl_xor_sync(0xffffffffu, at, 1));
        if (l == 0)
            a.dst[((size_t)(seq * a.T + t) * a.H + h) * S + col] = __fmul_rn(at, a.scale);

        const int slot = a.T - 1 - t;
        if ((a.slots > 1 && slot < a.slots) || (a.slots == 1 && t + 1 == a.T)) {
            float *o = snap + (size_t)(a.slots == 1 ? 0 : slot) * slot_elems + snap_off;
#pragma unroll
            for (int e = 0; e < EPT; ++e)
                o[l + TPC * e] = st[e];
        }
    }
}

// Long sequences (T > 8): the same recurrence, the token inputs staged through
// shared memory 16 tokens at a time (double-buffered cp.async), and the
// arithmetic reorganised for issue rate instead of the reference mirror's
// lane order: lane l of a column's TPC lanes owns key elements
// 4l + 4 TPC j + {0..3} (so each input vector arrives as conflict-free
// 16-byte shared loads), dot products are packed FP32x2 FMAs, the decay is applied
// to the reduced dot product (S k after the decay equals decay * (S k)) and
// fused into the state update S = S * decay + k * delta, and a token's output
// dot (q_t . S_t) and the next token's (k_{t+1} . S_t) share one shuffle tree.
// Results agree with the sequential reference to float rounding, not bit for
// bit.
template <int S, int CB, int VW, int TPC>
__global__ void __launch_bounds__(CB * TPC) gdn_stream_kernel(const GdnArgs a) {
    constexpr int NT = CB * TPC;
    constexpr int J = S / (4 * TPC); // float4 groups of key elements per lane
    static_assert(TPC == 8 || TPC == 16, "lanes per column");
    constexpr int TC = 16;      // tokens per staged chunk
    constexpr int PR = S * 4 / VW;
    static_assert(S == 128, "element ownership assumes 128-long rows");
    __shared__ __align__(16) float k_s[2][TC][S];
    __shared__ __align__(16) float q_s[2][TC][S];
    __shared__ __align__(16) float v_s[2][TC][CB];
    __shared__ float g_s[2][TC], b_s[2][TC], d_s[2][TC];
    const int tid = threadIdx.x;
    const int h = blockIdx.x % a.H, seq = blockIdx.x / a.H;
    const int col0 = blockIdx.y * CB, cc = tid / TPC, col = col0 + cc;
    const int l = tid % TPC;
    const int hk = (h + a.h_off) % a.H_k;
    const int sq = seq / a.rq3, sk = seq / a.rk3;

    // state row `col`, elements 4l + 4 TPC j + x held as float2 pairs st[2j], st[2j+1]
    const float *st_row = reinterpret_cast<const float *>(
        reinterpret_cast<const char *>(a.state) + seq * a.s_nb3 + (int64_t)h * a.s_nb2 +
        (int64_t)col * a.s_nb1);
    float2 st[2 * J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int e = 4 * l + 4 * TPC * j;
        st[2 * j] = make_float2(st_row[e], st_row[e + 1]);
        st[2 * j + 1] = make_float2(st_row[e + 2], st_row[e + 3]);
    }
    const size_t slot_elems = (size_t)S * S * a.H * a.n_seq;
    float *snap = a.dst + (size_t)S * a.H * a.T * a.n_seq;
    const size_t snap_off = ((size_t)(seq * a.H + h) * S + col) * S;

    auto ptr = [](const float *base, int64_t o) {
        return reinterpret_cast<const float *>(reinterpret_cast<const char *>(base) + o);
    };
    const float *qb = ptr(a.q, sq * a.q_nb3 + hk * a.q_nb1);
    const float *kb = ptr(a.k, sk * a.k_nb3 + hk * a.k_nb1);
    const float *vb = ptr(a.v, seq * a.v_nb3 + h * a.v_nb1);
    const float *gb = ptr(a.g, seq * a.g_nb3 + h * a.g_nb1);
    const float *bb = ptr(a.beta, seq * a.b_nb3 + h * a.b_nb1);

    auto stage = [&](int c, int buf) {
        const int t0 = a.t_begin + c * TC, nt = min(TC, a.T - t0);
        for (int idx = tid; idx < TC * PR; idx += NT) {
            const int r = idx / PR, pc = idx - r * PR;
            if (r < nt) {
                cp_async<VW>(smem_u32(&k_s[buf][r][0]) + pc * VW,
                             reinterpret_cast<const char *>(ptr(kb, (int64_t)(t0 + r) * a.k_nb2)) +
                                 pc * VW);
                cp_async<VW>(smem_u32(&q_s[buf][r][0]) + pc * VW,
                             reinterpret_cast<const char *>(ptr(qb, (int64_t)(t0 + r) * a.q_nb2)) +
                                 pc * VW);
            }
        }
        for (int idx = tid; idx < TC * CB; idx += NT) {
            const int r = idx / CB, c2 = idx - r * CB;
            if (r < nt)
                cp_async<4>(smem_u32(&v_s[buf][r][c2]), ptr(vb, (int64_t)(t0 + r) * a.v_nb2) +
                                                            col0 + c2);
        }
        if (tid < nt) {
            cp_async<4>(smem_u32(&g_s[buf][tid]), ptr(gb, (int64_t)(t0 + tid) * a.g_nb2));
            cp_async<4>(smem_u32(&b_s[buf][tid]), ptr(bb, (int64_t)(t0 + tid) * a.b_nb2));
        }
        cp_async_commit();
    };
    const int n_chunks = (a.T - a.t_begin + TC - 1) / TC;
    stage(0, 0);
    stage(1, 1);
    for (int c = 0; c < n_chunks; ++c) {
        const int buf = c & 1, t0 = a.t_begin + c * TC, nt = min(TC, a.T - t0);
        cp_async_wait<1>(); // chunk c has landed (chunk c + 1 may be in flight)
        __syncthreads();
        if (tid < nt)
            d_s[buf][tid] = (float)exp((double)g_s[buf][tid]);
        __syncthreads();
        // software pipeline over the chunk: the dot products of token r's
        // updated state with q_r (its output) and with k_{r+1} (the next
        // token's delta) share one interleaved shuffle tree
        auto dot = [&](const float4 (&x)[J]) {
            float2 p0 = make_float2(0.0f, 0.0f), p1 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < J; ++j) {
                p0 = __ffma2_rn(st[2 * j], make_float2(x[j].x, x[j].y), p0);
                p1 = __ffma2_rn(st[2 * j + 1], make_float2(x[j].z, x[j].w), p1);
            }
            return (p0.x + p0.y) + (p1.x + p1.y);
        };
        auto load = [&](float4 (&x)[J], const float (*rows)[S], int r) {
#pragma unroll
            for (int j = 0; j < J; ++j)
                x[j] = *reinterpret_cast<const float4 *>(&rows[r][4 * l + 4 * TPC * j]);
        };
        float4 kcur[J];
        load(kcur, k_s[buf], 0);
        float kvp = dot(kcur); // S_{t0-1} . k_{t0}, reduced below
#pragma unroll
        for (int o = TPC / 2; o > 0; o >>= 1)
            kvp += __shfl_xor_sync(0xffffffffu, kvp, o);
        auto step = [&](int r) {
            const int t = t0 + r;
            float4 qx[J], knext[J];
            load(qx, q_s[buf], r);
            load(knext, k_s[buf], r + 1 < nt ? r + 1 : r);
            const float vv = v_s[buf][r][cc], beta = b_s[buf][r], decay = d_s[buf][r];
            const float delta = (vv - kvp * decay) * beta;
            const float2 d2 = make_float2(decay, decay), dl2 = make_float2(delta, delta);
#pragma unroll
            for (int j = 0; j < J; ++j) {
                st[2 * j] = __ffma2_rn(make_float2(kcur[j].x, kcur[j].y), dl2,
                                       __fmul2_rn(st[2 * j], d2));
                st[2 * j + 1] = __ffma2_rn(make_float2(kcur[j].z, kcur[j].w), dl2,
                                           __fmul2_rn(st[2 * j + 1], d2));
            }
            float at = dot(qx), kn = dot(knext);
#pragma unroll
            for (int o = TPC / 2; o > 0; o >>= 1) {
                at += __shfl_xor_sync(0xffffffffu, at, o);
                kn += __shfl_xor_sync(0xffffffffu, kn, o);
            }
            kvp = kn;
#pragma unroll
            for (int j = 0; j < J; ++j)
                kcur[j] = knext[j];
            if (l == 0)
                a.dst[((size_t)(seq * a.T + t) * a.H + h) * S + col] = at * a.scale;

            const int slot = a.T - 1 - t;
            if ((a.slots > 1 && slot < a.slots) || (a.slots == 1 && t + 1 == a.T)) {
                float *o = snap + (size_t)(a.slots == 1 ? 0 : slot) * slot_elems + snap_off;
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    const int e = 4 * l + 4 * TPC * j;
                    o[e] = st[2 * j].x;
                    o[e + 1] = st[2 * j].y;
                    o[e + 2] = st[2 * j + 1].x;
                    o[e + 3] = st[2 * j + 1].y;
                }
            }
        };
        if (nt == TC) {
#pragma unroll
            for (int r = 0; r < TC; ++r)
                step(r);
        } else {
            for (int r = 0; r < nt; ++r)
                step(r);
        }
        __syncthreads(); // buffer buf is free again
        stage(c + 2, buf);
    }
    cp_async_wait<0>();
}

cudaError_t launch_gdn(const GdnArgs &a, cudaStream_t st) {
    constexpr int S = 128, CB = 16;
    dim3 grid((unsigned)(a.H * a.n_seq), S / CB);
    // 16-byte staging when every q / k row starts on a 16-byte boundary
    const bool v16 = ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                       (uintptr_t)a.q_nb1 | (uintptr_t)a.q_nb2 | (uintptr_t)a.q_nb3 |
                       (uintptr_t)a.k_nb1 | (uintptr_t)a.k_nb2 | (uintptr_t)a.k_nb3) &
                      15) == 0;
    // a few tokens (decode, speculative verify): the reference mirror's exact
    // lane order; longer sequences: the staged, packed-FMA stream kernel
    if (a.T <= 8) {
        // programmatic dependent of the previous kernel on the stream (see the
        // kernel's griddepcontrol.wait)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(CB * 8, 1, 1);
        cfg.stream = st;
        cudaLaunchAttribute pdl[1];
        pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        pdl[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = pdl;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, gdn_recurrent_kernel<S, CB>, a);
    } else {
        // 8 lanes per value column, 16 columns per CTA (16 lanes per column
        // measured slower: the extra shuffle level outweighs the extra warps)
        constexpr int SC = 16, TPC = 8;
        dim3 sgrid((unsigned)(a.H * a.n_seq), S / SC);
        if (v16)
            gdn_stream_kernel<S, SC, 16, TPC><<<sgrid, SC * TPC, 0, st>>>(a);
        else
            gdn_stream_kernel<S, SC, 4, TPC><<<sgrid, SC * TPC, 0, st>>>(a);
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Block codecs (ggml-quants.c reference arithmetic; one thread per 32-block).

template <int T>
__global__ void dequant_kernel(const uint8_t *__restrict__ src, uint64_t ss,
                               float *__restrict__ dst, uint64_t ds, int64_t n_rows,
                               int64_t n_per_row) {
    const int64_t nb = T == kF16 ? n_per_row : n_per_row / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * nb)
        return;
    const int64_t r = i / nb, b = i - r * nb;
    const uint8_t *s = src + r * ss;
    float *d = reinterpret_cast<float *>(reinterpret_cast<char *>(dst) + r * ds);
    if constexpr (T == kF16) {
        d[b] = h2f_bits(*reinterpret_cast<const uint16_t *>(s + 2 * b));
    } else if constexpr (T == kQ8) {
        const uint8_t *blk = s + 34 * b;
        const float sc = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int j = 0; j < 32; ++j)
            d[32 * b + j] = (float)(int)(int8_t)blk[2 + j] * sc;
    } else {
        const uint8_t *blk = s + 18 * b;
        const float sc = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int j = 0; j < 16; ++j) {
            d[32 * b + j] = (float)((int)(blk[2 + j] & 15) - 8) * sc;
            d[32 * b + j + 16] = (float)((int)(blk[2 + j] >> 4) - 8) * sc;
        }
    }
}

// One output unit of the ggml reference quantizers for row x: element b (F32,
// F16) or 32-element block b (Q8_0: quantize_row_q8_0_ref, Q4_0:
// quantize_row_q4_0_ref) written to row y.
template <int T>
__device__ __forceinline__ void quant_block(const float *__restrict__ x, uint8_t *__restrict__ y,
                                            int64_t b) {
    if constexpr (T == kF32) {
        reinterpret_cast<float *>(y)[b] = x[b];
    } else if constexpr (T == kF16) {
        reinterpret_cast<uint16_t *>(y)[b] = __half_as_ushort(__float2half_rn(x[b]));
    } else if constexpr (T == kQ8) {
        const float *xb = x + 32 * b;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j)
            amax = fmaxf(amax, fabsf(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t *blk = y + 34 * b;
        *reinterpret_cast<uint16_t *>(blk) = __half_as_ushort(__float2half_rn(d));
        for (int j = 0; j < 32; ++j)
            blk[2 + j] = (uint8_t)(int8_t)roundf(__fmul_rn(xb[j], id));
    } else {
        const float *xb = x + 32 * b;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            if (amax < fabsf(xb[j])) {
                amax = fabsf(xb[j]);
                vmax = xb[j];
            }
        }
        const float d = vmax / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t *blk = y + 18 * b;
        *reinterpret_cast<uint16_t *>(blk) = __half_as_ushort(__float2half_rn(d));
        for (int j = 0; j < 16; ++j) {
            const int lo = min(15, (int)(int8_t)__fadd_rn(__fmul_rn(xb[j], id), 8.5f));
            const int hi = min(15, (int)(int8_t)__fadd_rn(__fmul_rn(xb[16 + j], id), 8.5f));
            blk[2 + j] = (uint8_t)(lo | (hi << 4));
        }
    }
}

template <int T>
__global__ void quant_kernel(const float *__restrict__ src, uint64_t ss, uint8_t *__restrict__ dst,
                             uint64_t ds, int64_t n_rows, int64_t n_per_row) {
    const int64_t nb = T == kF16 ? n_per_row : n_per_row / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * nb)
        return;
    const int64_t r = i / nb, b = i - r * nb;
    const float *x = reinterpret_cast<const float *>(reinterpret_cast<const char *>(src) + r * ss);
    quant_block<T>(x, dst + r * ds, b);
}

// ggml SET_ROWS (the KV-cache write): source row (i1, i2, i3) of F32 `src`
// goes, converted by the reference quantizer of dst's type, to row
// idx[i1, i2 % idx_ne1, i3 % idx_ne2] of dst (same i2, i3).  One thread per
// output unit; rows whose index falls outside [0, dst_rows) are skipped.
template <int T>
__global__ void set_rows_kernel(const SetRowsArgs a) {
    const int64_t nb = (T == kF16 || T == kF32) ? a.ne0 : a.ne0 / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n_units)
        return;
    const int64_t row = i / nb, b = i - row * nb;
    const int64_t i1 = row % a.ne1, i2 = (row / a.ne1) % a.ne2, i3 = row / (a.ne1 * a.ne2);
    const uint8_t *ip = a.idx + i1 * a.i_nb0 + (i2 % a.i_ne1) * a.i_nb1 + (i3 % a.i_ne2) * a.i_nb2;
    const int64_t dr = a.idx_i64 ? *reinterpret_cast<const int64_t *>(ip)
                                 : (int64_t)*reinterpret_cast<const int32_t *>(ip);
    if (dr < 0 || dr >= a.d_rows)
        return;
    const float *x = reinterpret_cast<const float *>(a.src + i1 * a.s_nb1 + i2 * a.s_nb2 +
                                                     i3 * a.s_nb3);
    quant_block<T>(x, a.dst + dr * a.d_nb1 + i2 * a.d_nb2 + i3 * a.d_nb3, b);
}

// The same for Q8_0 / Q4_0 with 8 lanes per 32-element block: each lane loads
// one float4 (a warp reads 512 contiguous bytes), amax (and Q4_0's signed max,
// the first element of largest magnitude as in the reference loop) meet in a
// 3-level shuffle tree, and the per-element arithmetic is the reference's.
// Needs 16-byte aligned source rows.
// Grid: x over the blocks of one (i2, i3) plane (32-bit: ne1 * ne0 / 32 units),
// z over the planes, so the only per-lane division is unit -> (row, block).
template <int T>
__global__ void __launch_bounds__(256) set_rows_coop_kernel(const SetRowsArgs a) {
    const uint32_t nb = (uint32_t)(a.ne0 / 32);
    const uint32_t plane_units = (uint32_t)a.ne1 * nb;
    const uint32_t unit = (blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int sub = threadIdx.x & 7;
    const bool live = unit < plane_units; // whole 8-lane groups share `live`
    const uint32_t u = live ? unit : 0;
    const uint32_t i1u = u / nb;
    const int64_t i1 = i1u, b = u - i1u * nb;
    const int64_t i2 = blockIdx.z % a.ne2, i3 = blockIdx.z / a.ne2; // uniform
    const uint8_t *ip = a.idx + i1 * a.i_nb0 + (i2 % a.i_ne1) * a.i_nb1 + (i3 % a.i_ne2) * a.i_nb2;
    const int64_t dr = a.idx_i64 ? *reinterpret_cast<const int64_t *>(ip)
                                 : (int64_t)*reinterpret_cast<const int32_t *>(ip);
    const bool store = live && dr >= 0 && dr < a.d_rows;
    const float4 x = *reinterpret_cast<const float4 *>(
        a.src + i1 * a.s_nb1 + i2 * a.s_nb2 + i3 * a.s_nb3 + 4 * (32 * b + 4 * sub));
    const float xv[4] = {x.x, x.y, x.z, x.w};
    uint8_t *blk = a.dst + (store ? dr : 0) * a.d_nb1 + i2 * a.d_nb2 + i3 * a.d_nb3;
    if constexpr (T == kQ8) {
        float amax = fmaxf(fmaxf(fabsf(xv[0]), fabsf(xv[1])), fmaxf(fabsf(xv[2]), fabsf(xv[3])));
#pragma unroll
        for (int o = 4; o > 0; o >>= 1)
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint32_t w = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w |= (uint32_t)(uint8_t)(int8_t)roundf(__fmul_rn(xv[j], id)) << (8 * j);
        if (store) {
            blk += 34 * b;
            uint16_t *c = reinterpret_cast<uint16_t *>(blk + 2 + 4 * sub);
            c[0] = (uint16_t)w;
            c[1] = (uint16_t)(w >> 16);
            if (sub == 0)
                *reinterpret_cast<uint16_t *>(blk) = __half_as_ushort(__float2half_rn(d));
        }
    } else {
        // first element of largest magnitude: (|x|, -index) ordering
        float am = -1.0f, vm = 0.0f;
        int im = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (fabsf(xv[j]) > am) {
                am = fabsf(xv[j]);
                vm = xv[j];
                im = 4 * sub + j;
            }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
            const float a2 = __shfl_xor_sync(0xffffffffu, am, o);
            const float v2 = __shfl_xor_sync(0xffffffffu, vm, o);
            const int i2x = __shfl_xor_sync(0xffffffffu, im, o);
            if (a2 > am || (a2 == am && i2x < im)) {
                am = a2;
                vm = v2;
                im = i2x;
            }
        }
        const float d = (am > 0.0f ? vm : 0.0f) / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint32_t q4 = 0; // four 4-bit codes of this lane's elements
#pragma unroll
        for (int j = 0; j < 4; ++j)
            q4 |= (uint32_t)min(15, (int)(int8_t)__fadd_rn(__fmul_rn(xv[j], id), 8.5f)) << (8 * j);
        // byte k of the block holds element k (low nibble) and k + 16 (high):
        // lanes 0-3 combine their codes with those of lanes 4-7
        const uint32_t hi = __shfl_down_sync(0xffffffffu, q4, 4);
        if (store && sub < 4) {
            blk += 18 * b;
            const uint32_t w = q4 | (hi << 4);
            uint16_t *c = reinterpret_cast<uint16_t *>(blk + 2 + 4 * sub);
            c[0] = (uint16_t)w;
            c[1] = (uint16_t)(w >> 16);
            if (sub == 0)
                *reinterpret_cast<uint16_t *>(blk) = __half_as_ushort(__float2half_rn(d));
        }
    }
}

// Float4 unit f = 32 j + lane of a source row (elements 4 f .. 4 f + 3) in
// dst type T: a 32-element block is the 8 lanes of a quarter warp with
// set_rows_coop_kernel's arithmetic; Q8_0 / Q4_0 codes and scales go to the
// staging row `out` (the destination row's bytes), F16 / F32 to `out` itself.
// Warp-collective for Q8_0 / Q4_0.
template <int T>
__device__ __forceinline__ void row_unit(const float4 v, int f, int sub, uint8_t *out) {
    const float e[4] = {v.x, v.y, v.z, v.w};
    const int b = f >> 3;
    if constexpr (T == kF32) {
        reinterpret_cast<float4 *>(out)[f] = v;
    } else if constexpr (T == kF16) {
        const uint32_t lo = (uint32_t)__half_as_ushort(__float2half_rn(e[0])) |
                            ((uint32_t)__half_as_ushort(__float2half_rn(e[1])) << 16);
        const uint32_t hi = (uint32_t)__half_as_ushort(__float2half_rn(e[2])) |
                            ((uint32_t)__half_as_ushort(__float2half_rn(e[3])) << 16);
        reinterpret_cast<uint2 *>(out)[f] = make_uint2(lo, hi);
    } else if constexpr (T == kQ8) {
        float amax = fmaxf(fmaxf(fabsf(e[0]), fabsf(e[1])), fmaxf(fabsf(e[2]), fabsf(e[3])));
#pragma unroll
        for (int o = 4; o > 0; o >>= 1)
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint32_t w = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w |= (uint32_t)(uint8_t)(int8_t)roundf(__fmul_rn(e[j], id)) << (8 * j);
        uint16_t *c = reinterpret_cast<uint16_t *>(out + 34 * b + 2 + 4 * sub);
        c[0] = (uint16_t)w;
        c[1] = (uint16_t)(w >> 16);
        if (sub == 0)
            *reinterpret_cast<uint16_t *>(out + 34 * b) = __half_as_ushort(__float2half_rn(d));
    } else {
        float am = -1.0f, vm = 0.0f;
        int im = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (fabsf(e[j]) > am) {
                am = fabsf(e[j]);
                vm = e[j];
                im = 4 * sub + j;
            }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) {
            const float a2 = __shfl_xor_sync(0xffffffffu, am, o);
            const float v2 = __shfl_xor_sync(0xffffffffu, vm, o);
            const int i2x = __shfl_xor_sync(0xffffffffu, im, o);
            if (a2 > am || (a2 == am && i2x < im)) {
                am = a2;
                vm = v2;
                im = i2x;
            }
        }
        const float d = (am > 0.0f ? vm : 0.0f) / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint32_t q4 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            q4 |= (uint32_t)min(15, (int)(int8_t)__fadd_rn(__fmul_rn(e[j], id), 8.5f)) << (8 * j);
        const uint32_t hi = __shfl_down_sync(0xffffffffu, q4, 4);
        if (sub < 4) {
            const uint32_t w = q4 | (hi << 4);
            uint16_t *c = reinterpret_cast<uint16_t *>(out + 18 * b + 2 + 4 * sub);
            c[0] = (uint16_t)w;
            c[1] = (uint16_t)(w >> 16);
            if (sub == 0)
                *reinterpret_cast<uint16_t *>(out + 18 * b) = __half_as_ushort(__float2half_rn(d));
        }
    }
}

// One source row per warp, for destination rows made of whole 16-byte chunks
// (16-byte aligned; ne0 % 256 == 0 for Q8_0 / Q4_0, % 128 for F16 / F32;
// ne0 <= 4096).  Each lane loads float4 units 32 j + lane of the row, up to
// eight in flight before any is used, and converts them with row_unit; Q8_0 /
// Q4_0 rows are assembled in a per-warp staging row in shared memory and leave
// in 16-byte stores.  Rows of one sequence (blockIdx.y = i3) go KV head
// fastest (i2, then i1), so a CTA reads and writes contiguous runs of a
// token's heads; the row indexing is 32-bit (ne1 * ne2 < 2^31).  (Four rows
// per warp, more loads in flight at 80 registers, measured slower on 256-wide
// Q8_0 rows: 32.4 against 29.4 us for a 8192-token K+V write.)
template <int T>
__global__ void __launch_bounds__(256) set_rows_row_kernel(const SetRowsArgs a, uint32_t seq_rows,
                                                           int row_bytes) {
    constexpr int UJ = 8; // float4 units per lane per load batch
    extern __shared__ __align__(16) uint8_t stage[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane & 7;
    const uint32_t row = blockIdx.x * 8u + (uint32_t)warp;
    if (row >= seq_rows)
        return; // warp-uniform, and nothing below synchronises the CTA
    const uint32_t ne2 = (uint32_t)a.ne2, i3 = blockIdx.y;
    const uint32_t i1 = row / ne2, i2 = row - i1 * ne2;
    const uint8_t *ip = a.idx + (uint64_t)i1 * (uint64_t)a.i_nb0 +
                        (uint64_t)(i2 % (uint32_t)a.i_ne1) * (uint64_t)a.i_nb1 +
                        (uint64_t)(i3 % (uint32_t)a.i_ne2) * (uint64_t)a.i_nb2;
    const int64_t dr = a.idx_i64 ? *reinterpret_cast<const int64_t *>(ip)
                                 : (int64_t)*reinterpret_cast<const int32_t *>(ip);
    if (dr < 0 || dr >= a.d_rows)
        return;
    const float4 *x = reinterpret_cast<const float4 *>(
        a.src + (uint64_t)i1 * (uint64_t)a.s_nb1 + (uint64_t)i2 * (uint64_t)a.s_nb2 +
        (uint64_t)i3 * (uint64_t)a.s_nb3);
    uint8_t *y = a.dst + dr * a.d_nb1 + (uint64_t)i2 * (uint64_t)a.d_nb2 +
                 (uint64_t)i3 * (uint64_t)a.d_nb3;
    constexpr bool QUANT = T == kQ8 || T == kQ4;
    uint8_t *srow = stage + warp * row_bytes;
    const int nj = (int)(a.ne0 >> 7);
    for (int j0 = 0; j0 < nj; j0 += UJ) {
        float4 xv[UJ];
#pragma unroll
        for (int u = 0; u < UJ; ++u)
            if (j0 + u < nj)
                xv[u] = __ldcs(x + 32 * (j0 + u) + lane); // read once: evict first
#pragma unroll
        for (int u = 0; u < UJ; ++u)
            if (j0 + u < nj) // warp-uniform
                row_unit<T>(xv[u], 32 * (j0 + u) + lane, sub, QUANT ? srow : y);
    }
    if constexpr (QUANT) {
        __syncwarp();
        for (int c = lane; c < row_bytes / 16; c += 32)
            reinterpret_cast<uint4 *>(y)[c] = reinterpret_cast<const uint4 *>(srow)[c];
    }
}

template <int T>
cudaError_t launch_set_rows_rows(const SetRowsArgs &a, uint32_t seq_rows, int rb, cudaStream_t st) {
    const dim3 grid((seq_rows + 7u) / 8u, (unsigned)a.ne3);
    const size_t smem = (size_t)8 * rb; // <= 34.8 KB: no opt-in needed
    set_rows_row_kernel<T><<<grid, 256, smem, st>>>(a, seq_rows, rb);
    return cudaGetLastError();
}

// One lane per 32-element block, for Q8_0 / Q4_0 destinations whose rows are
// 8, 16 or 32 blocks long (ne0 = 256, 512, 1024) and 16-byte aligned.  A tile
// is 32 consecutive blocks of one sequence (4, 2 or 1 rows, KV head fastest);
// each warp runs through tiles (persistent grid), its next tile's rows copied
// into shared memory by 16-byte cp.async (coalesced, two tiles in flight, no
// spin waits: cp.async.wait_group) while it quantizes the current one.  A lane
// reads its block's 128 bytes (chunk k of block l at slot k ^ (l & 7): no bank
// conflicts) and runs the reference quantizer on the block alone
// (quantize_row_q8_0_ref / quantize_row_q4_0_ref: no shuffles, one division
// and one reciprocal per block); the 34- or 18-byte blocks are packed into a
// per-warp staging area in row order and the tile's rows leave in 16-byte
// stores.  A row whose index is out of range is not written.
namespace srb {
constexpr int TILE_IN = 32 * 128;                  // input bytes per tile
__host__ __device__ constexpr int out_bytes(int T) { return 32 * (T == kQ8 ? 34 : 18); }
__host__ __device__ constexpr int warp_bytes(int T) { return 2 * TILE_IN + out_bytes(T); }
} // namespace srb

template <int T, int LNB>
__global__ void __launch_bounds__(256) set_rows_block_kernel(const SetRowsArgs a,
                                                             uint32_t seq_rows, uint32_t tiles_seq) {
    constexpr int NB = 1 << LNB;               // blocks per row
    constexpr int BB = T == kQ8 ? 34 : 18;     // bytes per block
    constexpr int RB = NB * BB;                // bytes per row (a multiple of 16)
    constexpr int RPT = 32 / NB;               // rows per tile
    constexpr int CPR = RB / 16;               // 16-byte output chunks per row
    static_assert(RB % 16 == 0, "whole chunks per row");
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t *in = smem + warp * srb::warp_bytes(T); // [2][32 blocks][128 B]
    uint8_t *out = in + 2 * srb::TILE_IN;           // [32 blocks][BB]
    const uint32_t ne2 = (uint32_t)a.ne2;
    const uint32_t n_tiles = tiles_seq * (uint32_t)a.ne3; // < 2^31 (checked by the launcher)
    const uint32_t stride = gridDim.x * 8u;
    const uint32_t first = blockIdx.x * 8u + (uint32_t)warp;

    // tile -> buffer: lane copies chunks lane + 32 m (row m >> (LNB - 2) of
    // the tile for NB >= 4), always one commit group (possibly empty)
    auto issue = [&](uint32_t tile, int buf) {
        if (tile < n_tiles) {
            const uint32_t i3 = tile / tiles_seq;
            const uint32_t row0 = (tile - i3 * tiles_seq) * RPT;
            const uint32_t base = smem_u32(in + buf * srb::TILE_IN);
            uint32_t i1 = row0 / ne2, i2 = row0 - i1 * ne2; // stepped per row below
#pragma unroll
            for (int k = 0; k < RPT; ++k) {
                if (row0 + k >= seq_rows)
                    break;
                const uint8_t *src = a.src + (uint64_t)i1 * (uint64_t)a.s_nb1 +
                                     (uint64_t)i2 * (uint64_t)a.s_nb2 +
                                     (uint64_t)i3 * (uint64_t)a.s_nb3;
                if (++i2 == ne2) {
                    i2 = 0;
                    ++i1;
                }
#pragma unroll
                for (int m = 0; m < 8 / RPT; ++m) {
                    const int w = lane + 32 * m;          // 16-byte chunk within the row
                    const int l = k * NB + (w >> 3), kk = w & 7; // block of the tile, chunk
                    cp_async<16>(base + 128 * l + 16 * (kk ^ (l & 7)), src + 16 * w);
                }
            }
        }
        cp_async_commit();
    };

    // this lane's row of a tile: its index (loaded one tile ahead, so the
    // load's latency hides behind the current tile) and its address terms
    struct RowRef {
        int64_t dr; // destination row, or -1
        uint32_t i2, i3;
    };
    auto row_ref = [&](uint32_t tile) {
        RowRef r = {-1, 0u, 0u};
        if (tile >= n_tiles)
            return r;
        const uint32_t i3 = tile / tiles_seq;
        const uint32_t row = (tile - i3 * tiles_seq) * RPT + (uint32_t)(lane >> LNB);
        if (row >= seq_rows)
            return r;
        const uint32_t i1 = row / ne2, i2 = row - i1 * ne2;
        // ggml broadcasts the index over heads and sequences (i_ne1 | ne2,
        // i_ne2 | ne3); the usual 1 and full extents need no division
        const uint32_t in1 = (uint32_t)a.i_ne1, in2 = (uint32_t)a.i_ne2;
        const uint32_t j2 = in1 == 1u ? 0u : in1 == ne2 ? i2 : i2 % in1;
        const uint32_t j3 = in2 == 1u ? 0u : in2 == (uint32_t)a.ne3 ? i3 : i3 % in2;
        const uint8_t *ip = a.idx + (uint64_t)i1 * (uint64_t)a.i_nb0 +
                            (uint64_t)j2 * (uint64_t)a.i_nb1 + (uint64_t)j3 * (uint64_t)a.i_nb2;
        r.dr = a.idx_i64 ? *reinterpret_cast<const int64_t *>(ip)
                         : (int64_t)*reinterpret_cast<const int32_t *>(ip);
        r.i2 = i2;
        r.i3 = i3;
        return r;
    };

    issue(first, 0);
    issue(first + stride, 1);
    RowRef next = row_ref(first);
    int buf = 0;
    for (uint32_t tile = first; tile < n_tiles; tile += stride, buf ^= 1) {
        const RowRef cur = next;
        next = row_ref(tile + stride);
        cp_async_wait<1>(); // this tile's copies (the next tile's may be in flight)
        __syncwarp();       // ... and every other lane's
        float x[32];
        {
            const uint8_t *blkin = in + buf * srb::TILE_IN + 128 * lane;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 v = *reinterpret_cast<const float4 *>(blkin + 16 * (k ^ (lane & 7)));
                x[4 * k] = v.x;
                x[4 * k + 1] = v.y;
                x[4 * k + 2] = v.z;
                x[4 * k + 3] = v.w;
            }
        }
        uint16_t *blk = reinterpret_cast<uint16_t *>(out + BB * lane); // 2-byte aligned
        if constexpr (T == kQ8) {
            float m[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                m[j] = fmaxf(fabsf(x[j]), fabsf(x[j + 16]));
#pragma unroll
            for (int w = 8; w > 0; w >>= 1)
#pragma unroll
                for (int j = 0; j < w; ++j)
                    m[j] = fmaxf(m[j], m[j + w]);
            const float d = m[0] / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            blk[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t c0 = (uint8_t)(int8_t)roundf(__fmul_rn(x[2 * j], id));
                const uint32_t c1 = (uint8_t)(int8_t)roundf(__fmul_rn(x[2 * j + 1], id));
                blk[1 + j] = (uint16_t)(c0 | (c1 << 8));
            }
        } else {
            // the first element of largest magnitude, in element order
            float amax = 0.0f, vmax = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (amax < fabsf(x[j])) {
                    amax = fabsf(x[j]);
                    vmax = x[j];
                }
            const float d = vmax / -8.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            blk[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t w = 0;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int e = 2 * j + h;
                    const uint32_t lo =
                        (uint32_t)min(15, (int)(int8_t)__fadd_rn(__fmul_rn(x[e], id), 8.5f));
                    const uint32_t hi =
                        (uint32_t)min(15, (int)(int8_t)__fadd_rn(__fmul_rn(x[16 + e], id), 8.5f));
                    w |= (lo | (hi << 4)) << (8 * h);
                }
                blk[1 + j] = (uint16_t)w;
            }
        }
        uint8_t *yrow = nullptr; // this lane's destination row (null: not written)
        if (cur.dr >= 0 && cur.dr < a.d_rows)
            yrow = a.dst + cur.dr * a.d_nb1 + (uint64_t)cur.i2 * (uint64_t)a.d_nb2 +
                   (uint64_t)cur.i3 * (uint64_t)a.d_nb3;
        // destination rows of the tile: row k's pointer from its first block's lane
        uint8_t *yk[RPT];
#pragma unroll
        for (int k = 0; k < RPT; ++k)
            yk[k] = reinterpret_cast<uint8_t *>(
                __shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(yrow), k * NB));
        __syncwarp();
        for (int c = lane; c < RPT * CPR; c += 32) {
            const int k = c / CPR, off = c - k * CPR;
            uint8_t *y = yk[0];
#pragma unroll
            for (int kk = 1; kk < RPT; ++kk)
                y = k == kk ? yk[kk] : y;
            if (y)
                reinterpret_cast<uint4 *>(y)[off] = reinterpret_cast<const uint4 *>(out)[c];
        }
        __syncwarp(); // the input buffer and the staging area are free again
        issue(tile + 2 * stride, buf); // no wrap: n_tiles + 2 stride < 2^32
    }
    cp_async_wait<0>(); // no copy outlives the kernel
}

template <int T>
cudaError_t launch_set_rows_blocks(const SetRowsArgs &a, uint32_t seq_rows, cudaStream_t st) {
    static std::atomic<unsigned long long> attr[3][2];
    const int nb = (int)(a.ne0 / 32), lnb = nb == 8 ? 3 : nb == 16 ? 4 : 5;
    const uint32_t rpt = 32u / (uint32_t)nb;
    const uint32_t tiles_seq = (seq_rows + rpt - 1) / rpt;
    const uint64_t n_tiles = (uint64_t)tiles_seq * (uint64_t)a.ne3;
    const size_t smem = (size_t)8 * srb::warp_bytes(T); // 71 or 74 KB: three CTAs per SM
    const uint64_t want = (n_tiles + 7) / 8, cap = (uint64_t)3 * (a.n_sm > 0 ? a.n_sm : 148);
    const dim3 grid((unsigned)(want < cap ? want : cap));
    if (n_tiles > 0x7fffffffull || grid.x > 65535u)
        return cudaErrorInvalidValue; // the launcher only sends shapes below these bounds
    const void *kern = lnb == 3   ? (const void *)set_rows_block_kernel<T, 3>
                       : lnb == 4 ? (const void *)set_rows_block_kernel<T, 4>
                                  : (const void *)set_rows_block_kernel<T, 5>;
    cudaError_t e = set_smem_limit(kern, smem, attr[lnb - 3][T == kQ8 ? 0 : 1]);
    if (e != cudaSuccess)
        return e;
    if (lnb == 3)
        set_rows_block_kernel<T, 3><<<grid, 256, smem, st>>>(a, seq_rows, tiles_seq);
    else if (lnb == 4)
        set_rows_block_kernel<T, 4><<<grid, 256, smem, st>>>(a, seq_rows, tiles_seq);
    else
        set_rows_block_kernel<T, 5><<<grid, 256, smem, st>>>(a, seq_rows, tiles_seq);
    return cudaGetLastError();
}

cudaError_t launch_set_rows(int type, const SetRowsArgs &a, cudaStream_t st) {
    if (a.n_units <= 0)
        return cudaSuccess;
    const bool src16 = ((reinterpret_cast<uintptr_t>(a.src) | (uintptr_t)a.s_nb1 |
                         (uintptr_t)a.s_nb2 | (uintptr_t)a.s_nb3) & 15) == 0;
    const bool dst16 = ((reinterpret_cast<uintptr_t>(a.dst) | (uintptr_t)a.d_nb1 |
                         (uintptr_t)a.d_nb2 | (uintptr_t)a.d_nb3) & 15) == 0;
    const bool quant = type == kQ8 || type == kQ4;
    const int64_t seq_rows = a.ne1 * a.ne2;
    if (src16 && dst16 && a.ne0 <= 4096 && a.ne0 % (quant ? 256 : 128) == 0 &&
        seq_rows <= 0x7fffffffll && a.ne3 <= 65535) {
        const int rb = type == kQ8 ? 34 * (int)(a.ne0 / 32) : type == kQ4 ? 18 * (int)(a.ne0 / 32) : 0;
        const uint32_t sr = (uint32_t)seq_rows;
        if (quant && (a.ne0 == 256 || a.ne0 == 512 || a.ne0 == 1024) &&
            (uint64_t)((sr + 31u) / 32u * (a.ne0 / 32)) * (uint64_t)a.ne3 <= 0x3fffffffull &&
            a.n_sm > 0 && a.n_sm <= 8192)
            return type == kQ8 ? launch_set_rows_blocks<kQ8>(a, sr, st)
                               : launch_set_rows_blocks<kQ4>(a, sr, st);
        switch (type) {
        case kF32: return launch_set_rows_rows<kF32>(a, sr, rb, st);
        case kF16: return launch_set_rows_rows<kF16>(a, sr, rb, st);
        case kQ8: return launch_set_rows_rows<kQ8>(a, sr, rb, st);
        case kQ4: return launch_set_rows_rows<kQ4>(a, sr, rb, st);
        default: return cudaErrorInvalidValue;
        }
    }
    const int64_t planes = a.ne2 * a.ne3, plane_units = a.ne1 * (a.ne0 / 32);
    if ((type == kQ8 || type == kQ4) && src16 && planes <= 65535 &&
        plane_units * 8 <= 0x7fffffffll) {
        const dim3 grid((unsigned)((plane_units * 8 + 255) / 256), 1, (unsigned)planes);
        if (type == kQ8)
            set_rows_coop_kernel<kQ8><<<grid, 256, 0, st>>>(a);
        else
            set_rows_coop_kernel<kQ4><<<grid, 256, 0, st>>>(a);
        return cudaGetLastError();
    }
    const unsigned blocks = (unsigned)((a.n_units + 255) / 256);
    switch (type) {
    case kF32: set_rows_kernel<kF32><<<blocks, 256, 0, st>>>(a); break;
    case kF16: set_rows_kernel<kF16><<<blocks, 256, 0, st>>>(a); break;
    case kQ8: set_rows_kernel<kQ8><<<blocks, 256, 0, st>>>(a); break;
    case kQ4: set_rows_kernel<kQ4><<<blocks, 256, 0, st>>>(a); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant(int type, const void *src, uint64_t ss, float *dst, uint64_t ds,
                           int64_t n_rows, int64_t n_per_row, cudaStream_t st) {
    const int64_t units = n_rows * (type == kF16 ? n_per_row : n_per_row / 32);
    if (units <= 0)
        return cudaSuccess;
    const unsigned blocks = (unsigned)((units + 255) / 256);
    const uint8_t *s = static_cast<const uint8_t *>(src);
    switch (type) {
    case kF16: dequant_kernel<kF16><<<blocks, 256, 0, st>>>(s, ss, dst, ds, n_rows, n_per_row); break;
    case kQ8: dequant_kernel<kQ8><<<blocks, 256, 0, st>>>(s, ss, dst, ds, n_rows, n_per_row); break;
    case kQ4: dequant_kernel<kQ4><<<blocks, 256, 0, st>>>(s, ss, dst, ds, n_rows, n_per_row); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_quant(int type, const float *src, uint64_t ss, void *dst, uint64_t ds,
                         int64_t n_rows, int64_t n_per_row, cudaStream_t st) {
    const int64_t units = n_rows * (type == kF16 ? n_per_row : n_per_row / 32);
    if (units <= 0)
        return cudaSuccess;
    const unsigned blocks = (unsigned)((units + 255) / 256);
    uint8_t *d = static_cast<uint8_t *>(dst);
    switch (type) {
    case kF16: quant_kernel<kF16><<<blocks, 256, 0, st>>>(src, ss, d, ds, n_rows, n_per_row); break;
    case kQ8: quant_kernel<kQ8><<<blocks, 256, 0, st>>>(src, ss, d, ds, n_rows, n_per_row); break;
    case kQ4: quant_kernel<kQ4><<<blocks, 256, 0, st>>>(src, ss, d, ds, n_rows, n_per_row); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

} // namespace xq
