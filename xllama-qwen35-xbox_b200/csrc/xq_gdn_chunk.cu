// GATED_DELTA_NET over long sequences in chunked (WY) form on the tcgen05
// tensor cores, TF32 operands with FP32 accumulation.
//
// Recurrence (ggml-cpu, one value head; S is S_v x S_k, row j = value column):
//   S_t = g~_t S_{t-1} + u_t k_t^T,   u_t = beta_t (v_t - g~_t S_{t-1} k_t),
//   y_t = scale * S_t q_t,            g~_t = exp(g_t)
// Over a chunk of C = 64 tokens with S_0 the state entering it, G_t the
// inclusive prefix sum of g inside the chunk, b_t = exp(G_t),
// e_t = exp(G_C - G_t):
//   A_ts = beta_t exp(G_t - G_s) k_t.k_s          (s < t, else 0)
//   T''  = (I + A)^-1 diag(beta)
//   M_ts = scale exp(G_t - G_s) q_t.k_s           (s <= t, else 0)
//   X    = K S_0^T,  X' = V - diag(b) X,  U = T'' X'
//   Y    = scale diag(b) Q S_0^T + M U
//   S_C^T = b_C S_0^T + K^T diag(e) U
// (u_t of the recurrence is row t of U; expanding S_{t-1} over the chunk gives
// (I + A) U = diag(beta) (V - diag(b) K S_0^T).)
//
// Two kernels:
//   gdn_chunk_prep_kernel  one CTA per (chunk, head, sequence), all in
//     parallel (chunk-major order), 3 CTAs per SM: [K;Q] K^T on the tensor core (M=128, N=64,
//     K=128), the gates, the unit lower-triangular inverse in FP32 (16x16
//     diagonal blocks by forward substitution, then block rows; four lanes
//     per column), and writes [T''; M] (128 x 64) plus b, e, b_C to the
//     workspace.
//   gdn_chunk_scan_kernel  one CTA per (32 state rows, head, sequence),
//     sequential over chunks with the state in FP32 registers (two threads
//     per TMEM lane i, 16 of the 32 rows each) and a TF32 copy in shared
//     memory as the B operand of MMA1:
//       MMA1  [K;Q'] S_0^T         TS, M=128 (64 K rows + 64 rows of
//                                  Q' = diag(scale b) Q), N=32, K=128
//       MMA2  [T'';M] X'           TS, A in TMEM, B = X' MN-major, K=64
//       MMA4  K^T (diag(e) U)      TS (M=128 over the key elements): the
//                                  state update
//       MMA3  [T'';M] U            TS, accumulated onto MMA1's result: rows
//                                  64..127 become y = scale b Q S_0^T + M U
//     MN-major TF32 operands (X', U, diag(e) U) use the 128-byte swizzle with
//     32-byte granules, the only MN-major layout for 32-bit elements; K-major
//     operands use the plain 128-byte swizzle TMA writes.  Warp roles: 8
//     chain warps, 4 copier warps that move the next chunk's A operands into
//     TMEM and the finished output rows to a TMA store, and a producer warp
//     whose three lanes stream K/Q tiles, V tiles + factors and [T''; M]
//     independently.
// Operands produced here (S, X', U, T'', M) are rounded to TF32 to nearest;
// K, Q, V tiles enter the tensor core as stored (fp32 read as TF32).  Tokens
// past T read as zeros with g = beta = 0, so a partial last chunk is exact.
// Every mbarrier wait is bounded; on timeout the kernel records an error,
// drains its own copies and MMAs with bounded waits, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include "xq_common.cuh"
#include "xq_internal.h"
#include "xq_tc.cuh"

namespace xq {

namespace gc {
constexpr int C = 64;        // tokens per chunk
constexpr int SK = 128;      // head size (key and value)
constexpr int R = 32;        // state rows per scan CTA
constexpr int AST = 68;      // padded row stride (floats) of the solve matrices
constexpr int ATM_FLOATS = 128 * 64; // [T''; M] per unit
constexpr int FAC_FLOATS = 256;      // b[64], e[64], b_C, pad (workspace stride)
constexpr int FAC_BYTES = 528;       // the part the scan loads: b, e, b_C (+3 pad)
constexpr int PREP_NT = 256;
constexpr int SCAN_NT = 416;         // 8 chain warps, 4 copier warps, 1 producer warp
constexpr float kLog2e = 1.4426950408889634f;

// prep kernel shared memory (3 CTAs per SM): the solve matrices reuse the
// K/Q tile once the tensor core has read it
constexpr int P_KQ = 0;                       // 4 slabs x 16 KB, rows 0-63 K, 64-127 Q
constexpr int P_AM = 0;                       // A [64][AST]            (after the MMA)
constexpr int P_TT = P_AM + 64 * AST * 4;     // T transposed [col][row] (after the MMA)
constexpr int P_G = 65536;                    // G[64], beta[64]
constexpr int P_BAR = P_G + 512;
constexpr int P_BYTES = P_BAR + 32 + 1024;    // + alignment slack

// scan kernel shared memory
constexpr int S_KQ = 0;                       // 2 stages x 64 KB
constexpr int S_V = 131072;                   // 2 stages x 8 KB
constexpr int S_ATM = 147456;                 // landing buffer, 2 slabs x 16 KB
constexpr int S_SB = 180224;                  // S operand, MN-major: row i (128), 32 columns
constexpr int S_XB = 196608;                  // X' (MN-major, 64 x 32)
constexpr int S_UB = 204800;                  // U
constexpr int S_U2 = 212992;                  // diag(e) U
constexpr int S_Y = 221184;                   // output tile (64 x 32, 128-byte swizzled)
constexpr int S_FAC = 229376;                 // 2 stages x FAC_BYTES
constexpr int S_BAR = S_FAC + 2 * FAC_BYTES;
constexpr int S_BYTES = S_BAR + 192 + 1024;

// scan kernel TMEM columns (A operands copied in by the copier warps)
constexpr uint32_t TM_ATM = 0;   // [T''; M], 2 buffers x 64
constexpr uint32_t TM_KT = 128;  // K^T (lane i, column t), 2 buffers x 64
constexpr uint32_t TM_KQ = 256;  // [K; diag(scale b) Q] rows, 128 columns
constexpr uint32_t TM_D1 = 384;  // MMA1 (+ MMA3 on rows 64-127), 2 buffers x 32
constexpr uint32_t TM_D2 = 448, TM_D4 = 480;
constexpr uint32_t TM_COLS = 512;

__host__ __device__ constexpr int n_chunks(int T, int slots) {
    // one snapshot slot: every token, the last chunk padded; K > 1 slots: the
    // last K tokens go to the per-token kernel, which writes the snapshots
    return slots == 1 ? (T + C - 1) / C : (T > slots ? (T - slots) / C : 0);
}

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}
__device__ __forceinline__ const float *at(const float *base, int64_t off) {
    return reinterpret_cast<const float *>(reinterpret_cast<const char *>(base) + off);
}
} // namespace gc

struct GdnChunkArgs {
    const float *g, *beta, *state;
    int64_t g_nb1, g_nb2, g_nb3, b_nb1, b_nb2, b_nb3, s_nb1, s_nb2, s_nb3;
    float *atm;       // [unit][128][64]
    float *fac;       // [unit][256]
    float *dst;       // y [n_seq][T][H][128]
    float *state_out; // [n_seq][H][128][128]
    int *err;
    int H, H_k, T, n_seq, rq3, rk3, NC;
    int h_off; // global index of value head 0 (key head of h: (h + h_off) % H_k)
    float scale;
};

// ---------------------------------------------------------------------------
// Per-chunk preparation (256 threads; four lanes per column of T in the
// solve, adjacent lanes of one warp).

// Block row BI of T = (I + A)^-1 for column cc (BI > cc / 16), lane p of the
// column's four computing rows 4p..4p+3 of the block row:
// E = A[16BI.., 16j:16BI] T[16j:16BI, cc] (T is zero above the column's own
// diagonal block j), then T[16BI + r, cc] = -(D_BI E)_r with
// D_BI = T[16BI.., 16BI..] (already in Tt).  Tt is column-major: Tt[col][row].
template <int BI>
__device__ __forceinline__ void solve_block_row(const float *Am, float *Tt, int cc, int p,
                                                int lane) {
    using namespace gc;
    const int j = cc >> 4;
    float e[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float *tcol = Tt + cc * AST;
    const float *arow = Am + (16 * BI + 4 * p) * AST;
#pragma unroll
    for (int m4 = 0; m4 < 4 * BI; ++m4) {
        if (m4 < 4 * j)
            continue;
        const float4 tv = *reinterpret_cast<const float4 *>(tcol + 4 * m4);
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            const float4 av = *reinterpret_cast<const float4 *>(arow + x * AST + 4 * m4);
            e[x] = fmaf(av.x, tv.x, e[x]);
            e[x] = fmaf(av.y, tv.y, e[x]);
            e[x] = fmaf(av.z, tv.z, e[x]);
            e[x] = fmaf(av.w, tv.w, e[x]);
        }
    }
    // the column's 16 E values from its four lanes
    float E[16];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int x = 0; x < 4; ++x)
            E[4 * q + x] = __shfl_sync(0xffffffffu, e[x], (lane & ~3) | q);
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int m = 0; m < 16; ++m) {
        // D[4p + x][m] for x = 0..3 (zero above the diagonal)
        const float4 d =
            *reinterpret_cast<const float4 *>(Tt + (16 * BI + m) * AST + 16 * BI + 4 * p);
        o[0] = fmaf(d.x, E[m], o[0]);
        o[1] = fmaf(d.y, E[m], o[1]);
        o[2] = fmaf(d.z, E[m], o[2]);
        o[3] = fmaf(d.w, E[m], o[3]);
    }
    *reinterpret_cast<float4 *>(Tt + cc * AST + 16 * BI + 4 * p) =
        make_float4(-o[0], -o[1], -o[2], -o[3]);
}

__global__ void __launch_bounds__(gc::PREP_NT, 3)
    gdn_chunk_prep_kernel(const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap qmap, const GdnChunkArgs a) {
    using namespace tc;
    using namespace gc;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    float *Am = reinterpret_cast<float *>(smem + P_AM);
    float *Tt = reinterpret_cast<float *>(smem + P_TT);
    float *Gs = reinterpret_cast<float *>(smem + P_G);
    float *Bs = Gs + 64;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P_BAR);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2);
    volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // blocks run chunk by chunk; inside a chunk the value heads that share a
    // key head (h = hk + j H_k) are adjacent, so the second CTA's K/Q tiles
    // come from L2
    const int c = (int)(blockIdx.x / (unsigned)a.H), x = (int)(blockIdx.x % (unsigned)a.H);
    const int J = a.H % a.H_k == 0 ? a.H / a.H_k : 1;
    const int h = J > 1 ? (x % J) * a.H_k + x / J : x, n = blockIdx.z;
    const int hk = (h + a.h_off) % a.H_k, t0 = c * C;
    const size_t unit = ((size_t)n * a.H + h) * a.NC + c;
    const uint32_t bar_tma = smem_u32(bars), bar_mma = smem_u32(bars + 1);

    if (tid == 0) {
        prefetch_map(&kmap);
        prefetch_map(&qmap);
        mbar_init(bar_tma, 1);
        mbar_init(bar_mma, 1);
        *abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        mbar_expect_tx(bar_tma, 65536);
#pragma unroll
        for (int ib = 0; ib < 4; ++ib) {
            const uint32_t slab = smem_u32(smem + P_KQ + ib * 16384);
            tma_load_4d(slab, &kmap, 32 * ib, hk, t0, n / a.rk3, bar_tma);
            tma_load_4d(slab + 8192, &qmap, 32 * ib, hk, t0, n / a.rq3, bar_tma);
        }
    }
    if (warp == 1)
        tmem_alloc(smem_u32(tmem_slot), 64);
    if (tid < 64) {
        // G = inclusive prefix sum of g over the chunk; padding tokens g = beta = 0
        const int t = t0 + tid;
        float gv = 0.0f, bv = 0.0f;
        if (t < a.T) {
            gv = *at(a.g, n * a.g_nb3 + (int64_t)t * a.g_nb2 + h * a.g_nb1);
            bv = *at(a.beta, n * a.b_nb3 + (int64_t)t * a.b_nb2 + h * a.b_nb1);
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, gv, o);
            if (lane >= o)
                gv += y;
        }
        Gs[tid] = gv;
        Bs[tid] = bv;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tid >= 32 && tid < 64)
        Gs[tid] += Gs[31];

    // S = [K; Q] K^T  (rows 0-63: K K^T, rows 64-127: Q K^T)
    if (warp == 0) {
        const bool ok = __all_sync(0xffffffffu, mbar_wait(bar_tma, 0, abort_s));
        if (ok) {
            tc_fence_after();
            if (elect_one()) {
                constexpr uint32_t ID = idesc_tf32(128, 64, 0, 0);
                const uint32_t base = smem_u32(smem + P_KQ);
#pragma unroll
                for (int kk = 0; kk < 16; ++kk) {
                    const uint64_t d = sdesc(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
                    mma_ss_tf32(tmem, d, d, ID, kk > 0);
                }
                mma_commit(bar_mma);
            }
            __syncwarp();
        } else {
            *abort_s = 1;
        }
    }
    __syncthreads(); // Gs complete
    __all_sync(0xffffffffu, mbar_wait(bar_mma, 0, abort_s));
    tc_fence_after();
    // thread (row r = TMEM lane, column half hh): columns 32 hh .. +31 of S;
    // the K/Q tile is dead now and its space holds A and T
    const int r = 32 * (warp & 3) + lane, hh = warp >> 2;
    float sv[32];
    tmem_ld32(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 32 * hh, sv);
    float *atm = a.atm + unit * ATM_FLOATS;
    if (r < 64) {
        const int t = r;
        const float Gt = Gs[t], bt = Bs[t];
#pragma unroll
        for (int s4 = 0; s4 < 8; ++s4) {
            float w[4];
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                const int s = 32 * hh + 4 * s4 + x;
                w[x] = s < t ? bt * ex2((Gt - Gs[s]) * kLog2e) * sv[4 * s4 + x] : 0.0f;
            }
            *reinterpret_cast<float4 *>(Am + t * AST + 32 * hh + 4 * s4) =
                make_float4(w[0], w[1], w[2], w[3]);
        }
    } else {
        const int t = r - 64;
        const float Gt = Gs[t];
        float4 *row = reinterpret_cast<float4 *>(atm + (64 + t) * 64 + 32 * hh);
#pragma unroll
        for (int s4 = 0; s4 < 8; ++s4) {
            uint32_t w[4];
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                const int s = 32 * hh + 4 * s4 + x;
                w[x] = s <= t ? to_tf32(a.scale * ex2((Gt - Gs[s]) * kLog2e) * sv[4 * s4 + x])
                              : 0u;
            }
            row[s4] = make_float4(__uint_as_float(w[0]), __uint_as_float(w[1]),
                                  __uint_as_float(w[2]), __uint_as_float(w[3]));
        }
    }
    __syncthreads(); // A complete

    // T = (I + A)^-1.  Diagonal 16x16 blocks by forward substitution: column
    // cc = tid / 4, lane p = tid % 4 holds x[4k + p]; row r's dot product is
    // split over the four lanes (A is zero on and above the diagonal, and the
    // x entries not yet computed are zero, so every row sums all 16 terms)
    const int cc = tid >> 2, p = tid & 3;
    {
        const int bi = cc >> 4, c0 = cc & 15;
        float *tcol = Tt + cc * AST;
        *reinterpret_cast<float4 *>(tcol + 16 * p) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4 *>(tcol + 16 * p + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4 *>(tcol + 16 * p + 8) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4 *>(tcol + 16 * p + 12) = make_float4(0.f, 0.f, 0.f, 0.f);
        float xs[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            xs[k] = 4 * k + p == c0 ? 1.0f : 0.0f;
        const float *Ab = Am + (16 * bi) * AST + 16 * bi + p;
#pragma unroll
        for (int rr = 1; rr < 16; ++rr) {
            float part = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                part = fmaf(Ab[rr * AST + 4 * k], xs[k], part);
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            if (rr > c0 && (rr & 3) == p)
                xs[rr >> 2] = -part;
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k)
            tcol[16 * bi + 4 * k + p] = xs[k];
    }
    __syncthreads(); // every diagonal block is in Tt
    {
        // the block rows below the column's own diagonal block, in order
        const int j = cc >> 4; // warp-uniform: a warp holds 8 columns of one block
        if (j < 1)
            solve_block_row<1>(Am, Tt, cc, p, lane);
        __syncwarp();
        if (j < 2)
            solve_block_row<2>(Am, Tt, cc, p, lane);
        __syncwarp();
        if (j < 3)
            solve_block_row<3>(Am, Tt, cc, p, lane);
    }
    __syncthreads(); // T complete
    {
        // T'' = T diag(beta) as rows 0-63 of [T''; M]: thread (column s, row
        // quarter q) reads its column of Tt 4 rows at a time; every warp store
        // covers 128 contiguous bytes of one row
        const int sc = tid & 63, t0r = 16 * (tid >> 6);
        const float bc = Bs[sc];
        const float *tcol = Tt + sc * AST + t0r;
#pragma unroll
        for (int t4 = 0; t4 < 4; ++t4) {
            const float4 v = *reinterpret_cast<const float4 *>(tcol + 4 * t4);
            float *o = atm + (t0r + 4 * t4) * 64 + sc;
            o[0] = __uint_as_float(to_tf32(v.x * bc));
            o[64] = __uint_as_float(to_tf32(v.y * bc));
            o[128] = __uint_as_float(to_tf32(v.z * bc));
            o[192] = __uint_as_float(to_tf32(v.w * bc));
        }
    }
    if (tid < 64) {
        // decay factors
        float *fac = a.fac + unit * FAC_FLOATS;
        const float Gt = Gs[tid], GC = Gs[63];
        fac[tid] = ex2(Gt * kLog2e);
        fac[64 + tid] = ex2((GC - Gt) * kLog2e);
        if (tid == 0)
            fac[128] = ex2(GC * kLog2e);
    }

    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        if (*abort_s) {
            // the tile copies may still be landing: bounded drain before exit
            volatile int none = 0;
            mbar_wait(bar_tma, 0, &none, 100000000ull);
            atomicExch(a.err, 1);
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 64);
    }
}

// ---------------------------------------------------------------------------
// Sequential scan over chunks, warp-specialised:
//   warps 0-7   chain: TMEM lane quarter (warp & 3), state columns
//               16 (warp >> 2) .. +15 of the CTA's 32; warp 0 issues MMA1,
//               MMA2, MMA4 and warp 4 issues MMA3
//   warps 8-11  copier: the next chunk's A operands into TMEM ([T''; M] rows
//               and K^T double-buffered, [K; diag(scale b) Q] rows single-
//               buffered once the chain's MMA1 is done), then the finished
//               chunk's output rows from TMEM to a TMA store
//   warp 12     producer: lane 0 K/Q tiles, lane 1 V tile + factors, lane 2
//               the [T''; M] landing buffer
// With Q pre-scaled by scale b_t, MMA1's rows 64-127 are the first term of
// y; MMA3 accumulates M U onto them, so the output never enters the chain.
__global__ void __launch_bounds__(gc::SCAN_NT, 1)
    gdn_chunk_scan_kernel(const __grid_constant__ CUtensorMap kmap,
                          const __grid_constant__ CUtensorMap qmap,
                          const __grid_constant__ CUtensorMap vmap,
                          const __grid_constant__ CUtensorMap amap,
                          const __grid_constant__ CUtensorMap ymap, const GdnChunkArgs a) {
    using namespace tc;
    using namespace gc;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = align1024(smem_raw);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + S_BAR);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 20);
    volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);
    auto bar = [&](int i) { return smem_u32(bars + i); };
    // kq_full[2], vf_full[2], kq_empty[2] (copier done with the K/Q tiles),
    // vf_empty[2], atm_full, atm_empty, tmem_ready[2] (copier -> chain: A
    // operands of chunk c in TMEM), kq_free (chain -> copier: MMA1 done, the
    // [K; Q] columns may be overwritten), d1_free[2] (copier -> chain: output
    // rows read), mma (MMA1/MMA2/MMA4), mma3
    constexpr int B_KQF = 0, B_VFF = 2, B_KQE = 4, B_VFE = 6, B_AF = 8, B_AE = 9, B_TR = 10,
                  B_KQFREE = 12, B_D1F = 13, B_MMA = 15, B_MMA3 = 16;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slice = blockIdx.x, h = blockIdx.y, n = blockIdx.z;
    const int j0 = slice * R, hk = (h + a.h_off) % a.H_k;
    const size_t unit0 = ((size_t)n * a.H + h) * a.NC;

    if (tid == 0) {
        prefetch_map(&kmap);
        prefetch_map(&qmap);
        prefetch_map(&vmap);
        prefetch_map(&amap);
        prefetch_map(&ymap);
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar(B_KQF + i), 1);
            mbar_init(bar(B_VFF + i), 1);
            mbar_init(bar(B_KQE + i), 128);
            mbar_init(bar(B_VFE + i), 1);
            mbar_init(bar(B_TR + i), 128);
            mbar_init(bar(B_D1F + i), 1);
        }
        mbar_init(bar(B_AF), 1);
        mbar_init(bar(B_AE), 128);
        mbar_init(bar(B_KQFREE), 1);
        mbar_init(bar(B_MMA), 1);
        mbar_init(bar(B_MMA3), 1);
        *abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0)
        tmem_alloc(smem_u32(tmem_slot), TM_COLS);

    // chain thread (row r = TMEM lane = key element i, column half hc) holds
    // state rows j0 + 16 hc .. +15 at column i in FP32 registers; the TF32
    // operand copy is the MN-major S tile (row i, 32 value columns)
    const int r = 32 * (warp & 3) + lane, hc = (warp >> 2) & 1;
    float S[16];
    auto store_s = [&]() {
        uint32_t v[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj)
            v[jj] = to_tf32_fast(S[jj]);
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            uint8_t *p = smem + S_SB + sw128_32b(r, 2 * hc + g);
            *reinterpret_cast<uint4 *>(p) = make_uint4(v[8 * g], v[8 * g + 1], v[8 * g + 2], v[8 * g + 3]);
            *reinterpret_cast<uint4 *>(p + 16) =
                make_uint4(v[8 * g + 4], v[8 * g + 5], v[8 * g + 6], v[8 * g + 7]);
        }
    };
    if (warp < 8) {
        const float *sp = at(a.state, n * a.s_nb3 + (int64_t)h * a.s_nb2);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj)
            S[jj] = *at(sp, (int64_t)(j0 + 16 * hc + jj) * a.s_nb1 + 4 * r);
        store_s();
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);

    if (warp == 12) {
        // ----------------------------- producer -----------------------------
        if (lane < 3) {
            int issued = 0;
            for (int c = 0; c < a.NC; ++c) {
                const int s = c & 1, use = c >> 1;
                if (lane == 0) {
                    if (use >= 1 && !mbar_wait(bar(B_KQE + s), (use - 1) & 1, abort_s))
                        break;
                    mbar_expect_tx(bar(B_KQF + s), 65536);
                    const uint32_t kq = smem_u32(smem + S_KQ + s * 65536);
#pragma unroll
                    for (int ib = 0; ib < 4; ++ib) {
                        tma_load_4d(kq + ib * 16384, &kmap, 32 * ib, hk, c * C, n / a.rk3,
                                    bar(B_KQF + s));
                        tma_load_4d(kq + ib * 16384 + 8192, &qmap, 32 * ib, hk, c * C,
                                    n / a.rq3, bar(B_KQF + s));
                    }
                } else if (lane == 1) {
                    if (use >= 1 && !mbar_wait(bar(B_VFE + s), (use - 1) & 1, abort_s))
                        break;
                    mbar_expect_tx(bar(B_VFF + s), 8192 + FAC_BYTES);
                    tma_load_4d(smem_u32(smem + S_V + s * 8192), &vmap, j0, h, c * C, n,
                                bar(B_VFF + s));
                    bulk_load(smem_u32(smem + S_FAC + s * FAC_BYTES),
                              a.fac + (unit0 + c) * FAC_FLOATS, FAC_BYTES, bar(B_VFF + s));
                } else {
                    if (c >= 1 && !mbar_wait(bar(B_AE), (c - 1) & 1, abort_s))
                        break;
                    mbar_expect_tx(bar(B_AF), 32768);
                    const int row = (int)((unit0 + c) * 128);
                    tma_load_2d(smem_u32(smem + S_ATM), &amap, 0, row, bar(B_AF));
                    tma_load_2d(smem_u32(smem + S_ATM + 16384), &amap, 32, row, bar(B_AF));
                }
                issued = c + 1;
            }
            if (issued < a.NC) {
                // a wait failed: stop everyone, then let this lane's copies in
                // flight complete their barriers (bounded)
                *abort_s = 1;
                volatile int none = 0;
                for (int m = issued - 2 < 0 ? 0 : issued - 2; m < issued; ++m) {
                    if (lane == 0)
                        mbar_wait(bar(B_KQF + (m & 1)), (m >> 1) & 1, &none, 100000000ull);
                    else if (lane == 1)
                        mbar_wait(bar(B_VFF + (m & 1)), (m >> 1) & 1, &none, 100000000ull);
                    else if (m == issued - 1)
                        mbar_wait(bar(B_AF), m & 1, &none, 100000000ull);
                }
            }
        }
    } else if (warp >= 8) {
        // ------------------------------ copier ------------------------------
        auto copier_sync = []() { asm volatile("bar.sync 2, 128;" ::: "memory"); };
        uint32_t w[16];
        int y_pending = 0;
        // output rows of chunk cy: D1 rows 64-127 once MMA3 has accumulated
        // M U onto them; 128-byte swizzled tile, one TMA store
        auto emit_y = [&](int cy) -> bool {
            if (!mbar_wait(bar(B_MMA3), cy & 1, abort_s))
                return false;
            tc_fence_after();
            if (tid == 256 && y_pending) {
                bulk_wait_read(); // the previous tile has left the buffer
                y_pending = 0;
            }
            copier_sync();
            if (r >= 64) {
                float y[32];
                tmem_ld32(lane_base + TM_D1 + 32 * (cy & 1), y);
                const int t = r - 64;
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4)
                    *reinterpret_cast<float4 *>(smem + S_Y + sw128(t, q4)) =
                        make_float4(y[4 * q4], y[4 * q4 + 1], y[4 * q4 + 2], y[4 * q4 + 3]);
            }
            fence_async_smem();
            tc_fence_before();
            copier_sync();
            if (tid == 256) {
                mbar_arrive(bar(B_D1F + (cy & 1))); // MMA1 may overwrite these columns
                // rows past T fall outside the map and are not written
                tma_store_4d(&ymap, smem_u32(smem + S_Y), j0, h, cy * C, n);
                bulk_commit();
                y_pending = 1;
            }
            return true;
        };
        bool ok = true;
        for (int cn = 0; cn < a.NC && ok; ++cn) {
            const int b = cn & 1;
            ok = mbar_wait(bar(B_KQF + b), (cn >> 1) & 1, abort_s) &&
                 mbar_wait(bar(B_AF), cn & 1, abort_s) &&
                 mbar_wait(bar(B_VFF + b), (cn >> 1) & 1, abort_s);
            // the previous chunk's MMA1 done: every MMA of chunk cn-2 (the last
            // reader of TMEM buffer b) and of the [K; Q] columns has completed
            if (ok && cn >= 1)
                ok = mbar_wait(bar(B_KQFREE), (cn - 1) & 1, abort_s);
            if (!ok)
                break;
            tc_fence_after();
            // [T''; M] row r -> TMEM buffer b (A of MMA2 / MMA3)
#pragma unroll
            for (int half = 0; half < 2; ++half)
#pragma unroll
                for (int hq = 0; hq < 2; ++hq) {
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(
                            smem + S_ATM + half * 16384 + sw128(r, 4 * hq + q4));
                        w[4 * q4] = v.x;
                        w[4 * q4 + 1] = v.y;
                        w[4 * q4 + 2] = v.z;
                        w[4 * q4 + 3] = v.w;
                    }
                    tmem_st16(lane_base + TM_ATM + 64 * b + 32 * half + 16 * hq, w);
                }
            // K^T: lane r takes column r of the K tile (rows t = 0..63), the A
            // operand of MMA4
            const uint8_t *kq = smem + S_KQ + b * 65536;
            const uint8_t *kcol = kq + (r >> 5) * 16384 + (r & 3) * 4;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
#pragma unroll
                for (int x = 0; x < 16; ++x)
                    w[x] = *reinterpret_cast<const uint32_t *>(
                        kcol + sw128(16 * q + x, (r & 31) >> 2));
                tmem_st16(lane_base + TM_KT + 64 * b + 16 * q, w);
            }
            mbar_arrive(bar(B_AE)); // the landing buffer is free
            // [K; diag(scale b) Q] rows -> TMEM (A of MMA1)
            const float qs = r >= 64 ? a.scale * reinterpret_cast<const float *>(
                                                     smem + S_FAC + b * FAC_BYTES)[r - 64]
                                     : 0.0f;
#pragma unroll
            for (int ib = 0; ib < 4; ++ib)
#pragma unroll
                for (int hq = 0; hq < 2; ++hq) {
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(
                            kq + ib * 16384 + sw128(r, 4 * hq + q4));
                        if (r >= 64) {
                            w[4 * q4] = to_tf32_fast(qs * __uint_as_float(v.x));
                            w[4 * q4 + 1] = to_tf32_fast(qs * __uint_as_float(v.y));
                            w[4 * q4 + 2] = to_tf32_fast(qs * __uint_as_float(v.z));
                            w[4 * q4 + 3] = to_tf32_fast(qs * __uint_as_float(v.w));
                        } else {
                            w[4 * q4] = v.x;
                            w[4 * q4 + 1] = v.y;
                            w[4 * q4 + 2] = v.z;
                            w[4 * q4 + 3] = v.w;
                        }
                    }
                    tmem_st16(lane_base + TM_KQ + 32 * ib + 16 * hq, w);
                }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(B_KQE + b)); // this thread is done with the K/Q tiles
            mbar_arrive(bar(B_TR + b));  // chunk cn's A operands are in TMEM
            if (cn >= 1)
                ok = emit_y(cn - 1);
        }
        if (ok && a.NC > 0)
            ok = emit_y(a.NC - 1);
        if (tid == 256 && y_pending)
            bulk_wait_all();
        if (!ok)
            *abort_s = 1;
    } else {
        // ------------------------------- chain --------------------------------
        constexpr uint32_t ID1 = idesc_tf32(128, R, 0, 1);
        constexpr uint32_t ID2 = idesc_tf32(128, R, 0, 1);
        const uint32_t sb = smem_u32(smem + S_SB), xb = smem_u32(smem + S_XB),
                       ub = smem_u32(smem + S_UB), u2 = smem_u32(smem + S_U2);
        auto chain_and = [](bool v) {
            uint32_t res;
            asm volatile("{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\n"
                         "bar.red.and.pred q, 1, 256, p;\nselp.u32 %0, 1, 0, q;\n}\n"
                         : "=r"(res)
                         : "r"((uint32_t)v)
                         : "memory");
            return res != 0;
        };
        int mma_pending = 0, mma3_issued = 0, mma_phase = 0;
        bool ok = true;
        for (int c = 0; c < a.NC && ok; ++c) {
            const int s = c & 1;
            const uint32_t d1 = tmem + TM_D1 + 32 * (uint32_t)s;
            const uint32_t atm_t = tmem + TM_ATM + 64 * (uint32_t)s;
            const uint32_t kt_t = tmem + TM_KT + 64 * (uint32_t)s;
            const float *fac = reinterpret_cast<const float *>(smem + S_FAC + s * FAC_BYTES);
            // 1. MMA1: D1 = [K; diag(scale b) Q] S_0^T once the copier has
            // chunk c's operands and the output rows of chunk c-2 are out
            ok = chain_and(mbar_wait(bar(B_TR + s), (c >> 1) & 1, abort_s) &&
                           (c < 2 || mbar_wait(bar(B_D1F + s), ((c >> 1) - 1) & 1, abort_s)));
            if (!ok)
                break;
            if (warp == 0) {
                tc_fence_after();
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < 16; ++kk)
                        mma_ts_tf32(d1, tmem + TM_KQ + kk * 8,
                                    sdesc_mn32(sb + kk * 1024, 8192, 512), ID1, kk > 0);
                    mma_commit(bar(B_MMA));
                }
                __syncwarp();
            }
            mma_pending = 1;
            ok = chain_and(mbar_wait(bar(B_VFF + s), (c >> 1) & 1, abort_s) &&
                           mbar_wait(bar(B_MMA), mma_phase & 1, abort_s));
            ++mma_phase;
            mma_pending = 0;
            if (!ok)
                break;
            tc_fence_after();
            if (tid == 0)
                mbar_arrive(bar(B_KQFREE)); // MMA1 has read the [K; Q] columns
            // 2. X' = V - b X (rows 0-63)
            if (r < 64) {
                float d[16];
                tmem_ld16(lane_base + TM_D1 + 32 * s + 16 * hc, d);
                const int t = r;
                const float bt = fac[t];
                const uint8_t *vrow = smem + S_V + s * 8192;
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const float4 v = *reinterpret_cast<const float4 *>(vrow + sw128(t, 4 * hc + q4));
                    uint4 x;
                    x.x = to_tf32_fast(fmaf(-bt, d[4 * q4], v.x));
                    x.y = to_tf32_fast(fmaf(-bt, d[4 * q4 + 1], v.y));
                    x.z = to_tf32_fast(fmaf(-bt, d[4 * q4 + 2], v.z));
                    x.w = to_tf32_fast(fmaf(-bt, d[4 * q4 + 3], v.w));
                    const int q8 = 4 * hc + q4; // 16-byte unit of the 128-byte row
                    *reinterpret_cast<uint4 *>(smem + S_XB + sw128_32b(t, q8 >> 1) +
                                               (q8 & 1) * 16) = x;
                }
            }
            fence_async_smem();
            tc_fence_before();
            chain_and(true);
            // 3. MMA2: U = T'' X'
            if (warp == 0) {
                tc_fence_after();
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        mma_ts_tf32(tmem + TM_D2, atm_t + kk * 8,
                                    sdesc_mn32(xb + kk * 1024, 8192, 512), ID2, kk > 0);
                    mma_commit(bar(B_MMA));
                }
                __syncwarp();
            }
            mma_pending = 1;
            ok = chain_and(mbar_wait(bar(B_MMA), mma_phase & 1, abort_s));
            ++mma_phase;
            mma_pending = 0;
            if (!ok)
                break;
            tc_fence_after();
            // 4. U and diag(e) U as MN-major operands (rows 0-63)
            if (r < 64) {
                float u[16];
                tmem_ld16(lane_base + TM_D2 + 16 * hc, u);
                const int t = r;
                const float et = fac[64 + t];
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    uint4 x, x2;
                    x.x = to_tf32_fast(u[4 * q4]);
                    x.y = to_tf32_fast(u[4 * q4 + 1]);
                    x.z = to_tf32_fast(u[4 * q4 + 2]);
                    x.w = to_tf32_fast(u[4 * q4 + 3]);
                    x2.x = to_tf32_fast(et * u[4 * q4]);
                    x2.y = to_tf32_fast(et * u[4 * q4 + 1]);
                    x2.z = to_tf32_fast(et * u[4 * q4 + 2]);
                    x2.w = to_tf32_fast(et * u[4 * q4 + 3]);
                    const int q8 = 4 * hc + q4;
                    const uint32_t off = sw128_32b(t, q8 >> 1) + (q8 & 1) * 16;
                    *reinterpret_cast<uint4 *>(smem + S_UB + off) = x;
                    *reinterpret_cast<uint4 *>(smem + S_U2 + off) = x2;
                }
            }
            fence_async_smem();
            tc_fence_before();
            chain_and(true);
            // 5. MMA4 (warp 0): K^T diag(e) U, the state update; MMA3 (warp 4):
            // M U accumulated onto D1 rows 64-127, the output (rows 0-63 of D1,
            // X, are no longer needed)
            if (warp == 0 || warp == 4) {
                tc_fence_after();
                if (elect_one()) {
                    if (warp == 0) {
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk)
                            mma_ts_tf32(tmem + TM_D4, kt_t + kk * 8,
                                        sdesc_mn32(u2 + kk * 1024, 8192, 512), ID2, kk > 0);
                        mma_commit(bar(B_MMA));
                    } else {
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk)
                            mma_ts_tf32(d1, atm_t + kk * 8, sdesc_mn32(ub + kk * 1024, 8192, 512),
                                        ID2, 1);
                        mma_commit(bar(B_MMA3));
                    }
                }
                __syncwarp();
            }
            mma_pending = 1;
            ++mma3_issued;
            ok = chain_and(mbar_wait(bar(B_MMA), mma_phase & 1, abort_s));
            ++mma_phase;
            mma_pending = 0;
            if (!ok)
                break;
            tc_fence_after();
            // 6. S = b_C S + D4 (FP32 registers); TF32 copy for the next MMA1
            {
                float d[16];
                tmem_ld16(lane_base + TM_D4 + 16 * hc, d);
                const float bC = fac[128];
#pragma unroll
                for (int jj = 0; jj < 16; ++jj)
                    S[jj] = fmaf(bC, S[jj], d[jj]);
                store_s();
            }
            fence_async_smem();
            tc_fence_before();
            chain_and(true);
            if (tid == 0)
                mbar_arrive(bar(B_VFE + s)); // V / factors of chunk c are no longer read
        }
        if (!ok) {
            *abort_s = 1;
            volatile int none = 0;
            if (mma_pending)
                mbar_wait(bar(B_MMA), mma_phase & 1, &none, 100000000ull);
            if (mma3_issued > 0) // the last MMA3 (the copier may not have waited it)
                mbar_wait(bar(B_MMA3), (mma3_issued - 1) & 1, &none, 100000000ull);
        } else {
            float *so = a.state_out + (((size_t)n * a.H + h) * SK + j0 + 16 * hc) * SK + r;
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
                so[(size_t)jj * SK] = S[jj];
        }
    }

    // ---- teardown ----
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && *abort_s)
        atomicExch(a.err, 1);
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TM_COLS);
    }
}

// ---------------------------------------------------------------------------
// host side

size_t gdn_chunk_workspace(int T, int H, int n_seq, int slots) {
    const int nc = gc::n_chunks(T, slots);
    if (nc < 2) // the per-token kernel runs: no workspace
        return 0;
    const size_t units = (size_t)nc * H * n_seq;
    size_t b = units * (gc::ATM_FLOATS + gc::FAC_FLOATS) * 4; // [T''; M], factors
    b += 256;                                                  // error flag
    if (nc * gc::C < T)
        b += (size_t)H * n_seq * gc::SK * gc::SK * 4; // state handed to the per-token kernel
    return b;
}

static bool encode_map(CUtensorMap *m, const void *base, int rank, const cuuint64_t *dims,
                       const cuuint64_t *strides, const cuuint32_t *box) {
    auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
    if (!enc)
        return false;
    cuuint32_t es[4] = {1, 1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<void *>(base), dims, strides,
               box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// [S, heads, T, seqs] fp32 rows, boxes of 32 elements x 64 tokens.
static bool encode_rows(CUtensorMap *m, const float *p, int heads, int T, int seqs, int64_t nb1,
                        int64_t nb2, int64_t nb3) {
    const cuuint64_t dims[4] = {(cuuint64_t)gc::SK, (cuuint64_t)heads, (cuuint64_t)T,
                                (cuuint64_t)seqs};
    const cuuint64_t strides[3] = {(cuuint64_t)nb1, (cuuint64_t)nb2, (cuuint64_t)nb3};
    const cuuint32_t box[4] = {32, 1, (cuuint32_t)gc::C, 1};
    return encode_map(m, p, 4, dims, strides, box);
}

bool gdn_chunk_eligible(const GdnArgs &a) {
    const uintptr_t bits =
        reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
        reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.dst) |
        (uintptr_t)a.q_nb1 | (uintptr_t)a.q_nb2 |
        (uintptr_t)a.q_nb3 | (uintptr_t)a.k_nb1 | (uintptr_t)a.k_nb2 | (uintptr_t)a.k_nb3 |
        (uintptr_t)a.v_nb1 | (uintptr_t)a.v_nb2 | (uintptr_t)a.v_nb3;
    return (bits & 15) == 0 && gc::n_chunks(a.T, a.slots) >= 2 && a.H <= 65535 &&
           a.n_seq <= 65535 && tensor_map_encoder() != nullptr;
}

cudaError_t launch_gdn_chunked(const GdnArgs &a, void *ws, size_t ws_bytes, cudaStream_t st) {
    using namespace gc;
    const int nc = n_chunks(a.T, a.slots);
    const size_t units = (size_t)nc * a.H * a.n_seq;
    if (ws_bytes < gdn_chunk_workspace(a.T, a.H, a.n_seq, a.slots) || units * 128 > 0x7fffffffull)
        return cudaErrorInvalidValue;
    uint8_t *w = static_cast<uint8_t *>(ws);
    GdnChunkArgs c;
    c.g = a.g;
    c.beta = a.beta;
    c.state = a.state;
    c.g_nb1 = a.g_nb1; c.g_nb2 = a.g_nb2; c.g_nb3 = a.g_nb3;
    c.b_nb1 = a.b_nb1; c.b_nb2 = a.b_nb2; c.b_nb3 = a.b_nb3;
    c.s_nb1 = a.s_nb1; c.s_nb2 = a.s_nb2; c.s_nb3 = a.s_nb3;
    c.atm = reinterpret_cast<float *>(w);
    c.fac = reinterpret_cast<float *>(w + units * ATM_FLOATS * 4);
    c.err = reinterpret_cast<int *>(w + units * (ATM_FLOATS + FAC_FLOATS) * 4);
    const bool tail = nc * C < a.T;
    float *handoff = reinterpret_cast<float *>(w + units * (ATM_FLOATS + FAC_FLOATS) * 4 + 256);
    c.dst = a.dst;
    c.state_out = tail ? handoff : a.dst + (size_t)SK * a.H * a.T * a.n_seq; // snapshot slot 0
    c.H = a.H;
    c.H_k = a.H_k;
    c.h_off = a.h_off;
    c.T = a.T;
    c.n_seq = a.n_seq;
    c.rq3 = a.rq3;
    c.rk3 = a.rk3;
    c.NC = nc;
    c.scale = a.scale;

    CUtensorMap kmap, qmap, vmap, amap, ymap;
    const int seq_k = a.n_seq / a.rk3, seq_q = a.n_seq / a.rq3;
    if (!encode_rows(&kmap, a.k, a.H_k, a.T, seq_k, a.k_nb1, a.k_nb2, a.k_nb3) ||
        !encode_rows(&qmap, a.q, a.H_k, a.T, seq_q, a.q_nb1, a.q_nb2, a.q_nb3) ||
        !encode_rows(&vmap, a.v, a.H, a.T, a.n_seq, a.v_nb1, a.v_nb2, a.v_nb3) ||
        !encode_rows(&ymap, a.dst, a.H, a.T, a.n_seq, (int64_t)SK * 4, (int64_t)a.H * SK * 4,
                     (int64_t)a.T * a.H * SK * 4))
        return cudaErrorNotSupported;
    {
        const cuuint64_t dims[2] = {64, (cuuint64_t)units * 128};
        const cuuint64_t strides[1] = {256};
        const cuuint32_t box[2] = {32, 128};
        if (!encode_map(&amap, c.atm, 2, dims, strides, box))
            return cudaErrorNotSupported;
    }
    cudaError_t e = cudaMemsetAsync(c.err, 0, sizeof(int), st);
    if (e != cudaSuccess)
        return e;
    static std::atomic<unsigned long long> prep_attr{0}, scan_attr{0};
    if ((e = set_smem_limit((const void *)gdn_chunk_prep_kernel, P_BYTES, prep_attr)) !=
            cudaSuccess ||
        (e = set_smem_limit((const void *)gdn_chunk_scan_kernel, S_BYTES, scan_attr)) !=
            cudaSuccess)
        return e;
    gdn_chunk_prep_kernel<<<dim3((unsigned)(nc * a.H), 1, (unsigned)a.n_seq), PREP_NT,
                            P_BYTES, st>>>(kmap, qmap, c);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return e;
    gdn_chunk_scan_kernel<<<dim3(SK / R, (unsigned)a.H, (unsigned)a.n_seq), SCAN_NT, S_BYTES,
                            st>>>(kmap, qmap, vmap, amap, ymap, c);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return e;
    if (tail) {
        // the last tokens (the snapshot slots) one at a time from the handed-off state
        GdnArgs r = a;
        r.t_begin = nc * C;
        r.state = handoff;
        r.s_nb1 = SK * 4;
        r.s_nb2 = (int64_t)SK * SK * 4;
        r.s_nb3 = (int64_t)a.H * SK * SK * 4;
        return launch_gdn(r, st);
    }
    return cudaSuccess;
}

} // namespace xq
