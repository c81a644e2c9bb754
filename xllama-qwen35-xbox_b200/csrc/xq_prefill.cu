// Causal / masked prefill attention on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), F16 K/V, F32 Q and output (ggml FLASH_ATTN_EXT with
// many queries; semantics as ggml-cpu's one_chunk path: q rounded to f16,
// s = scale * q.k + mask, masked -inf entries skipped, rows with no live key
// give 0; the reference's bring-up kernel shaders/rkva/rkva_flash_attn.hlsl:61-125
// states the same online-softmax contract).
//
// Q8_0 / Q4_0 caches (the reference's product configuration: a quantized KV
// cache forces flash attention on, src/bridge/session.cpp:600-607, and every
// prompt chunk reaches this op).  ggml-cpu takes them through one_chunk at any
// query count (patches/0008-flash-attn-query-consistency.patch:18-35): q is
// quantized to Q8_0 (the K vec_dot type), K.q is the integer block dot times
// both block scales, V is dequantized to f32.  Here a pre-pass
// (kv_to_f16_kernel) widens every K and V row once into the workspace -- the
// exact dequantized value code * f32(d), rounded once to f16 -- and the
// kernel below (QQ = true) quantizes each q row to Q8_0 exactly as ggml does
// (d = amax / 127 rounded to f16, codes roundf(x / d)) before rounding the
// exact q code * d to f16 for the tensor core.  Every operand is therefore
// ggml's value to within one f16 rounding (2^-11 relative), the same
// precision as the f16 probabilities P; the products and sums run in fp32 in
// TMEM.  (Exact int8 block sums would need one int32 TMEM accumulator per
// 32-dim block per key tile -- 8 x 64 columns at D = 256 -- beside the 256
// columns of O: more than the 512 columns an SM has.)
//
// One CTA = 128 query rows of one head (TMEM lane r <-> query row r).
//   warp 0      TMA producer: K_j, V_j tiles (64 keys x D, SW128) into a
//               6-slot (D=256) / 8-slot ring, completion on mbarriers (expect_tx)
//   warp 1      TMEM allocator + MMA issuer (one lane):
//                 S_j = Q K_j^T   (TS, M=128, N=64, K=D; A = Q in TMEM, so
//                                  only K is read from shared memory; S in
//                                  TMEM, 2 buffers)
//                 O  += P_j V_j   (TS, A = P_j in TMEM, B = V_j MN-major, N=D)
//               issue order S_0, S_1, PV_0, S_2, PV_1, ... so the tensor
//               core computes S_{j+1} while the softmax works on S_j
//   warps 4-7   softmax: tcgen05.ld S_j, mask, running max in the log2
//               domain, p = 2^(s - m_used) written back to TMEM as f16 (the
//               A operand of PV_j), row sums; O is rescaled in TMEM only when
//               the running max grows by more than 2^8 (lazy rescale, exact:
//               the same m_used scales both O and l); epilogue O / l
//   warps 4-7   first store their query rows (F32 -> f16 pairs) into TMEM
// A 128x64 block classification of the mask (all -inf / all 0 / mixed),
// computed by a pre-pass over the mask, lets every role skip dead blocks and
// read mask values only for mixed blocks.
//
// Every mbarrier wait is bounded: on timeout the kernel records an error code,
// stops issuing work, drains its own copies and MMAs with bounded waits,
// frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <float.h>
#include <math.h>

#include "xq_common.cuh"
#include "xq_internal.h"
#include "xq_tc.cuh"

namespace xq {

namespace pf {

constexpr int BM = 128;   // query rows per CTA
constexpr int BN = 64;    // keys per tile
// K/V ring slots (one K or V tile each): the whole shared memory goes to the ring
__host__ __device__ constexpr int nslot(int D) { return D == 256 ? 6 : 8; }
constexpr int NT = 256;   // threads
using namespace tc; // mbarrier / TMA / tcgen05 helpers

} // namespace pf

struct PrefillArgs {
    const uint8_t *q;
    int64_t q_nb1, q_nb2, q_nb3;
    const uint8_t *mask;
    int64_t m_nb1, m_nb2, m_nb3;
    int m_ne2, m_ne3;
    const uint8_t *block_map; // [m3][m2][n_qt][n_kt]: 0 dead, 1 all-zero, 2 mixed
    float *dst;
    int *err;
    int n_q, n_head, n_head_kv, n_seq, n_kv, rk3;
    int n_qt, n_kt;
    float scale_log2; // scale * log2(e)
};

template <int D, bool QQ>
__global__ void __launch_bounds__(pf::NT, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const PrefillArgs a) {
    using namespace pf;
    constexpr int NSLOT = nslot(D);
    constexpr int TBYTES = BN * D * 2;            // one K or V tile
    constexpr int NBOX = D / 64;                  // 64-element (128 B) column boxes
    constexpr uint32_t TM_O = 0;                  // O: columns [0, D)
    constexpr uint32_t TM_S = D;                  // S buffers: [D, D + 2*BN)
    constexpr uint32_t TM_Q = D + 2 * BN;         // Q as f16 pairs: [TM_Q, TM_Q + D/2)
    constexpr uint32_t TM_COLS = 512;
    static_assert(TM_Q + D / 2 <= TM_COLS, "TMEM columns");
    constexpr uint32_t ID_QK = idesc(BM, BN, 0, 0);
    constexpr uint32_t ID_PV = idesc(BM, D, 0, 1);
    static_assert(D == 128 || D == 256, "head dim");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned by an offset on the shared array (accesses stay
    // shared-memory accesses; an integer round trip leaves generic addresses)
    uint8_t *smem =
        smem_raw + ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) &
                    1023u);
    uint8_t *ring = smem;
    uint64_t *bars = reinterpret_cast<uint64_t *>(ring + NSLOT * TBYTES);
    // bars: full[NSLOT], empty[NSLOT], s_full[2], p_full[2], o_done, drain, q_ready
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * NSLOT + 7);
    volatile int *abort_s = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int per_q = a.n_head * a.n_seq;
    const int qt = a.n_qt - 1 - (int)(blockIdx.x / per_q); // heaviest tiles first
    const int rem = (int)(blockIdx.x % per_q);
    const int h = rem % a.n_head, s = rem / a.n_head;
    const int kvh = h / (a.n_head / a.n_head_kv);
    const int q0 = qt * BM;
    const uint8_t *bmap = a.block_map +
                          ((size_t)((s % a.m_ne3) * a.m_ne2 + (h % a.m_ne2)) * a.n_qt + qt) * a.n_kt;

    auto bar = [&](int i) { return smem_u32(bars + i); };
    const int B_FULL = 0, B_EMPTY = NSLOT, B_S = 2 * NSLOT, B_P = 2 * NSLOT + 2,
              B_O = 2 * NSLOT + 4, B_DRAIN = 2 * NSLOT + 5, B_Q = 2 * NSLOT + 6;

    if (tid == 0) {
        for (int i = 0; i < NSLOT; ++i) {
            mbar_init(bar(B_FULL + i), 1);
            mbar_init(bar(B_EMPTY + i), 1);
        }
        mbar_init(bar(B_S), 1);
        mbar_init(bar(B_S + 1), 1);
        mbar_init(bar(B_P), 128);
        mbar_init(bar(B_P + 1), 128);
        mbar_init(bar(B_O), 1);
        mbar_init(bar(B_DRAIN), 1);
        mbar_init(bar(B_Q), 128);
        *abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // number of live key tiles for this query tile (same list in every role)
    int n_live = 0;
    for (int kt = 0; kt < a.n_kt; ++kt)
        n_live += bmap[kt] != 0;

    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            int j = 0, issued = 0; // K/V tiles issued so far
            for (int kt = 0; kt < a.n_kt && !*abort_s; ++kt) {
                if (!bmap[kt])
                    continue;
                for (int half = 0; half < 2; ++half) { // 0: K_j, 1: V_j
                    const int n = 2 * j + half, slot = n % NSLOT, use = n / NSLOT;
                    if (use > 0 && !mbar_wait(bar(B_EMPTY + slot), (use - 1) & 1, abort_s)) {
                        *abort_s = 1;
                        break;
                    }
                    const uint32_t dst = smem_u32(ring + slot * TBYTES);
                    mbar_expect_tx(bar(B_FULL + slot), TBYTES);
                    const CUtensorMap *m = half ? &vmap : &kmap;
#pragma unroll
                    for (int b = 0; b < NBOX; ++b)
                        tma_load_4d(dst + b * (BN * 128), m, 64 * b, kt * BN, kvh, s / a.rk3,
                                    bar(B_FULL + slot));
                    ++issued;
                }
                ++j;
            }
            if (*abort_s) {
                // our copies still in flight land on their full barriers
                volatile int none = 0;
                for (int n = issued - NSLOT < 0 ? 0 : issued - NSLOT; n < issued; ++n)
                    mbar_wait(bar(B_FULL + n % NSLOT), (n / NSLOT) & 1, &none, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // -------------------------------- MMA ---------------------------------
        // The whole warp runs the schedule (its waits, descriptors and TMEM
        // addresses stay warp-uniform); one elected lane issues each MMA and
        // commit.  Shared-memory descriptors are precomputed for ring slot 0
        // and offset by constants (the 14-bit address field cannot carry: shared
        // memory is below 256 KB).
        if (n_live > 0) {
            const uint64_t dk0 = sdesc(smem_u32(ring), 16, 1024);       // K: K-major
            const uint64_t dv0 = sdesc(smem_u32(ring), BN * 128, 1024); // V: MN-major
            constexpr uint64_t SLOT_STEP = TBYTES >> 4;
            const bool leader = elect_one();
            auto wait_all = [&](int b, uint32_t parity) {
                return __all_sync(0xffffffffu, mbar_wait(bar(b), parity, abort_s));
            };
            auto issue_s = [&](int j) -> bool {
                const int n = 2 * j, slot = n % NSLOT, use = n / NSLOT;
                if (!wait_all(B_FULL + slot, use & 1))
                    return false;
                // S buffer j%2 is free: PV_{j-2} (which read P_{j-2} there) was
                // issued before this point and the tensor pipe runs in order.
                tc_fence_after();
                const uint64_t db0 = dk0 + (uint64_t)slot * SLOT_STEP;
                const uint32_t d_tm = tmem + TM_S + (j & 1) * BN;
                if (leader) {
                    // A = Q from TMEM (8 columns = 16 f16 per K step), B = K from
                    // smem: step kk at byte (kk / 4) * BN * 128 + (kk % 4) * 32
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk)
                        mma_ts(d_tm, tmem + TM_Q + kk * 8,
                               db0 + (uint64_t)((kk / 4) * (BN * 128 / 16) + (kk & 3) * 2),
                               ID_QK, kk > 0);
                    mma_commit(bar(B_S + (j & 1)));
                    mma_commit(bar(B_EMPTY + slot));
                }
                __syncwarp();
                return true;
            };
            // Q rows are in TMEM once all 128 softmax threads arrived
            bool ok = wait_all(B_Q, 0);
            tc_fence_after();
            ok = ok && issue_s(0);
            for (int j = 0; ok && j < n_live; ++j) {
                if (j + 1 < n_live)
                    ok = issue_s(j + 1);
                if (!ok)
                    break;
                // PV_j: wait for P_j from the softmax warps and V_j from TMA
                const int n = 2 * j + 1, slot = n % NSLOT, use = n / NSLOT;
                if (!wait_all(B_P + (j & 1), (j >> 1) & 1) || !wait_all(B_FULL + slot, use & 1)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t db0 = dv0 + (uint64_t)slot * SLOT_STEP;
                const uint32_t p_tm = tmem + TM_S + (j & 1) * BN;
                if (leader) {
                    // B = V rows [16kk, 16kk+16) x all D columns, MN-major SW128:
                    // 64-column boxes BN*128 bytes apart (LBO), 8-row groups
                    // 1024 bytes apart (SBO); step kk at byte kk * 2048
#pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk)
                        mma_ts(tmem + TM_O, p_tm + kk * 8, db0 + (uint64_t)(kk * 128), ID_PV,
                               (j > 0 || kk > 0));
                    mma_commit(bar(B_O));
                    mma_commit(bar(B_EMPTY + slot));
                }
                __syncwarp();
            }
            if (!ok && lane == 0)
                *abort_s = 1;
            // every tcgen05.mma issued above has completed once this commits
            if (leader)
                mma_commit(bar(B_DRAIN));
            __syncwarp();
            volatile int none = 0;
            mbar_wait(bar(B_DRAIN), 0, &none, 100000000ull);
        }
    } else if (warp >= 4) {
        // ------------------------------ softmax -------------------------------
        const int r = tid - 128;                 // query row in tile == TMEM lane
        const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp - 4)) << 16);
        const int qrow = q0 + r;
        const uint8_t *mrow = a.mask ? a.mask + (int64_t)min(qrow, a.n_q - 1) * a.m_nb1 +
                                           (int64_t)(h % a.m_ne2) * a.m_nb2 +
                                           (int64_t)(s % a.m_ne3) * a.m_nb3
                                     : nullptr;
        {
            // this thread's query row -> f16 pairs in TMEM lane r (the A operand of S);
            // with QQ first through ggml's Q8_0 quantizer (quantize_row_q8_0_ref)
            const float4 *src = reinterpret_cast<const float4 *>(
                a.q + (int64_t)min(qrow, a.n_q - 1) * a.q_nb1 + (int64_t)h * a.q_nb2 +
                (int64_t)s * a.q_nb3);
#pragma unroll 1
            for (int c0 = 0; c0 < D; c0 += 64) {
                float x[64];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float4 v = qrow < a.n_q ? src[c0 / 4 + i] : make_float4(0, 0, 0, 0);
                    x[4 * i] = v.x;
                    x[4 * i + 1] = v.y;
                    x[4 * i + 2] = v.z;
                    x[4 * i + 3] = v.w;
                }
                if constexpr (QQ) {
#pragma unroll
                    for (int hb = 0; hb < 2; ++hb) { // two 32-element Q8_0 blocks
                        float amax = 0.0f;
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            amax = fmaxf(amax, fabsf(x[32 * hb + i]));
                        const float d = amax / 127.0f;
                        const float id = d != 0.0f ? 1.0f / d : 0.0f;
                        const float dh = __half2float(__float2half_rn(d)); // the stored scale
#pragma unroll
                        for (int i = 0; i < 32; ++i) // code * scale: exact in fp32
                            x[32 * hb + i] = roundf(x[32 * hb + i] * id) * dh;
                    }
                }
                uint32_t w[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const __half2 hh = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
                    w[i] = *reinterpret_cast<const uint32_t *>(&hh);
                }
                tmem_st32(lane_base + TM_Q + c0 / 2, w);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(B_Q));
        }
        float m_used = -INFINITY, l = 0.0f;
        int j = 0;
        bool ok = true;
        for (int kt = 0; kt < a.n_kt && ok; ++kt) {
            const int cls = bmap[kt];
            if (!cls)
                continue;
            // warp-uniform outcome: the tcgen05.ld/st below are warp-collective
            if (!__all_sync(0xffffffffu, mbar_wait(bar(B_S + (j & 1)), (j >> 1) & 1, abort_s))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t s_tm = lane_base + TM_S + (j & 1) * BN;
            float sv[64];
            {
                float t[32];
                tmem_ld32(s_tm, t);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    sv[i] = t[i];
                tmem_ld32(s_tm + 32, t);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    sv[32 + i] = t[i];
            }
            const int kbase = kt * BN;
            if (kbase + BN > a.n_kv) { // last tile: keys past n_kv are dead
#pragma unroll
                for (int i = 0; i < 64; ++i)
                    if (kbase + i >= a.n_kv)
                        sv[i] = -INFINITY;
            }
            // mt: the tile's row max in the log2 domain; p = 2^(sv * c - m_used)
            float c = 1.0f;
            const bool raw = cls == 1 && a.scale_log2 > 0.0f;
            if (!raw) {
                const __half *mp = reinterpret_cast<const __half *>(mrow) + kbase;
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    float x = sv[i] * a.scale_log2;
                    if (cls == 2 && kbase + i < a.n_kv) {
                        const float mv = __half2float(mp[i]);
                        x = mv == -INFINITY ? -INFINITY : x + mv * 1.4426950408889634f;
                    }
                    sv[i] = sv[i] == -INFINITY ? -INFINITY : x;
                }
            } else {
                c = a.scale_log2; // scale > 0: the max of the raw scores, scaled once
            }
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int i = 0; i < 64; i += 4) {
                m4[0] = fmaxf(m4[0], sv[i]);
                m4[1] = fmaxf(m4[1], sv[i + 1]);
                m4[2] = fmaxf(m4[2], sv[i + 2]);
                m4[3] = fmaxf(m4[3], sv[i + 3]);
            }
            const float mraw = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            const float mt = mraw == -INFINITY ? -INFINITY : mraw * c;
            // lazy rescale: move m_used only when the max grew by > 8 (log2); the
            // decision is per row, the TMEM traffic is warp-collective
            const bool grow = mt > m_used + 8.0f || (m_used == -INFINITY && mt != -INFINITY);
            const float mnew = grow ? mt : m_used;
            const float f = (!grow || m_used == -INFINITY) ? (grow ? 0.0f : 1.0f)
                                                           : ex2(m_used - mnew);
            if (__any_sync(0xffffffffu, grow && j > 0 && m_used != -INFINITY)) {
                // O holds PV_0..PV_{j-1}; wait for PV_{j-1} before scaling
                if (!__all_sync(0xffffffffu, mbar_wait(bar(B_O), (j - 1) & 1, abort_s))) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll 1
                for (int cc = 0; cc < D; cc += 32) {
                    float o[32];
                    tmem_ld32(lane_base + TM_O + cc, o);
                    uint32_t w[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        w[i] = __float_as_uint(o[i] * f);
                    tmem_st32(lane_base + TM_O + cc, w);
                }
            }
            l *= f;
            m_used = mnew;
            // p = 2^(sv * c - m_used): -inf scores give 2^-inf = 0 (m_used is
            // finite whenever a live key exists; a row with none keeps 0)
            const float mu = m_used == -INFINITY ? 0.0f : m_used;
            const float2 c2 = make_float2(c, c), nm2 = make_float2(-mu, -mu);
            uint32_t pk[32];
            float2 lt2 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const float2 x = __ffma2_rn(make_float2(sv[2 * i], sv[2 * i + 1]), c2, nm2);
                const float2 pp = make_float2(ex2(x.x), ex2(x.y));
                lt2 = __fadd2_rn(lt2, pp);
                const __half2 hp = __floats2half2_rn(pp.x, pp.y);
                pk[i] = *reinterpret_cast<const uint32_t *>(&hp);
            }
            const float lt = lt2.x + lt2.y;
            l += lt;
            tmem_st32(s_tm, pk);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(B_P + (j & 1)));
            ++j;
        }
        // ---- epilogue: O / l ----
        if (ok && n_live > 0) {
            // the MMA thread's last commit (B_DRAIN, one phase) covers every MMA;
            // B_O's parity alone cannot tell PV_{n-1} from a pending PV_{n-2}
            ok = __all_sync(0xffffffffu, mbar_wait(bar(B_DRAIN), 0, abort_s));
            tc_fence_after();
        }
        if (!ok) {
            *abort_s = 1;
        } else {
            const float inv = l == 0.0f ? 0.0f : 1.0f / l;
            float *out = a.dst + ((int64_t)(s * a.n_q + qrow) * a.n_head + h) * D;
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
                float o[32];
                if (n_live > 0)
                    tmem_ld32(lane_base + TM_O + c, o); // all lanes: warp-collective
                if (qrow < a.n_q) {
#pragma unroll
                    for (int i = 0; i < 32; i += 4) {
                        float4 v = n_live > 0 ? make_float4(o[i] * inv, o[i + 1] * inv,
                                                            o[i + 2] * inv, o[i + 3] * inv)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
                        *reinterpret_cast<float4 *>(out + c + i) = v;
                    }
                }
            }
        }
    }

    // ---- teardown: all roles done; drain on abort; free TMEM ----
    tc_fence_before();
    __syncthreads();
    if (*abort_s && tid == 0)
        atomicExch(a.err, 1);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                     "r"(TM_COLS));
    }
}

// Mask block classes for BM x BN blocks: 0 all -inf, 1 all 0, 2 otherwise.
// One CTA per block.  Where the block's rows are whole 16-byte runs (a full
// block of columns, 16-byte aligned rows) each thread reads half a row with
// four 16-byte loads and classifies the f16 bit patterns (-inf = 0xFC00,
// zero = +0 or -0); elsewhere element by element.  The mask is read once, at
// the HBM rate.
__global__ void __launch_bounds__(256) mask_block_map_kernel(
    const uint8_t *mask, int64_t nb1, int64_t nb2, int64_t nb3, int m2, int n_q, int n_kv,
    int n_qt, int n_kt, int vec, uint8_t *map) {
    const int kt = blockIdx.x, qt = blockIdx.y, plane = blockIdx.z;
    const int i2 = plane % m2, i3 = plane / m2;
    const uint8_t *base = mask + (int64_t)i2 * nb2 + (int64_t)i3 * nb3;
    const int r0 = qt * pf::BM, c0 = kt * pf::BN;
    const int rows = min(pf::BM, n_q - r0);
    int all_inf = 1, all_zero = 1;
    if (vec && c0 + pf::BN <= n_kv) {
        const int r = threadIdx.x >> 1;
        if (r < rows) {
            const uint4 *p = reinterpret_cast<const uint4 *>(base + (int64_t)(r0 + r) * nb1 +
                                                             2 * c0 + 64 * (threadIdx.x & 1));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint4 w = __ldcs(p + i);
                const uint32_t x[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    all_inf &= x[j] == 0xFC00FC00u;
                    all_zero &= (x[j] & 0x7FFF7FFFu) == 0u;
                }
            }
        }
    } else {
        for (int e = threadIdx.x; e < pf::BM * pf::BN; e += blockDim.x) {
            const int r = r0 + e / pf::BN, c = c0 + e % pf::BN;
            if (r >= n_q || c >= n_kv)
                continue;
            const uint16_t h =
                *reinterpret_cast<const uint16_t *>(base + (int64_t)r * nb1 + 2 * (int64_t)c);
            all_inf &= h == 0xFC00u;
            all_zero &= (h & 0x7FFFu) == 0u;
        }
    }
    all_inf = __syncthreads_and(all_inf);
    all_zero = __syncthreads_and(all_zero);
    if (threadIdx.x == 0) {
        // a block entirely beyond n_kv is dead as well
        const bool beyond = c0 >= n_kv;
        map[((size_t)plane * n_qt + qt) * n_kt + kt] =
            (beyond || all_inf) ? 0 : (all_zero ? 1 : 2);
    }
}

__global__ void fill_map_kernel(uint8_t *map, size_t n, int n_kt, int n_kv) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        map[i] = ((int)(i % n_kt) * pf::BN < n_kv) ? 1 : 0;
}

// Q8_0 / Q4_0 K or V rows (a ggml view) -> contiguous f16 rows [seq][kv head]
// [row][D]: value = code * f32(d) as ggml's to_float computes it (exact in
// fp32: <= 8-bit code times an 11-bit scale), then one round-to-nearest to
// f16.  One warp per row: the row's 4-byte words are read coalesced into
// shared memory, then each lane widens D / 32 consecutive elements and
// stores them with one 16- (D = 256) or 8-byte (D = 128) store.  Rows must
// be 4-byte aligned (every Q8_0 / Q4_0 row of a multiple of 32 elements is a
// multiple of 4 bytes); kv_to_f16_u16_kernel below takes 2-byte aligned views.
template <int T, int D>
__global__ void __launch_bounds__(256) kv_to_f16_kernel(const uint8_t *__restrict__ src,
                                                        int64_t nb1, int64_t nb2, int64_t nb3,
                                                        int n_kv, int n_hkv,
                                                        __half *__restrict__ dst) {
    constexpr int BB = T == kQ8 ? 34 : 18, REC = D / 32 * BB, WORDS = REC / 4, EPL = D / 32;
    static_assert(REC % 4 == 0, "rows of whole words");
    __shared__ uint32_t row_s[8][WORDS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;  // row in the plane
    const int plane = blockIdx.y;         // seq * n_hkv + kv head
    if (r >= n_kv)
        return;
    const int hh = plane % n_hkv, sq = plane / n_hkv;
    const uint32_t *rp = reinterpret_cast<const uint32_t *>(src + (int64_t)r * nb1 +
                                                            (int64_t)hh * nb2 + (int64_t)sq * nb3);
    for (int w = lane; w < WORDS; w += 32)
        row_s[warp][w] = __ldcs(rp + w);
    __syncwarp();
    const uint8_t *rb = reinterpret_cast<const uint8_t *>(row_s[warp]);
    const int j0 = lane * EPL, b = j0 / 32, i0 = j0 % 32; // EPL elements stay in one block
    const float d = __half2float(*reinterpret_cast<const __half *>(rb + BB * b));
    uint32_t out[EPL / 2];
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
        float x[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = i0 + e + k;
            if constexpr (T == kQ8) {
                x[k] = (float)(int)(int8_t)rb[BB * b + 2 + i] * d;
            } else {
                const uint8_t byte = rb[BB * b + 2 + (i & 15)];
                x[k] = (float)((int)(i < 16 ? byte & 15u : byte >> 4) - 8) * d;
            }
        }
        const __half2 hv = __floats2half2_rn(x[0], x[1]);
        out[e / 2] = *reinterpret_cast<const uint32_t *>(&hv);
    }
    __half *o = dst + ((int64_t)plane * n_kv + r) * D + j0;
    if constexpr (EPL == 8)
        *reinterpret_cast<uint4 *>(o) = make_uint4(out[0], out[1], out[2], out[3]);
    else
        *reinterpret_cast<uint2 *>(o) = make_uint2(out[0], out[1]);
}

// The same widening for views whose rows are only 2-byte aligned: one thread
// per 8 elements (a quarter of a 32-element block), 2-byte loads.
template <int T>
__global__ void kv_to_f16_u16_kernel(const uint8_t *__restrict__ src, int64_t nb1, int64_t nb2,
                                     int64_t nb3, int D, int n_kv, int n_hkv, int64_t n_units,
                                     __half *__restrict__ dst) {
    const int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= n_units)
        return;
    const int per_row = D / 8;
    const int64_t row = u / per_row; // [seq][kv head][row] order
    const int c = (int)(u - row * per_row);
    const int64_t r = row % n_kv, hh = (row / n_kv) % n_hkv, sq = row / ((int64_t)n_kv * n_hkv);
    const uint8_t *rp = src + r * nb1 + hh * nb2 + sq * nb3;
    const int b = c >> 2, part = c & 3;
    constexpr int BB = T == kQ8 ? 34 : 18;
    const uint8_t *blk = rp + BB * b;
    const float d = h2f_bits(*reinterpret_cast<const uint16_t *>(blk));
    float x[8];
    if constexpr (T == kQ8) {
        const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2 + 8 * part);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w = p[i];
            x[2 * i] = (float)(int)(int8_t)(w & 0xffu) * d;
            x[2 * i + 1] = (float)(int)(int8_t)(w >> 8) * d;
        }
    } else {
        // elements 0..15 are the low nibbles of bytes 0..15, 16..31 the high ones
        const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2 + 8 * (part & 1));
        const int sh = 4 * (part >> 1);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t w = p[i];
            x[2 * i] = (float)((int)(((w & 0xffu) >> sh) & 15u) - 8) * d;
            x[2 * i + 1] = (float)((int)(((w >> 8) >> sh) & 15u) - 8) * d;
        }
    }
    uint4 o;
    uint32_t *ow = reinterpret_cast<uint32_t *>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 hv = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        ow[i] = *reinterpret_cast<const uint32_t *>(&hv);
    }
    *reinterpret_cast<uint4 *>(dst + row * D + 8 * c) = o;
}

// ---------------------------------------------------------------------------
// host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

void *tensor_map_encoder() { return reinterpret_cast<void *>(get_encode()); }

static size_t map_bytes(const PrefillShape &ps) {
    const size_t n_qt = (ps.n_q + pf::BM - 1) / pf::BM, n_kt = (ps.n_kv + pf::BN - 1) / pf::BN;
    return ((size_t)ps.m_planes * n_qt * n_kt + 255) / 256 * 256 + 256;
}

// f16 copy of one of K / V: [n_seq_kv][n_head_kv][n_kv][D], 256-byte multiple
static size_t f16_copy_bytes(const PrefillShape &ps) {
    return ((size_t)ps.n_seq_kv * ps.n_head_kv * ps.n_kv * ps.D * 2 + 255) / 256 * 256;
}

size_t prefill_ws_bytes(const PrefillShape &ps) {
    return map_bytes(ps) + (ps.kv_type == kF16 ? 0 : 2 * f16_copy_bytes(ps));
}

static cudaError_t launch_kv_to_f16(int type, const void *src, const int64_t *nb,
                                    const PrefillShape &ps, __half *dst, cudaStream_t st) {
    const uint8_t *s8 = static_cast<const uint8_t *>(src);
    const bool words = ((reinterpret_cast<uintptr_t>(src) | (uintptr_t)nb[1] | (uintptr_t)nb[2] |
                         (uintptr_t)nb[3]) & 3) == 0;
    if (words) {
        const dim3 grid((unsigned)((ps.n_kv + 7) / 8), (unsigned)(ps.n_seq_kv * ps.n_head_kv));
        const int key = (type == kQ8 ? 0 : 2) + (ps.D == 256 ? 1 : 0);
        switch (key) {
        case 0: kv_to_f16_kernel<kQ8, 128><<<grid, 256, 0, st>>>(s8, nb[1], nb[2], nb[3], ps.n_kv, ps.n_head_kv, dst); break;
        case 1: kv_to_f16_kernel<kQ8, 256><<<grid, 256, 0, st>>>(s8, nb[1], nb[2], nb[3], ps.n_kv, ps.n_head_kv, dst); break;
        case 2: kv_to_f16_kernel<kQ4, 128><<<grid, 256, 0, st>>>(s8, nb[1], nb[2], nb[3], ps.n_kv, ps.n_head_kv, dst); break;
        default: kv_to_f16_kernel<kQ4, 256><<<grid, 256, 0, st>>>(s8, nb[1], nb[2], nb[3], ps.n_kv, ps.n_head_kv, dst); break;
        }
        return cudaGetLastError();
    }
    const int64_t n_units = (int64_t)ps.n_seq_kv * ps.n_head_kv * ps.n_kv * (ps.D / 8);
    const unsigned blocks = (unsigned)((n_units + 255) / 256);
    if (type == kQ8)
        kv_to_f16_u16_kernel<kQ8><<<blocks, 256, 0, st>>>(s8, nb[1], nb[2], nb[3], ps.D, ps.n_kv,
                                                           ps.n_head_kv, n_units, dst);
    else
        kv_to_f16_u16_kernel<kQ4><<<blocks, 256, 0, st>>>(s8, nb[1], nb[2], nb[3], ps.D, ps.n_kv,
                                                           ps.n_head_kv, n_units, dst);
    return cudaGetLastError();
}

cudaError_t launch_prefill(const PrefillShape &ps_in, void *ws, cudaStream_t st, const char **why) {
    auto encode = get_encode();
    if (!encode) {
        *why = "cuTensorMapEncodeTiled unavailable";
        return cudaErrorNotSupported;
    }
    PrefillShape ps = ps_in;
    const int D = ps.D;
    const int n_qt = (ps.n_q + pf::BM - 1) / pf::BM, n_kt = (ps.n_kv + pf::BN - 1) / pf::BN;
    uint8_t *map = static_cast<uint8_t *>(ws);
    int *err = reinterpret_cast<int *>(map + map_bytes(ps) - 256);
    cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), st);
    if (e != cudaSuccess)
        return e;
    const bool quant = ps.kv_type != kF16;
    if (quant) {
        // K and V widened once into the workspace; the kernel then reads them
        // through the same tensor maps as an F16 cache
        __half *k16 = reinterpret_cast<__half *>(map + map_bytes(ps));
        __half *v16 = reinterpret_cast<__half *>(map + map_bytes(ps) + f16_copy_bytes(ps));
        if ((e = launch_kv_to_f16(ps.kv_type, ps.k, ps.k_nb, ps, k16, st)) != cudaSuccess ||
            (e = launch_kv_to_f16(ps.kv_type, ps.v, ps.v_nb, ps, v16, st)) != cudaSuccess)
            return e;
        const int64_t nb[4] = {2, 2 * (int64_t)D, 2 * (int64_t)D * ps.n_kv,
                               2 * (int64_t)D * ps.n_kv * ps.n_head_kv};
        ps.k = k16;
        ps.v = v16;
        for (int i = 0; i < 4; ++i)
            ps.k_nb[i] = ps.v_nb[i] = nb[i];
    }
    const int planes = ps.m_planes;
    if (ps.mask) {
        dim3 g(n_kt, n_qt, planes);
        const int vec = ((reinterpret_cast<uintptr_t>(ps.mask) | (uintptr_t)ps.m_nb1 |
                          (uintptr_t)ps.m_nb2 | (uintptr_t)ps.m_nb3) & 15) == 0;
        mask_block_map_kernel<<<g, 256, 0, st>>>(ps.mask, ps.m_nb1, ps.m_nb2, ps.m_nb3, ps.m_ne2,
                                                 ps.n_q, ps.n_kv, n_qt, n_kt, vec, map);
    } else {
        const size_t n = (size_t)planes * n_qt * n_kt;
        fill_map_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(map, n, n_kt, ps.n_kv);
    }
    if ((e = cudaGetLastError()) != cudaSuccess)
        return e;

    CUtensorMap maps[2];
    const void *bases[2] = {ps.k, ps.v};
    const int64_t *nbs[2] = {ps.k_nb, ps.v_nb};
    for (int i = 0; i < 2; ++i) {
        cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)ps.n_kv, (cuuint64_t)ps.n_head_kv,
                              (cuuint64_t)ps.n_seq_kv};
        cuuint64_t strides[3] = {(cuuint64_t)nbs[i][1], (cuuint64_t)nbs[i][2],
                                 (cuuint64_t)nbs[i][3]};
        cuuint32_t box[4] = {64, pf::BN, 1, 1};
        cuuint32_t estr[4] = {1, 1, 1, 1};
        CUresult r = encode(&maps[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                            const_cast<void *>(bases[i]), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            *why = "cuTensorMapEncodeTiled rejected the K/V layout";
            return cudaErrorInvalidValue;
        }
    }
    PrefillArgs a;
    a.q = ps.q;
    a.q_nb1 = ps.q_nb[1];
    a.q_nb2 = ps.q_nb[2];
    a.q_nb3 = ps.q_nb[3];
    a.mask = ps.mask;
    a.m_nb1 = ps.m_nb1;
    a.m_nb2 = ps.m_nb2;
    a.m_nb3 = ps.m_nb3;
    a.m_ne2 = ps.mask ? ps.m_ne2 : 1;
    a.m_ne3 = ps.mask ? ps.m_ne3 : 1;
    a.block_map = map;
    a.dst = ps.dst;
    a.err = err;
    a.n_q = ps.n_q;
    a.n_head = ps.n_head;
    a.n_head_kv = ps.n_head_kv;
    a.n_seq = ps.n_seq;
    a.n_kv = ps.n_kv;
    a.rk3 = ps.n_seq / ps.n_seq_kv;
    a.n_qt = n_qt;
    a.n_kt = n_kt;
    a.scale_log2 = ps.scale * 1.4426950408889634f;
    const size_t smem = 1024 + (size_t)pf::nslot(D) * pf::BN * D * 2 + 256;
    dim3 grid((unsigned)(n_qt * ps.n_head * ps.n_seq));
    static std::atomic<unsigned long long> attr_done[4];
    auto go = [&](auto kern, int slot) {
        cudaError_t r = set_smem_limit((const void *)kern, smem, attr_done[slot]);
        if (r != cudaSuccess)
            return r;
        kern<<<grid, pf::NT, smem, st>>>(maps[0], maps[1], a);
        return cudaSuccess;
    };
    if (D == 256)
        e = quant ? go(fa_prefill_kernel<256, true>, 3) : go(fa_prefill_kernel<256, false>, 1);
    else
        e = quant ? go(fa_prefill_kernel<128, true>, 2) : go(fa_prefill_kernel<128, false>, 0);
    if (e != cudaSuccess)
        return e;
    return cudaGetLastError();
}

} // namespace xq
