// Split-KV flash decode on warp-level tensor-core MMAs (ggml FLASH_ATTN_EXT
// semantics; see xq_decode.cu for the reference citations).
//
// Per CTA: one split of KV rows x one kv head x up to 8 q-rows (the GQA
// heads / queries sharing that kv head) x one sequence.  Each of the 4 warps
// owns every 4th group of 16 keys of the split and streams it through its own
// 3-stage cp.async ring, so warps never wait on each other until the final
// fixed-order merge of their (m, l, O) states.
//
// Scores, per 16-key group: S^T (16 keys x 8 q-rows)
//   Q8_0 / Q4_0 K:  one mma.m16n8k32 per 32-element block on the int8 codes
//                   (q is quantized to Q8_0 first, as ggml does), giving the
//                   exact integer block sums; s += float(sum) * (d_k * d_q) in
//                   block order -- ggml's vec_dot_q8_0_q8_0 / q4_0_q8_0.
//                   Q4_0 nibbles enter unsigned (u8 x s8) and the -8 offset
//                   is removed exactly as 8 * sum(q) per block.
//   F16 K:          mma.m16n8k16 on f16 (q rounded to f16, as ggml does),
//                   A fragments by ldmatrix.
// Softmax: running max in the log2 domain, rescaled whenever it grows.
// Values, per group: O^T (D x 8 q-rows) += V^T P^T with mma.m16n8k16 f16:
//   F16 V:          A fragments by ldmatrix.trans.
//   Q8_0 / Q4_0 V:  the codes (exact in f16) are gathered from shared memory
//                   with dims permuted so one 16/32-bit load per key feeds
//                   two M-tiles; the per-(key, block) scale is folded into P.
// Accumulation is fp32 throughout.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <float.h>
#include <math.h>
#include <string.h>

#include <utility>

#include "xq_common.cuh"
#include "xq_internal.h"

namespace xq {
namespace dm {

constexpr int NWARP = 4, NT = 32 * NWARP, KG = 16;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// The running max is only moved when a group's max exceeds it by more than
// this (log2 units), so p = 2^(x - max) stays <= 256 and the accumulator
// rescale is rare; O = acc / l and lse = max + log(l) hold for any max.
constexpr float kRescale = 8.0f;

// Load path of a (type, copy width) pair: quantized rows whose length is a
// multiple of 16 bytes arrive as one TMA box per 16-key group; 16-byte F16
// rows as one bulk copy per row; anything else by per-lane cp.async.
__host__ __device__ constexpr bool tma_mode(int T, int VW) { return VW == 16 && T != kF16; }

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                          uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// cp.async with zero fill when src_bytes == 0.
template <int VW>
__device__ __forceinline__ void cp_async_zfill(uint32_t dst, const void *src, int src_bytes) {
    if constexpr (VW == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                     "r"(src_bytes));
    else if constexpr (VW == 8)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(dst), "l"(src),
                     "r"(src_bytes));
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src),
                     "r"(src_bytes));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar),
                 "r"(bytes));
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 20000;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity));
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait (2 s, far beyond any legitimate wait); false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    while (!mbar_try(bar, parity))
        if (globaltimer() - t0 > 2000000000ull)
            return false;
    return true;
}
// One bulk (TMA engine) copy global -> shared, completion counted on bar.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];\n" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// One TMA tile (a 16-row box of a 4D tensor map) global -> shared.
__device__ __forceinline__ void tma_rows(uint32_t dst, const CUtensorMap *map, int row, int head,
                                         int seq, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(head), "r"(seq), "r"(bar)
        : "memory");
}
// L2 prefetch of one TMA box (no shared-memory destination, no completion).
__device__ __forceinline__ void tma_prefetch_rows(const CUtensorMap *map, int row, int head,
                                                  int seq) {
    asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];\n" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(0), "r"(row), "r"(head), "r"(seq)
                 : "memory");
}
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// 32-bit word at a 2-byte aligned shared address (compile-time alignment known).
template <bool ALIGNED4>
__device__ __forceinline__ uint32_t ld_word(const uint8_t *p) {
    if constexpr (ALIGNED4) {
        return *reinterpret_cast<const uint32_t *>(p);
    } else {
        const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
        return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
    }
}
__device__ __forceinline__ float h2f(const uint8_t *p) {
    return __half2float(*reinterpret_cast<const __half *>(p));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// Two signed int8 codes (byte 0 and byte 2 of x, already xor 0x80) -> half2.
__device__ __forceinline__ uint32_t s8pair_to_h2(uint32_t x) {
    uint32_t h = (x & 0x00FF00FFu) | 0x64006400u; // 1024 + (code + 128)
    __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&h), __half2(__float2half(1152.0f),
                                                                  __float2half(1152.0f)));
    return *reinterpret_cast<uint32_t *>(&r);
}
// Two unsigned nibble codes (low nibbles of byte 0 and byte 2) -> half2 of code - 8.
__device__ __forceinline__ uint32_t u4pair_to_h2(uint32_t x) {
    uint32_t h = (x & 0x000F000Fu) | 0x64006400u; // 1024 + nibble
    __half2 r = __hsub2(*reinterpret_cast<__half2 *>(&h), __half2(__float2half(1032.0f),
                                                                  __float2half(1032.0f)));
    return *reinterpret_cast<uint32_t *>(&r);
}

// Compile-time loop: f(std::integral_constant<int, I>) for I in [0, N).
template <class F, int... I>
__device__ __forceinline__ void static_for_impl(F &&f, std::integer_sequence<int, I...>) {
    (f(std::integral_constant<int, I>{}), ...);
}
template <int N, class F>
__device__ __forceinline__ void static_for(F &&f) {
    static_for_impl(f, std::make_integer_sequence<int, N>{});
}
// Shared-memory loads at a register base plus a compile-time byte offset.
template <int OFF>
__device__ __forceinline__ uint32_t lds16(uint32_t base) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1+%2];\n" : "=h"(v) : "r"(base), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint32_t lds32(uint32_t base) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1+%2];\n" : "=r"(v) : "r"(base), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ float2 ldsf2(uint32_t base) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2+%3];\n"
                 : "=f"(v.x), "=f"(v.y)
                 : "r"(base), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ int2 ldsi2(uint32_t base) {
    int2 v;
    asm volatile("ld.shared.v2.s32 {%0, %1}, [%2+%3];\n" : "=r"(v.x), "=r"(v.y) : "r"(base), "n"(OFF));
    return v;
}
// 32-bit word at a 2-byte aligned offset (even quant blocks start at +2 mod 4).
template <int OFF, bool ALIGNED4>
__device__ __forceinline__ uint32_t ldsw(uint32_t base) {
    if constexpr (ALIGNED4)
        return lds32<OFF>(base);
    else
        return __byte_perm(lds16<OFF>(base), lds16<OFF + 2>(base), 0x5410);
}
__device__ __forceinline__ float u16f(uint32_t h) { return __half2float(__ushort_as_half((uint16_t)h)); }
template <int OFF>
__device__ __forceinline__ void ldsm4(uint32_t base, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                      uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4+%5];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(base), "n"(OFF));
}
template <int OFF>
__device__ __forceinline__ void ldsm4t(uint32_t base, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                       uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4+%5];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(base), "n"(OFF));
}

// Output dim of O^T tile m, fragment row (g or g + 8) -> dim (the V gathers
// permute dims so that one load per key feeds two M-tiles).
template <int T>
__device__ __forceinline__ int out_dim(int m, int row) {
    if constexpr (T == kF16) {
        return 16 * m + row;
    } else if constexpr (T == kQ8) {
        const int b = m >> 1, hf = m & 1, g = row & 7, hi = row >> 3;
        return 32 * b + 4 * g + 2 * hf + hi;
    } else {
        const int b = m >> 1, hf = m & 1, g = row & 7, hi = row >> 3;
        return 32 * b + 2 * g + hi + 16 * hf;
    }
}

} // namespace dm

// Resident CTAs per SM the kernel is compiled for.  (Three for Q8_0 rows --
// 162 registers, 73 KB of shared memory, three 16-key rounds per warp on
// config 2 instead of four -- measured slower: 15.9 against 14.5 us a step.)
__host__ __device__ constexpr int mma_ctas_per_sm(int) { return 2; }

template <int T, int D, int STAGES, int VW, int QB>
__global__ void __launch_bounds__(dm::NT, mma_ctas_per_sm(T))
    fa_decode_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
    using namespace dm;
    constexpr bool TMA = tma_mode(T, VW);
    constexpr bool BULK = VW == 16; // mbarrier-tracked copies (TMA boxes or bulk rows)
    constexpr int REC = rec_bytes(T, D);
    constexpr int SS = smem_stride(REC);
    constexpr int NB = D / 32;             // quant blocks per row
    constexpr int MT = D / 16;             // O^T M-tiles
    constexpr int GBYTES = KG * SS;        // one 16-key group of K (or V)
    constexpr int RING = STAGES * 2 * GBYTES;
    constexpr int VPR = REC / VW;
    constexpr int BB = T == kQ8 ? 34 : 18; // bytes per quant block
    static_assert(REC % VW == 0, "copy width");
    // q-rows of the CTA: QB blocks of 8 (query, head) rows, each the N = 8 side
    // of the warp MMAs; every K/V group a warp loads serves all of them (the
    // block dots share the K fragments, the PV products the V conversion)
    constexpr int RQ = 8 * QB;
    constexpr int OWS = D + 4;               // merge buffer row stride (bank spread)
    constexpr int OWB = NWARP * RQ * OWS * 4; // merge buffer, aliases the rings
    constexpr int BIG = NWARP * RING > OWB ? NWARP * RING : OWB;

    extern __shared__ __align__(128) uint8_t smem[];
    if constexpr (TMA) {
        // TMA destinations must be 128-byte aligned (all ring offsets are)
        if (smem_u32(smem) & 127u) {
            if (a.err && threadIdx.x == 0)
                atomicExch(a.err, 3);
            return;
        }
    }
    uint8_t *rings = smem;                                   // [NWARP][STAGES][K|V][GBYTES]
    uint8_t *qsm = rings + BIG;                              // q codes: int8 or f16 [RQ][D]
    constexpr int QBYTES = T == kF16 ? RQ * D * 2 : RQ * D;  // f16 or int8 q codes
    float *dq_s = reinterpret_cast<float *>(qsm + QBYTES); // [NB][RQ]
    int *qsum_s = reinterpret_cast<int *>(dq_s + NB * RQ);   // [NB][RQ] (8 * sum q)
    float *pt_s = reinterpret_cast<float *>(qsum_s + NB * RQ); // [NWARP][QB][16][8]
    float *mw_s = pt_s + NWARP * QB * 16 * 8;                // [NWARP][RQ]
    float *lw_s = mw_s + NWARP * RQ;                         // [NWARP][RQ]
    float *slope_s = lw_s + NWARP * RQ;                      // [RQ]
    int64_t *moff_s = reinterpret_cast<int64_t *>(slope_s + RQ); // [RQ]
    int *lim_s = reinterpret_cast<int *>(moff_s + RQ);       // [RQ]
    uint64_t *bar_s = reinterpret_cast<uint64_t *>(lim_s + RQ); // [NWARP][STAGES]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int kvh = blockIdx.y % a.n_head_kv, qb = blockIdx.y / a.n_head_kv, s = blockIdx.z;
    const int64_t split = a.split_begin + blockIdx.x;
    const int64_t r0 = split * a.rows_per_split;
    const int64_t r1 = min((int64_t)a.n_kv, r0 + a.rows_per_split);
    const int nrows_split = (int)max((int64_t)0, r1 - r0);
    const int jbase = qb * RQ;
    const int nj = min(RQ, a.n_qrows - jbase);
    const uint8_t *kbase = a.k + (int64_t)kvh * a.k_nb2 + (int64_t)(s / a.rk3) * a.k_nb3 +
                           r0 * a.k_nb1;
    const uint8_t *vbase = a.v + (int64_t)kvh * a.v_nb2 + (int64_t)(s / a.rv3) * a.v_nb3 +
                           r0 * a.v_nb1;

    // ---- per-warp load pipeline over this warp's 16-key groups ----
    const int n_groups = (nrows_split + KG - 1) / KG;
    uint8_t *ring = rings + warp * RING;
    const uint32_t ring_s = smem_u32(ring);
    uint64_t *mybar = bar_s + warp * STAGES;
    // my groups: warp + NWARP * i
    const int my_n = n_groups > warp ? (n_groups - warp + NWARP - 1) / NWARP : 0;
    if constexpr (TMA) {
        if (tid == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kmap))
                         : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&vmap))
                         : "memory");
        }
    }
    if constexpr (BULK) {
        // before any load is in flight: this fence waits for outstanding memory operations
        if (lane < STAGES)
            mbar_init(smem_u32(mybar + lane), 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        __syncwarp();
    }
    if constexpr (TMA) {
        // Launched as a programmatic dependent: until griddepcontrol.wait the
        // kernel before this one may still be writing q or the KV cache, so
        // only L2 prefetches (coherent, no data consumed) are issued here.
        // (Prefetching every group of the split instead -- 160 KB per CTA --
        // measured slower on config 2: 16.1 against 14.9 us per step.)
        if (lane == 0)
            for (int st = 0; st < STAGES - 1 && st < my_n; ++st) {
                const int row = (int)(r0 + (warp + NWARP * st) * KG);
                tma_prefetch_rows(&kmap, row, kvh, s / a.rk3);
                tma_prefetch_rows(&vmap, row, kvh, s / a.rv3);
            }
    }
    grid_dep_wait();
    // q loads first: their latency overlaps the K/V copies issued next
    // quantizer units (two per q block of a q-row): unit tid + NT u, u < QB
    constexpr int QU = T == kF16 ? 0 : RQ * NB * 2;
    static_assert(QU <= NT * QB && QU % 32 == 0, "at most QB quantizer units per thread");
    float xq[QB][16];
    if constexpr (QU > 0) {
#pragma unroll
        for (int u = 0; u < QB; ++u) {
            const int unit = tid + NT * u;
            const int blk = unit >> 1, half = unit & 1;
            const int j = blk / NB, b = blk - j * NB;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                xq[u][i] = 0.0f;
            if (unit < QU && j < nj) {
                const int jj = jbase + j, iq1 = jj / a.G, h = kvh * a.G + jj % a.G;
                const float *src = reinterpret_cast<const float *>(
                                       a.q + (int64_t)iq1 * a.q_nb1 + (int64_t)h * a.q_nb2 +
                                       (int64_t)s * a.q_nb3) +
                                   b * 32 + half * 16;
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    xq[u][i] = src[i];
            }
        }
    }
    auto issue = [&](int grp, int stage) {
        const int k0 = grp * KG; // relative to r0
        uint8_t *kd = ring + stage * 2 * GBYTES;
        uint8_t *vd = kd + GBYTES;
        if constexpr (TMA) {
            // rows past the split end arrive too (p = 0 there); rows past n_kv
            // are zero-filled by the copy engine
            static_assert(SS == REC, "TMA boxes are dense");
            if (lane == 0) {
                const uint32_t bar = smem_u32(mybar + stage);
                mbar_expect_tx(bar, (uint32_t)(2 * KG * REC));
                const int row = (int)(r0 + k0);
                tma_rows(smem_u32(kd), &kmap, row, kvh, s / a.rk3, bar);
                tma_rows(smem_u32(vd), &vmap, row, kvh, s / a.rv3, bar);
            }
        } else if constexpr (BULK) {
            const int nrows = min(KG, nrows_split - k0);
            const uint32_t bar = smem_u32(mybar + stage);
            if (lane == 0)
                mbar_expect_tx(bar, (uint32_t)(2 * nrows * REC));
            const int r = lane & (KG - 1);
            uint8_t *dst = (lane < KG ? kd : vd) + r * SS;
            if (r < nrows) {
                const uint8_t *src = lane < KG ? kbase + (int64_t)(k0 + r) * a.k_nb1
                                               : vbase + (int64_t)(k0 + r) * a.v_nb1;
                bulk_g2s(smem_u32(dst), src, REC, bar);
            } else if (lane >= KG) {
                // V rows past the split end must be finite zeros (p = 0 there)
                for (int c = 0; c < REC; c += 16)
                    *reinterpret_cast<uint4 *>(dst + c) = make_uint4(0, 0, 0, 0);
            }
        } else {
            for (int idx = lane; idx < KG * VPR; idx += 32) {
                const int r = idx / VPR, c = idx - r * VPR;
                const bool ok = k0 + r < nrows_split;
                const int64_t row = ok ? k0 + r : 0;
                cp_async_zfill<VW>(smem_u32(kd + r * SS + c * VW), kbase + row * a.k_nb1 + c * VW,
                                   ok ? VW : 0);
                cp_async_zfill<VW>(smem_u32(vd + r * SS + c * VW), vbase + row * a.v_nb1 + c * VW,
                                   ok ? VW : 0);
            }
        }
    };
#pragma unroll
    for (int st = 0; st < STAGES - 1; ++st) {
        if (st < my_n)
            issue(warp + NWARP * st, st);
        if constexpr (!BULK)
            cp_async_commit();
    }

    // ---- prologue: q in K's dot type, per-q-row constants ----
    if (tid < RQ) {
        const int j = tid;
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
        } else {
            lim = -1; // padding q-row: every key masked
        }
        slope_s[j] = slope;
        moff_s[j] = moff;
        lim_s[j] = lim;
    }
    if constexpr (T == kF16) {
        __half *q16 = reinterpret_cast<__half *>(qsm);
        for (int idx = tid; idx < RQ * D; idx += NT) {
            const int j = idx / D, d = idx - j * D;
            float x = 0.0f;
            if (j < nj) {
                const int jj = jbase + j, iq1 = jj / a.G, h = kvh * a.G + jj % a.G;
                x = *reinterpret_cast<const float *>(a.q + (int64_t)iq1 * a.q_nb1 +
                                                     (int64_t)h * a.q_nb2 +
                                                     (int64_t)s * a.q_nb3 + 4 * d);
            }
            q16[idx] = __float2half_rn(x);
        }
    } else {
        // ggml quantize_row_q8_0 reference arithmetic; two threads per 32-block
        int8_t *q8 = reinterpret_cast<int8_t *>(qsm);
#pragma unroll
        for (int u = 0; u < QB; ++u) {
            const int unit = tid + NT * u;
            if (unit >= QU) // warp-uniform (QU is a multiple of 32)
                continue;
            const int blk = unit >> 1, half = unit & 1;
            const int j = blk / NB, b = blk - j * NB;
            const float *x = xq[u]; // loaded above (zeros for padding q-rows)
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                amax = fmaxf(amax, fabsf(x[i]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            uint32_t w[4] = {0, 0, 0, 0};
            int qs = 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int qi = (int)roundf(x[i] * id);
                qs += qi;
                w[i >> 2] |= (uint32_t)(uint8_t)(int8_t)qi << (8 * (i & 3));
            }
            qs += __shfl_xor_sync(0xffffffffu, qs, 1);
            *reinterpret_cast<uint4 *>(q8 + j * D + b * 32 + half * 16) =
                make_uint4(w[0], w[1], w[2], w[3]);
            if (half == 0) {
                dq_s[b * RQ + j] = __half2float(__float2half_rn(d));
                qsum_s[b * RQ + j] = 8 * qs;
            }
        }
    }
    __syncthreads();

    // q as the B operand (8 q-rows = N per block), kept in registers
    constexpr int QREGS = T == kF16 ? D / 8 : D / 16;
    uint32_t qf[QB][QREGS];
#pragma unroll
    for (int sb = 0; sb < QB; ++sb) {
        const int row = 8 * sb + g;
        if constexpr (T == kF16) {
            const __half *q16 = reinterpret_cast<const __half *>(qsm);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                qf[sb][2 * kk] =
                    *reinterpret_cast<const uint32_t *>(q16 + row * D + 16 * kk + 2 * t);
                qf[sb][2 * kk + 1] =
                    *reinterpret_cast<const uint32_t *>(q16 + row * D + 16 * kk + 8 + 2 * t);
            }
        } else {
            const int8_t *q8 = reinterpret_cast<const int8_t *>(qsm);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                qf[sb][2 * b] = *reinterpret_cast<const uint32_t *>(q8 + row * D + 32 * b + 4 * t);
                qf[sb][2 * b + 1] =
                    *reinterpret_cast<const uint32_t *>(q8 + row * D + 32 * b + 16 + 4 * t);
            }
        }
    }
    // this lane's two q-rows of each block (columns 2t, 2t+1 of block sb)
    const int c0 = 2 * t, c1 = 2 * t + 1;
    const bool plain = !a.mask && !a.positions && a.softcap == 0.0f; // uniform
    bool live0[QB], live1[QB];
    float slope0[QB], slope1[QB];
    int lim0[QB], lim1[QB];
    int64_t mo0[QB], mo1[QB];
    uint32_t dq_base[QB], qs_base[QB]; // + 4 RQ b bytes for block b of the row
#pragma unroll
    for (int sb = 0; sb < QB; ++sb) {
        const int r0c = 8 * sb + c0, r1c = 8 * sb + c1;
        live0[sb] = r0c < nj;
        live1[sb] = r1c < nj;
        slope0[sb] = slope_s[r0c];
        slope1[sb] = slope_s[r1c];
        lim0[sb] = lim_s[r0c];
        lim1[sb] = lim_s[r1c];
        mo0[sb] = moff_s[r0c];
        mo1[sb] = moff_s[r1c];
        dq_base[sb] = smem_u32(dq_s + r0c);
        qs_base[sb] = smem_u32(qsum_s + r0c);
    }

    float acc[QB][MT][4];
#pragma unroll
    for (int sb = 0; sb < QB; ++sb)
#pragma unroll
        for (int m = 0; m < MT; ++m)
            acc[sb][m][0] = acc[sb][m][1] = acc[sb][m][2] = acc[sb][m][3] = 0.0f;
    float mu0[QB], mu1[QB], l0[QB], l1[QB];
#pragma unroll
    for (int sb = 0; sb < QB; ++sb) {
        mu0[sb] = mu1[sb] = -INFINITY;
        l0[sb] = l1[sb] = 0.0f;
    }

    for (int i = 0; i < my_n; ++i) {
        {
            const int nxt = i + STAGES - 1;
            if (nxt < my_n)
                issue(warp + NWARP * nxt, nxt % STAGES);
            if constexpr (!BULK)
                cp_async_commit();
        }
        const int stage = i % STAGES;
        if constexpr (BULK) {
            // warp-uniform outcome: the MMAs and shuffles below are warp-collective
            if (!__all_sync(0xffffffffu,
                            mbar_wait(smem_u32(mybar + stage), (uint32_t)((i / STAGES) & 1)))) {
                if (a.err && lane == 0)
                    atomicExch(a.err, 2);
                break;
            }
        } else {
            cp_async_wait<STAGES - 1>();
        }
        __syncwarp();
        const uint32_t kg_s = ring_s + stage * 2 * GBYTES;
        const uint32_t vg_s = kg_s + GBYTES;
        const int k0 = (warp + NWARP * i) * KG; // relative to r0

        // ---------------- scores S^T[key][q-row], every q block ----------------
        float2 sA[QB], sB[QB]; // keys g, g+8 x this lane's two rows of block sb
#pragma unroll
        for (int sb = 0; sb < QB; ++sb)
            sA[sb] = sB[sb] = make_float2(0.0f, 0.0f);
        if constexpr (T == kF16) {
            float sc[QB][4];
#pragma unroll
            for (int sb = 0; sb < QB; ++sb)
                sc[sb][0] = sc[sb][1] = sc[sb][2] = sc[sb][3] = 0.0f;
            const uint32_t kl = kg_s + ((lane & 7) + ((lane >> 3) & 1) * 8) * SS +
                                ((lane >> 4) & 1) * 16;
            static_for<D / 16>([&](auto kk_) {
                constexpr int kk = decltype(kk_)::value;
                uint32_t a0, a1, a2, a3;
                ldsm4<32 * kk>(kl, a0, a1, a2, a3);
#pragma unroll
                for (int sb = 0; sb < QB; ++sb)
                    mma_f16(sc[sb], a0, a1, a2, a3, qf[sb][2 * kk], qf[sb][2 * kk + 1]);
            });
#pragma unroll
            for (int sb = 0; sb < QB; ++sb) {
                sA[sb] = make_float2(sc[sb][0], sc[sb][1]);
                sB[sb] = make_float2(sc[sb][2], sc[sb][3]);
            }
        } else {
            const uint32_t kA = kg_s + g * SS, kB = kA + 8 * SS;
            const uint32_t kAt = kA + 4 * t, kBt = kB + 4 * t;
            static_for<NB>([&](auto b_) {
                constexpr int b = decltype(b_)::value;
                constexpr int QO = BB * b + 2;
                constexpr bool AL = (QO % 4) == 0;
                int c[QB][4];
#pragma unroll
                for (int sb = 0; sb < QB; ++sb)
                    c[sb][0] = c[sb][1] = c[sb][2] = c[sb][3] = 0;
                if constexpr (T == kQ8) {
                    const uint32_t ka0 = ldsw<QO, AL>(kAt), kb0 = ldsw<QO, AL>(kBt);
                    const uint32_t ka1 = ldsw<QO + 16, AL>(kAt), kb1 = ldsw<QO + 16, AL>(kBt);
#pragma unroll
                    for (int sb = 0; sb < QB; ++sb)
                        mma_s8(c[sb], ka0, kb0, ka1, kb1, qf[sb][2 * b], qf[sb][2 * b + 1]);
                } else {
                    const uint32_t w0 = ldsw<QO, AL>(kAt), w1 = ldsw<QO, AL>(kBt);
                    const uint32_t l0w = w0 & 0x0F0F0F0Fu, l1w = w1 & 0x0F0F0F0Fu;
                    const uint32_t h0w = (w0 >> 4) & 0x0F0F0F0Fu, h1w = (w1 >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int sb = 0; sb < QB; ++sb) {
                        mma_u8s8(c[sb], l0w, l1w, h0w, h1w, qf[sb][2 * b], qf[sb][2 * b + 1]);
                        const int2 q8s = ldsi2<4 * RQ * b>(qs_base[sb]);
                        c[sb][0] -= q8s.x;
                        c[sb][1] -= q8s.y;
                        c[sb][2] -= q8s.x;
                        c[sb][3] -= q8s.y;
                    }
                }
                const float dk0 = u16f(lds16<BB * b>(kA)), dk1 = u16f(lds16<BB * b>(kB));
#pragma unroll
                for (int sb = 0; sb < QB; ++sb) {
                    const float2 dq = ldsf2<4 * RQ * b>(dq_base[sb]);
                    sA[sb] = __ffma2_rn(make_float2((float)c[sb][0], (float)c[sb][1]),
                                        __fmul2_rn(make_float2(dk0, dk0), dq), sA[sb]);
                    sB[sb] = __ffma2_rn(make_float2((float)c[sb][2], (float)c[sb][3]),
                                        __fmul2_rn(make_float2(dk1, dk1), dq), sB[sb]);
                }
            });
        }

        // ---------------- mask, softmax (log2 domain), per q block ----------------
        const int remk = nrows_split - k0; // keys g < remk are inside the split
        float2 pab[QB], pcd[QB];           // P^T fragments of each block
#pragma unroll
        for (int sb = 0; sb < QB; ++sb) {
            float x[4] = {sA[sb].x, sA[sb].y, sB[sb].x, sB[sb].y}; // (g,c0) (g,c1) (g+8,c0) (g+8,c1)
            if (plain) {
                const float sl = a.scale * kLog2e;
                x[0] = (g < remk && live0[sb]) ? x[0] * sl : -INFINITY;
                x[1] = (g < remk && live1[sb]) ? x[1] * sl : -INFINITY;
                x[2] = (g + 8 < remk && live0[sb]) ? x[2] * sl : -INFINITY;
                x[3] = (g + 8 < remk && live1[sb]) ? x[3] * sl : -INFINITY;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int kr = k0 + g + (e >> 1) * 8; // relative key
                    const int64_t key = r0 + kr;
                    const int col = e & 1;
                    float v = x[e] * a.scale;
                    if (a.softcap != 0.0f)
                        v = a.softcap * tanhf(v);
                    bool dead = kr >= nrows_split || key >= (col ? lim1[sb] : lim0[sb]);
                    if (a.mask && !dead) {
                        const float mv = (col ? slope1[sb] : slope0[sb]) *
                                         h2f(a.mask + (col ? mo1[sb] : mo0[sb]) + 2 * key);
                        dead = mv == -INFINITY;
                        v += mv;
                    }
                    x[e] = dead ? -INFINITY : v * kLog2e;
                }
            }
            float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            const bool up0 = mx0 > mu0[sb] + kRescale, up1 = mx1 > mu1[sb] + kRescale;
            if (__any_sync(0xffffffffu, up0 || up1)) {
                const float f0 = up0 ? (mu0[sb] == -INFINITY ? 0.0f : ex2(mu0[sb] - mx0)) : 1.0f;
                const float f1 = up1 ? (mu1[sb] == -INFINITY ? 0.0f : ex2(mu1[sb] - mx1)) : 1.0f;
                const float2 ff = make_float2(f0, f1);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    float2 lo = __fmul2_rn(make_float2(acc[sb][m][0], acc[sb][m][1]), ff);
                    float2 hi = __fmul2_rn(make_float2(acc[sb][m][2], acc[sb][m][3]), ff);
                    acc[sb][m][0] = lo.x;
                    acc[sb][m][1] = lo.y;
                    acc[sb][m][2] = hi.x;
                    acc[sb][m][3] = hi.y;
                }
                l0[sb] *= f0;
                l1[sb] *= f1;
                mu0[sb] = up0 ? mx0 : mu0[sb];
                mu1[sb] = up1 ? mx1 : mu1[sb];
            }
            const float p0 = x[0] == -INFINITY ? 0.0f : ex2(x[0] - mu0[sb]);
            const float p1 = x[1] == -INFINITY ? 0.0f : ex2(x[1] - mu1[sb]);
            const float p2 = x[2] == -INFINITY ? 0.0f : ex2(x[2] - mu0[sb]);
            const float p3 = x[3] == -INFINITY ? 0.0f : ex2(x[3] - mu1[sb]);
            l0[sb] += p0 + p2;
            l1[sb] += p1 + p3;
            // P^T fragment via a per-warp transpose: pt[key][q-row]
            float *pt = pt_s + (warp * QB + sb) * 128;
            *reinterpret_cast<float2 *>(pt + g * 8 + c0) = make_float2(p0, p1);
            *reinterpret_cast<float2 *>(pt + (g + 8) * 8 + c0) = make_float2(p2, p3);
        }
        __syncwarp();
#pragma unroll
        for (int sb = 0; sb < QB; ++sb) {
            const float *pt = pt_s + (warp * QB + sb) * 128;
            pab[sb] = make_float2(pt[(2 * t) * 8 + g], pt[(2 * t + 1) * 8 + g]);
            pcd[sb] = make_float2(pt[(2 * t + 8) * 8 + g], pt[(2 * t + 9) * 8 + g]);
        }

        // ---------------- O^T += V^T P^T (the V fragments serve every block) ----------------
        if constexpr (T == kF16) {
            uint32_t b0[QB], b1[QB];
#pragma unroll
            for (int sb = 0; sb < QB; ++sb) {
                b0[sb] = pack_h2(pab[sb].x, pab[sb].y);
                b1[sb] = pack_h2(pcd[sb].x, pcd[sb].y);
            }
            const uint32_t vl = vg_s + ((lane & 7) + ((lane >> 4) & 1) * 8) * SS +
                                ((lane >> 3) & 1) * 16;
            static_for<MT>([&](auto m_) {
                constexpr int m = decltype(m_)::value;
                uint32_t a0, a1, a2, a3;
                ldsm4t<32 * m>(vl, a0, a1, a2, a3);
#pragma unroll
                for (int sb = 0; sb < QB; ++sb)
                    mma_f16(acc[sb][m], a0, a1, a2, a3, b0[sb], b1[sb]);
            });
        } else {
            const uint32_t vA = vg_s + (2 * t) * SS, vB = vA + SS, vC = vA + 8 * SS,
                           vD = vC + SS;
            const uint32_t lo = T == kQ8 ? 4 * g : 2 * g; // this lane's code bytes
            static_for<NB>([&](auto b_) {
                constexpr int b = decltype(b_)::value;
                constexpr int SO = BB * b, CO = BB * b + 2;
                const float2 sab = make_float2(u16f(lds16<SO>(vA)), u16f(lds16<SO>(vB)));
                const float2 scd = make_float2(u16f(lds16<SO>(vC)), u16f(lds16<SO>(vD)));
                uint32_t b0[QB], b1[QB];
#pragma unroll
                for (int sb = 0; sb < QB; ++sb) {
                    const float2 p01 = __fmul2_rn(pab[sb], sab);
                    const float2 p23 = __fmul2_rn(pcd[sb], scd);
                    b0[sb] = pack_h2(p01.x, p01.y);
                    b1[sb] = pack_h2(p23.x, p23.y);
                }
                if constexpr (T == kQ8) {
                    constexpr bool AL = (CO % 4) == 0;
                    const uint32_t wa = ldsw<CO, AL>(vA + lo) ^ 0x80808080u;
                    const uint32_t wb = ldsw<CO, AL>(vB + lo) ^ 0x80808080u;
                    const uint32_t wc = ldsw<CO, AL>(vC + lo) ^ 0x80808080u;
                    const uint32_t wd = ldsw<CO, AL>(vD + lo) ^ 0x80808080u;
                    // tile 2b: bytes 0 (row g) and 1 (row g+8); tile 2b+1: bytes 2, 3
                    const uint32_t e0 = s8pair_to_h2(__byte_perm(wa, wb, 0x0400));
                    const uint32_t e1 = s8pair_to_h2(__byte_perm(wa, wb, 0x0501));
                    const uint32_t e2 = s8pair_to_h2(__byte_perm(wc, wd, 0x0400));
                    const uint32_t e3 = s8pair_to_h2(__byte_perm(wc, wd, 0x0501));
                    const uint32_t o0 = s8pair_to_h2(__byte_perm(wa, wb, 0x0602));
                    const uint32_t o1 = s8pair_to_h2(__byte_perm(wa, wb, 0x0703));
                    const uint32_t o2 = s8pair_to_h2(__byte_perm(wc, wd, 0x0602));
                    const uint32_t o3 = s8pair_to_h2(__byte_perm(wc, wd, 0x0703));
#pragma unroll
                    for (int sb = 0; sb < QB; ++sb) {
                        mma_f16(acc[sb][2 * b], e0, e1, e2, e3, b0[sb], b1[sb]);
                        mma_f16(acc[sb][2 * b + 1], o0, o1, o2, o3, b0[sb], b1[sb]);
                    }
                } else {
                    const uint32_t xab = __byte_perm(lds16<CO>(vA + lo), lds16<CO>(vB + lo), 0x5410);
                    const uint32_t xcd = __byte_perm(lds16<CO>(vC + lo), lds16<CO>(vD + lo), 0x5410);
                    // tile 2b: low nibbles (dims 2g, 2g+1); tile 2b+1: high nibbles
                    const uint32_t e0 = u4pair_to_h2(xab), e1 = u4pair_to_h2(xab >> 8);
                    const uint32_t e2 = u4pair_to_h2(xcd), e3 = u4pair_to_h2(xcd >> 8);
                    const uint32_t o0 = u4pair_to_h2(xab >> 4), o1 = u4pair_to_h2(xab >> 12);
                    const uint32_t o2 = u4pair_to_h2(xcd >> 4), o3 = u4pair_to_h2(xcd >> 12);
#pragma unroll
                    for (int sb = 0; sb < QB; ++sb) {
                        mma_f16(acc[sb][2 * b], e0, e1, e2, e3, b0[sb], b1[sb]);
                        mma_f16(acc[sb][2 * b + 1], o0, o1, o2, o3, b0[sb], b1[sb]);
                    }
                }
            });
        }
        __syncwarp(); // pt and this stage are reused
    }
    if constexpr (!BULK)
        cp_async_wait<0>();

    // the merge kernel that follows may start launching (it waits for this
    // grid's completion before reading the partials)
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    // ---- per-warp state -> shared memory ----
#pragma unroll
    for (int sb = 0; sb < QB; ++sb)
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            l0[sb] += __shfl_xor_sync(0xffffffffu, l0[sb], o);
            l1[sb] += __shfl_xor_sync(0xffffffffu, l1[sb], o);
        }
    __syncthreads(); // every warp is done with its ring: reuse it for O
    float *ow = reinterpret_cast<float *>(rings); // [NWARP][RQ][OWS]
#pragma unroll
    for (int sb = 0; sb < QB; ++sb) {
        const int r0c = 8 * sb + c0, r1c = 8 * sb + c1;
        if (g == 0) {
            mw_s[warp * RQ + r0c] = mu0[sb];
            mw_s[warp * RQ + r1c] = mu1[sb];
            lw_s[warp * RQ + r0c] = l0[sb];
            lw_s[warp * RQ + r1c] = l1[sb];
        }
        float *o0 = ow + (warp * RQ + r0c) * OWS, *o1 = ow + (warp * RQ + r1c) * OWS;
        const float(&ac)[MT][4] = acc[sb];
        if constexpr (T == kQ8) {
            // dims 32b + 4g .. +3 of one q-row are adjacent: one 16-byte store
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                *reinterpret_cast<float4 *>(o0 + 32 * b + 4 * g) =
                    make_float4(ac[2 * b][0], ac[2 * b][2], ac[2 * b + 1][0], ac[2 * b + 1][2]);
                *reinterpret_cast<float4 *>(o1 + 32 * b + 4 * g) =
                    make_float4(ac[2 * b][1], ac[2 * b][3], ac[2 * b + 1][1], ac[2 * b + 1][3]);
            }
        } else if constexpr (T == kQ4) {
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                *reinterpret_cast<float2 *>(o0 + 32 * b + 2 * g) =
                    make_float2(ac[2 * b][0], ac[2 * b][2]);
                *reinterpret_cast<float2 *>(o0 + 32 * b + 16 + 2 * g) =
                    make_float2(ac[2 * b + 1][0], ac[2 * b + 1][2]);
                *reinterpret_cast<float2 *>(o1 + 32 * b + 2 * g) =
                    make_float2(ac[2 * b][1], ac[2 * b][3]);
                *reinterpret_cast<float2 *>(o1 + 32 * b + 16 + 2 * g) =
                    make_float2(ac[2 * b + 1][1], ac[2 * b + 1][3]);
            }
        } else {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                const int dA = out_dim<T>(m, g), dB = out_dim<T>(m, g + 8);
                o0[dA] = ac[m][0];
                o1[dA] = ac[m][1];
                o0[dB] = ac[m][2];
                o1[dB] = ac[m][3];
            }
        }
    }
    __syncthreads();
    // per q-row: the warps' merge weights (fixed warp order) with the final
    // normalisation folded in, the row's statistics, and its output address
    float4 *wt_s = reinterpret_cast<float4 *>(pt_s);       // [RQ] (pt is free now)
    float **optr_s = reinterpret_cast<float **>(wt_s + RQ); // [RQ]
    int *nf_s = reinterpret_cast<int *>(optr_s + RQ);       // [RQ] non-finite numerator seen
    if (tid < nj) {
        const int j = tid;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NWARP; ++w)
            if (lw_s[w * RQ + j] != 0.0f)
                M = fmaxf(M, mw_s[w * RQ + j]);
        float f[NWARP], L = 0.0f;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) {
            const float lw = lw_s[w * RQ + j];
            f[w] = lw != 0.0f ? ex2(mw_s[w * RQ + j] - M) : 0.0f;
            L += lw * f[w];
        }
        float m_nat = M * kLn2, fin = 1.0f;
        const int jj = jbase + j, iq1 = jj / a.G, h = kvh * a.G + jj % a.G;
        const int64_t orow = ((int64_t)s * a.n_q + iq1) * a.n_head + h;
        float *optr;
        if (a.direct) {
            if (a.sinks) {
                const float sk = a.sinks[h];
                if (L == 0.0f || sk > m_nat) {
                    const float ms = L == 0.0f ? 0.0f : expf(m_nat - sk);
                    fin = ms;
                    L = L * ms + 1.0f;
                    m_nat = sk;
                } else {
                    L += expf(sk - m_nat);
                }
            }
            fin *= L == 0.0f ? 0.0f : 1.0f / L;
            if (a.lse)
                a.lse[orow] = L == 0.0f ? -INFINITY : m_nat + logf(L);
            optr = a.dst + orow * D;
        } else {
            optr = a.partials +
                   ((split - a.split_begin) * (int64_t)a.n_seq * a.n_q * a.n_head + orow) * (D + 2);
            optr[D] = L == 0.0f ? -FLT_MAX : m_nat;
            optr[D + 1] = L;
        }
        static_assert(NWARP == 4, "weights are one float4");
        wt_s[j] = make_float4(f[0] * fin, f[1] * fin, f[2] * fin, f[3] * fin);
        optr_s[j] = optr;
        nf_s[j] = 0;
    }
    __syncthreads();

    // ---- merged output: direct, or the split's partial record ----
    constexpr int HP = D / 2; // dim pairs per q-row
    const bool vec = ((reinterpret_cast<uintptr_t>(a.direct ? a.dst : a.partials)) & 7) == 0;
    for (int idx = tid; idx < nj * HP; idx += NT) {
        const int j = idx / HP, d = 2 * (idx - j * HP);
        const float4 wt = wt_s[j];
        const float2 x0 = *reinterpret_cast<const float2 *>(ow + (0 * RQ + j) * OWS + d);
        const float2 x1 = *reinterpret_cast<const float2 *>(ow + (1 * RQ + j) * OWS + d);
        const float2 x2 = *reinterpret_cast<const float2 *>(ow + (2 * RQ + j) * OWS + d);
        const float2 x3 = *reinterpret_cast<const float2 *>(ow + (3 * RQ + j) * OWS + d);
        float2 o = __fmul2_rn(x0, make_float2(wt.x, wt.x));
        o = __ffma2_rn(x1, make_float2(wt.y, wt.y), o);
        o = __ffma2_rn(x2, make_float2(wt.z, wt.z), o);
        o = __ffma2_rn(x3, make_float2(wt.w, wt.w), o);
        float *p = optr_s[j] + d;
        if (vec) {
            *reinterpret_cast<float2 *>(p) = o;
        } else {
            p[0] = o.x;
            p[1] = o.y;
        }
        if (!a.direct && (!isfinite(o.x) || !isfinite(o.y)))
            atomicOr(&nf_s[j], 1);
    }
    if (!a.direct) {
        // a live record (denominator != 0; the merge skips empty ones) with a
        // non-finite numerator carries a NaN denominator, so that every CTA
        // of the merge sees the row's poison in its (m, l) pass
        __syncthreads();
        if (tid < nj && nf_s[tid] && optr_s[tid][D + 1] != 0.0f)
            optr_s[tid][D + 1] = NAN;
    }
}

// ---------------------------------------------------------------------------
// host side

template <int T, int D, int ST, int QB>
constexpr size_t mma_smem() {
    constexpr int SS = smem_stride(rec_bytes(T, D));
    constexpr size_t RQ = 8 * QB;
    constexpr size_t ring = (size_t)dm::NWARP * ST * 2 * dm::KG * SS;
    constexpr size_t ow = (size_t)dm::NWARP * RQ * (D + 4) * 4;
    size_t b = ring > ow ? ring : ow;
    b += RQ * D * (T == kF16 ? 2 : 1) + (size_t)(D / 32) * RQ * 8; // q codes, dq, qsum
    b += (size_t)dm::NWARP * QB * 128 * 4 + 2 * dm::NWARP * RQ * 4 + RQ * 4 + RQ * 8 + RQ * 4;
    b += (size_t)dm::NWARP * ST * 8; // mbarriers
    return b;
}

// (query, head) rows per CTA of the warp-MMA decode: two q blocks (16 rows)
// once a KV head has more than 16, so that every K/V group a warp loads feeds
// both (multi-query steps: MTP verify, short batches); one block otherwise.
// Config 2's cache, graph-timed step: 4 queries 32.3 against 36.2 us, 9
// queries 65.9 against 94.3 us; at 2 queries (16 rows) one CTA of 16 rows
// measured 22.3 against 21.2 us for two CTAs of 8.
int decode_mma_rows_per_cta(int n_qrows) { return n_qrows > 16 ? 16 : 8; }

bool decode_mma_ok(int type, int D, const DecodeArgs &a) {
    return a.q_convert && (D == 128 || D == 256) &&
           (type == kF16 || type == kQ8 || type == kQ4);
}

// 4D map over one K or V tensor: {row bytes / 2 (u16), n_kv, n_head_kv, n_seq},
// box = one 16-row group of one head.  The last few encodings of each host
// thread are kept: a decode loop calls with the same cache views step after
// step, and encoding is host work on every eager call.
static bool encode_rows_map(CUtensorMap *m, const uint8_t *base, int rec, int n_kv, int n_hkv,
                            int n_seq, int64_t nb1, int64_t nb2, int64_t nb3) {
    struct Entry {
        const uint8_t *base;
        int64_t key[7];
        CUtensorMap map;
    };
    constexpr int kEntries = 8;
    thread_local Entry cache[kEntries];
    thread_local int next = 0;
    const int64_t key[7] = {rec, n_kv, n_hkv, n_seq, nb1, nb2, nb3};
    for (int i = 0; i < kEntries; ++i)
        if (cache[i].base == base && memcmp(cache[i].key, key, sizeof(key)) == 0) {
            *m = cache[i].map;
            return true;
        }
    auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encoder());
    if (!enc || rec % 16 || rec / 2 > 256 || n_kv <= 0)
        return false;
    cuuint64_t dims[4] = {(cuuint64_t)(rec / 2), (cuuint64_t)n_kv, (cuuint64_t)n_hkv,
                          (cuuint64_t)n_seq};
    cuuint64_t strides[3] = {(cuuint64_t)nb1, (cuuint64_t)nb2, (cuuint64_t)nb3};
    cuuint32_t box[4] = {(cuuint32_t)(rec / 2), (cuuint32_t)dm::KG, 1, 1};
    cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<uint8_t *>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    Entry &e = cache[next];
    next = (next + 1) % kEntries;
    e.base = base;
    memcpy(e.key, key, sizeof(key));
    e.map = *m;
    return true;
}

template <int T, int D, int ST, int VW, int QB>
static cudaError_t launch_mma(const DecodeArgs &a, dim3 grid, cudaStream_t st) {
    constexpr size_t smem = mma_smem<T, D, ST, QB>();
    auto kern = fa_decode_mma_kernel<T, D, ST, VW, QB>;
    static std::atomic<unsigned long long> attr_done{0};
    cudaError_t e = set_smem_limit((const void *)kern, smem, attr_done);
    if (e != cudaSuccess)
        return e;
    CUtensorMap maps[2];
    memset(maps, 0, sizeof(maps));
    if constexpr (dm::tma_mode(T, VW)) {
        constexpr int REC = rec_bytes(T, D);
        if (!encode_rows_map(&maps[0], a.k, REC, a.n_kv, a.n_head_kv, a.n_seq / a.rk3, a.k_nb1,
                             a.k_nb2, a.k_nb3) ||
            !encode_rows_map(&maps[1], a.v, REC, a.n_kv, a.n_head_kv, a.n_seq / a.rv3, a.v_nb1,
                             a.v_nb2, a.v_nb3))
            return cudaErrorNotSupported; // nothing launched: the caller picks another path
    }
    // programmatic dependent of the previous kernel on the stream: the kernel
    // prefetches K/V into L2 before its griddepcontrol.wait
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(dm::NT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], a);
}

// CTAs of the variant launch_mma<T, D, ST, VW, QB> that fit on one SM (its
// shared memory and register bound), asked once per device and variant.
template <int T, int D, int ST, int VW, int QB>
static int occupancy_of() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return 2;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n > 0)
        return n;
    constexpr size_t smem = mma_smem<T, D, ST, QB>();
    auto kern = fa_decode_mma_kernel<T, D, ST, VW, QB>;
    static std::atomic<unsigned long long> attr_done{0};
    if (set_smem_limit((const void *)kern, smem, attr_done) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, dm::NT, smem) != cudaSuccess ||
        n <= 0) {
        cudaGetLastError();
        return 2;
    }
    cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

template <int T, int D, int QB>
static int mma_occupancy(int vw) {
    constexpr int ST = smem_stride(rec_bytes(T, D)) <= 288 ? 3 : 2;
    if constexpr (rec_bytes(T, D) % 16 == 0)
        if (vw == 16) {
            constexpr int STV = dm::tma_mode(T, 16) ? (T == kQ4 ? 4 : 2) : ST;
            return occupancy_of<T, D, STV, 16, QB>();
        }
    if constexpr (rec_bytes(T, D) % 8 == 0)
        if (vw >= 8)
            return occupancy_of<T, D, ST, 8, QB>();
    return occupancy_of<T, D, ST, 4, QB>();
}

template <int T>
static int occupancy_td(int D, int vw, int qb) {
    if (D == 128)
        return qb == 2 ? mma_occupancy<T, 128, 2>(vw) : mma_occupancy<T, 128, 1>(vw);
    return qb == 2 ? mma_occupancy<T, 256, 2>(vw) : mma_occupancy<T, 256, 1>(vw);
}

int decode_mma_occupancy(int type, int D, int vw, int n_qrows) {
    const int qb = decode_mma_rows_per_cta(n_qrows) / 8;
    switch (type) {
    case kF16: return occupancy_td<kF16>(D, vw, qb);
    case kQ8: return occupancy_td<kQ8>(D, vw, qb);
    default: return occupancy_td<kQ4>(D, vw, qb);
    }
}

template <int T, int D, int QB>
static cudaError_t mma_vw(const DecodeArgs &a, int vw, dim3 grid, cudaStream_t st) {
    constexpr int ST = smem_stride(rec_bytes(T, D)) <= 288 ? 3 : 2;
    if constexpr (rec_bytes(T, D) % 16 == 0)
        if (vw == 16) {
            // TMA boxes.  Q8_0: two stages (one group in flight behind the one
            // in use) measured faster than three, as the first wave of requests
            // is smaller.  Q4_0 boxes are half as large and two stages leave the
            // stream short of requests: four (three groups in flight per warp,
            // still two CTAs per SM) measured 15.2 against 17.9 us on config 2.
            constexpr int STV = dm::tma_mode(T, 16) ? (T == kQ4 ? 4 : 2) : ST;
            const cudaError_t e = launch_mma<T, D, STV, 16, QB>(a, grid, st);
            if (e != cudaErrorNotSupported)
                return e;
            vw = 8; // the layout has no tensor map: per-lane copies
        }
    if constexpr (rec_bytes(T, D) % 8 == 0)
        if (vw >= 8)
            return launch_mma<T, D, ST, 8, QB>(a, grid, st);
    return launch_mma<T, D, ST, 4, QB>(a, grid, st);
}

template <int T>
static cudaError_t mma_td(const DecodeArgs &a, int D, int vw, dim3 grid, cudaStream_t st) {
    // the callers' grid counts CTAs of decode_mma_rows_per_cta(n_qrows) rows
    const bool two = decode_mma_rows_per_cta(a.n_qrows) == 16;
    if (D == 128)
        return two ? mma_vw<T, 128, 2>(a, vw, grid, st) : mma_vw<T, 128, 1>(a, vw, grid, st);
    return two ? mma_vw<T, 256, 2>(a, vw, grid, st) : mma_vw<T, 256, 1>(a, vw, grid, st);
}

cudaError_t launch_decode_mma(const DecodeArgs &a, int type, int D, int vw, dim3 grid,
                              cudaStream_t st) {
    switch (type) {
    case kF16: return mma_td<kF16>(a, D, vw, grid, st);
    case kQ8: return mma_td<kQ8>(a, D, vw, grid, st);
    default: return mma_td<kQ4>(a, D, vw, grid, st);
    }
}

} // namespace xq
