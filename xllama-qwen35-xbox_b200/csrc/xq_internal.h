// Internal (C++) interface between the C-ABI layer and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace xq {

// Raise a kernel's dynamic shared-memory limit on the current device once.
// The attribute belongs to the kernel on one device, so one process driving
// several GPUs needs it set on each: `done` holds one bit per device ordinal.
inline cudaError_t set_smem_limit(const void *kern, size_t smem,
                                  std::atomic<unsigned long long> &done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return e;
    const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
    if (bit && (done.load(std::memory_order_acquire) & bit))
        return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess && bit)
        done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

// One split-KV decode launch.  Byte strides follow ggml nb[].
struct DecodeArgs {
    const uint8_t *q;
    int64_t q_nb1, q_nb2, q_nb3;
    const uint8_t *k;
    int64_t k_nb1, k_nb2, k_nb3;
    const uint8_t *v;
    int64_t v_nb1, v_nb2, v_nb3;
    const uint8_t *mask; // F16 or null
    int64_t m_nb1, m_nb2, m_nb3;
    int m_ne2, m_ne3;
    const int32_t *positions; // RKVA causal limit per query, or null
    int origin, active;
    float *dst;      // direct mode: F32 [D, n_head, n_q, n_seq]
    float *lse;      // direct mode, optional: [n_seq][n_q][n_head]
    float *partials; // partial mode: [split - split_begin][n_rows][D + 2]
    const float *sinks; // direct mode only
    int n_q, n_head, n_head_kv, n_seq, n_kv;
    int G;          // q heads per kv head
    int rk3, rv3;   // n_seq / ne3 of k, v
    int n_qrows;    // n_q * G
    int64_t rows_per_split, split_begin;
    int direct;     // 1: single split writes dst; 0: write partial records
    int q_convert;  // 1: ggml converts q to the K dot type; 0: raw F32 (RKVA)
    float scale, softcap, m0, m1;
    int n_head_log2, alibi;
    int *err; // optional: set non-zero when a bounded wait gives up
};

struct DecodeConfig {
    int type, D, NR, R, VW;
    size_t smem;
};

// Pick NR/R/VW/shared memory for a shape; returns false if unsupported.
bool decode_config(int type, int D, int n_qrows, const DecodeArgs &a, DecodeConfig *cfg);
cudaError_t launch_decode(const DecodeArgs &a, const DecodeConfig &cfg, dim3 grid,
                          cudaStream_t st);
// Tensor-core (warp MMA) decode: 8 q-rows per CTA, ggml q conversion only.
bool decode_mma_ok(int type, int D, const DecodeArgs &a);
cudaError_t launch_decode_mma(const DecodeArgs &a, int type, int D, int vw, dim3 grid,
                              cudaStream_t st);
// (query, head) rows per CTA of the warp-MMA decode for n_qrows rows per KV
// head (8, or 16 when the KV head has more than 16: two q blocks per K/V load).
int decode_mma_rows_per_cta(int n_qrows);
// Resident CTAs per SM of the warp-MMA decode variant launch_decode_mma picks.
int decode_mma_occupancy(int type, int D, int vw, int n_qrows);
// n_groups > 1 merges consecutive blocks of n_splits splits separately; with
// records, the merged rows are written as partial records (see lse_merge_kernel).
// flagged: the partials come from fa_decode_mma_kernel, which gives a record
// whose numerator is not finite a NaN denominator, so the merge needs no
// cross-CTA exchange of poison flags (same results).
cudaError_t launch_merge(const float *partials, int64_t n_splits, int64_t n_rows, int D,
                         float *out, float *lse, const float *sinks, int n_head,
                         cudaStream_t st, int64_t n_groups = 1, bool records = false,
                         bool flagged = false);

// One tensor-core prefill launch (F32 q / dst; F16 K/V, or Q8_0 / Q4_0 K/V
// widened to f16 in the workspace first).
struct PrefillShape {
    const uint8_t *q;
    int64_t q_nb[4];
    const void *k, *v;
    int64_t k_nb[4], v_nb[4];
    int kv_type; // XQ_TYPE_F16 / Q8_0 / Q4_0
    const uint8_t *mask; // F16 or null
    int64_t m_nb1, m_nb2, m_nb3;
    int m_ne2, m_ne3, m_planes;
    float *dst;
    int D, n_q, n_head, n_head_kv, n_seq, n_seq_kv, n_kv;
    float scale;
};
// Workspace of one launch: the mask block map and an error word, then (Q8_0 /
// Q4_0) the f16 copies of K and V.
size_t prefill_ws_bytes(const PrefillShape &ps);
// The driver's cuTensorMapEncodeTiled (PFN_cuTensorMapEncodeTiled_v12000), or null.
void *tensor_map_encoder();
cudaError_t launch_prefill(const PrefillShape &ps, void *ws, cudaStream_t st, const char **why);

// ggml SET_ROWS: F32 rows -> rows of a F32/F16/Q8_0/Q4_0 tensor at I32/I64 indices.
struct SetRowsArgs {
    const uint8_t *src;             // F32 [ne0, ne1, ne2, ne3]
    int64_t s_nb1, s_nb2, s_nb3;
    const uint8_t *idx;             // I32/I64 [ne1, i_ne1, i_ne2]
    int64_t i_nb0, i_nb1, i_nb2, i_ne1, i_ne2;
    int idx_i64;
    uint8_t *dst;                   // [ne0, d_rows, ne2, ne3]
    int64_t d_nb1, d_nb2, d_nb3, d_rows;
    int64_t ne0, ne1, ne2, ne3, n_units;
    int n_sm; // SMs of the device (persistent grids)
};
cudaError_t launch_set_rows(int type, const SetRowsArgs &a, cudaStream_t st);

struct GdnArgs {
    const float *q, *k, *v, *g, *beta, *state;
    int64_t q_nb1, q_nb2, q_nb3, k_nb1, k_nb2, k_nb3, v_nb1, v_nb2, v_nb3;
    int64_t g_nb1, g_nb2, g_nb3, b_nb1, b_nb2, b_nb3, s_nb1, s_nb2, s_nb3;
    float *dst;
    int H, H_k, T, n_seq, rq3, rk3, slots;
    float scale;
    int t_begin = 0; // tokens before this one are already folded into `state`
    int h_off = 0;   // global index of value head 0: value head h reads key head (h + h_off) % H_k
};
cudaError_t launch_gdn(const GdnArgs &a, cudaStream_t st);
// Chunked (WY) form on the tensor cores for long sequences: workspace bytes
// (0 when the shape has fewer than one chunk), eligibility (16-byte aligned
// q/k/v rows, at least two chunks) and the launch (prep, scan, and the
// per-token kernel for the snapshot tail).
size_t gdn_chunk_workspace(int T, int H, int n_seq, int slots);
bool gdn_chunk_eligible(const GdnArgs &a);
cudaError_t launch_gdn_chunked(const GdnArgs &a, void *ws, size_t ws_bytes, cudaStream_t st);

// Native KVarN4 range-attention partials (xq_kvarn4.cu): one (acc[256], max,
// denom) record per (split, token, query head); splits cover rows_per_split
// rows, a multiple of 128.
struct Kvarn4Launch {
    const uint8_t *k, *v;
    const float *q;
    const int32_t *positions;
    float *partials;
    int64_t records_bytes;
    // splits [0, n_body) cover rows [0, active - tail) in rows_per_split
    // chunks (rotated domain); split n_body, when n_splits > n_body, covers the
    // precision tail (original domain)
    int origin, active, tail, n_head, n_head_kv, n_tokens, rows_per_split, n_body, n_splits;
    float scale;
};
cudaError_t launch_kvarn4(const Kvarn4Launch &l, cudaStream_t st);

// KV-sharded decode exchange (xq_shard.cu).
constexpr int kShardMaxRanks = 16;
struct ShardPushArgs {
    const float2 *src;  // this rank's group records, contiguous
    int64_t n8;         // their size in 8-byte units
    int64_t dst_off8;   // where they start in a half (8-byte units)
    size_t half_off;    // byte offset of the step's half in an exchange buffer
    size_t ctl_off;     // byte offset of the counters
    int parity;
    uint8_t *peers[kShardMaxRanks];
};
size_t shard_records_bytes(int64_t n_groups, int64_t n_rows, int D);
size_t shard_exchange_bytes(int64_t n_groups, int64_t n_rows, int D);
size_t shard_ctl_off(int64_t n_groups, int64_t n_rows, int D);
int64_t shard_chunks(size_t bytes);
cudaError_t launch_shard_push(const ShardPushArgs &a, int world, cudaStream_t st);
cudaError_t launch_shard_wait(void *exchange, int64_t n_groups, int64_t n_rows, int D,
                              int parity, unsigned expected, cudaStream_t st);

cudaError_t launch_dequant(int type, const void *src, uint64_t src_stride, float *dst,
                           uint64_t dst_stride, int64_t n_rows, int64_t n_per_row,
                           cudaStream_t st);
cudaError_t launch_quant(int type, const float *src, uint64_t src_stride, void *dst,
                         uint64_t dst_stride, int64_t n_rows, int64_t n_per_row,
                         cudaStream_t st);

} // namespace xq
