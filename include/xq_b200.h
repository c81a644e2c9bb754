/*
 * xq_b200.h -- C ABI of the B200 attention hot path (libxq_b200.so).
 *
 * Plain pointers, ggml ne/nb strides, a CUDA stream and an int status: no
 * torch or C++ types cross this boundary.  All tensor pointers are device
 * pointers unless stated otherwise.  Every entry point is asynchronous on the
 * given stream and returns XQ_OK or an XQ_ERR_* code; a kernel-launch failure
 * returns XQ_ERR_CUDA and xq_last_error() has the CUDA message.
 *
 * Each entry point replaces one reference interface (file:line in
 * hjotha/xllama-qwen35-xbox, whose ggml-cpu kernels live in the llama.cpp
 * submodule beellama.cpp @ 982eaadaa9dbe761f00205bc20b6c04b7329b58d):
 *
 *   xq_flash_attn_ext     GGML_OP_FLASH_ATTN_EXT as dispatched by the ggml
 *                         scheduler to ggml-cpu
 *                         (bench/results/diag-ubatch-20261007/snapshot-r108/
 *                         llama.cpp_ggml_src_ggml-cpu_ggml-cpu.c:2085-2088),
 *                         incl. the split-KV decode branch
 *                         (patches/0006-cpu-flash-attn-consistent-kv-reduction.patch:7-14)
 *   xq_gated_delta_net    GGML_OP_GATED_DELTA_NET (ggml-cpu.c:2148-2150 and the
 *                         D3D12 kernel dispatch src/bridge/ggml_d3d12.cpp:1905-1941)
 *   xq_gated_delta_net_ws the same op in chunked form for long prefill (the
 *                         CPU op's per-token loop, ops.cpp of the snapshot,
 *                         restated as 64-token WY chunks on the tensor cores)
 *   xq_gated_delta_net_heads  the same op over a block of value heads (the
 *                         D3D12 dispatch over value heads,
 *                         src/bridge/ggml_d3d12.cpp:1937, cut by head)
 *   xq_attend_range       RemoteAttnEngine::attend_range
 *                         (uwp/rkva/remote-attn-engine.h:152-154,
 *                          remote-attn-engine.cpp:2774-3251)
 *   xq_fa_shard_push /    the KV position split across devices with an
 *   xq_fa_shard_finish    (O, LSE) merge (uwp/rkva/remote-attn-engine.cpp:
 *                         2928-2978), across the GPUs of one box
 *   xq_fa_partials +      split partials + LSE reduction
 *   xq_lse_merge          (shaders/rkva/rkva_range_attn.hlsl:59-106,
 *                          rkva_range_reduce_opt.hlsl:26-133)
 *   xq_attend_range_kvarn4  RemoteAttnEngine::attend_range over native KVarN4
 *                         records (shaders/rkva/rkva_range_attn_kvarn4.hlsl)
 *   xq_split_k            rkva_rprof::reference_split_k / optimized_split_k
 *                         (uwp/rkva/rkva-range-profile.h:98-111)
 *   xq_dequantize_rows    ggml to_float for F16/Q8_0/Q4_0 (ggml-quants.c)
 *   xq_quantize_rows      ggml from_float reference quantizers (the KV-cache
 *                         write path, shaders/rkva/rkva_store_f16.hlsl)
 *   xq_set_rows           GGML_OP_SET_ROWS, the KV-cache write node
 *                         (ggml-cpu dispatch: ggml-cpu.c:1957-1959 of the
 *                         snapshot under bench/results/diag-ubatch-20261007;
 *                         node `cache_k_l1 (view)` in
 *                         docs/training-architecture.md:278-282)
 */
#ifndef XQ_B200_H
#define XQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *xq_stream_t; /* == cudaStream_t */

enum xq_status {
    XQ_OK = 0,
    XQ_ERR_INVALID = 1,     /* bad argument / shape contract violated */
    XQ_ERR_UNSUPPORTED = 2, /* valid ggml op this library does not claim */
    XQ_ERR_CUDA = 3,        /* a CUDA call failed; see xq_last_error() */
    XQ_ERR_WORKSPACE = 4,   /* workspace missing or too small */
};

/* ggml type ids (ggml.h enum ggml_type values, stable across versions). */
enum xq_type {
    XQ_TYPE_F32 = 0,
    XQ_TYPE_F16 = 1,
    XQ_TYPE_Q4_0 = 2,
    XQ_TYPE_Q8_0 = 8,
    XQ_TYPE_I32 = 26, /* row indices (SET_ROWS) */
    XQ_TYPE_I64 = 27
};

/* A ggml tensor view: ne = elements per dim, nb = byte strides. */
typedef struct {
    int32_t type;
    int32_t reserved;
    const void *data;
    int64_t ne[4];
    uint64_t nb[4];
} xq_tensor;

/* ------------------------------------------------------------------------ */
/* GGML_OP_FLASH_ATTN_EXT                                                    */
/*   q    F32  [DK, n_q, n_head, n_seq]                                      */
/*   k    F16/Q8_0/Q4_0 [DK, n_kv, n_head_kv, n_seq_kv]  (n_head % n_head_kv */
/*        == 0, n_seq % n_seq_kv == 0: ggml broadcast)                        */
/*   v    same type as k, [DV, n_kv, n_head_kv, n_seq_kv], DV == DK          */
/*   mask F16 [n_kv, >= n_q, m2, m3] or data == NULL (broadcast by modulo)   */
/*   sinks F32 [n_head] or NULL                                               */
/*   dst  F32 [DV, n_head, n_q, n_seq] contiguous                             */
/*   op_params: scale, max_bias, logit_softcap (ggml op_params[0..2])         */
/* DK in {64, 128, 256}.  Decode-shaped calls (n_q * n_head / n_head_kv <=   */
/* 16) run the split-KV kernel; larger F16 calls run the tensor-core prefill */
/* kernel.  Workspace: xq_flash_attn_ext_workspace() bytes, any contents;    */
/* it may be NULL when that size is 0.  q and dst may be pinned host memory:  */
/* q is then copied to the workspace by a kernel of this library and dst is  */
/* written in place; pageable host pointers return XQ_ERR_INVALID.           */
/* ------------------------------------------------------------------------ */
typedef struct {
    xq_tensor q, k, v, mask;
    const float *sinks;
    float *dst;
    float scale, max_bias, softcap;
    int32_t n_splits; /* 0: automatic (fill the GPU), else KV splits per head */
} xq_fa_params;

size_t xq_flash_attn_ext_workspace(const xq_fa_params *p);
int xq_flash_attn_ext(const xq_fa_params *p, void *workspace, size_t workspace_bytes,
                      xq_stream_t stream);
/* The plan xq_flash_attn_ext makes for these parameters on the current      */
/* device (host function; no launch): kernel 0 the CUDA-core split-KV       */
/* decode, 1 the warp-MMA split-KV decode, 2 the tensor-core prefill; for   */
/* the decodes the KV split count and rows per split (0 for the prefill).   */
/* A caller reproducing the call's split records with xq_fa_partials       */
/* passes these.  (ggml-cpu's thread split, ggml-cpu.c:2522 of the snapshot, */
/* is the reference's counterpart.)                                          */
int xq_flash_attn_ext_plan(const xq_fa_params *p, int32_t *kernel, int64_t *n_splits,
                           int64_t *rows_per_split);

/* ------------------------------------------------------------------------ */
/* Split partials for sharded / remote decode.                               */
/* Same tensors as xq_flash_attn_ext (mask/sinks allowed), but the KV rows   */
/* are cut into fixed global splits of rows_per_split rows; this call        */
/* computes splits [split_begin, split_end) and writes their records to      */
/* partials[(s - split_begin) * n_rows + row] * (DV + 2) floats =            */
/* (acc[DV] unnormalised, max, denom), row = (seq * n_q + iq1) * n_head + h. */
/* An empty split writes (0, -FLT_MAX, 0).  The records of all splits,       */
/* gathered in split order from any number of GPUs, merge bit-identically.   */
/* ------------------------------------------------------------------------ */
int xq_fa_partials(const xq_fa_params *p, int64_t rows_per_split, int64_t split_begin,
                   int64_t split_end, float *partials, xq_stream_t stream);

/* partials [n_splits][n_rows][D+2] -> out [n_rows][D] (F32) and, if lse is  */
/* not NULL, lse [n_rows] (natural log).  Fixed split order; empty splits    */
/* (denom == 0) are skipped; all empty => O = 0, LSE = -inf; a participating */
/* non-finite state poisons the row with NaN (rkva_range_reduce_opt.hlsl).   */
/* partials must be 4-byte aligned; 8-byte aligned partials (any cudaMalloc  */
/* pointer) take the faster wide-load kernels, with bit-identical results.   */
int xq_lse_merge(const float *partials, int64_t n_splits, int64_t n_rows, int64_t D,
                 float *out, float *lse, xq_stream_t stream);

/* First level of a two-level merge (the reduce step of the reference's      */
/* split-K reduction, rkva_range_reduce_opt.hlsl:26-133, applied per group).  */
/* partials [n_groups * splits_per_group][n_rows][D+2] -> records            */
/* [n_groups][n_rows][D+2]: group g merges its splits in order and writes    */
/* (O, lse, 1), (0, -FLT_MAX, 0) when empty, NaN when poisoned.  The records  */
/* merge again with xq_lse_merge exactly like splits; with a fixed grouping  */
/* the result is bit-identical however the groups are spread over GPUs.      */
int xq_lse_merge_records(const float *partials, int64_t n_groups, int64_t splits_per_group,
                         int64_t n_rows, int64_t D, float *records, xq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* KV-sharded decode across the GPUs of one box (one process per GPU).      */
/* The reference splits a sequence's KV cache by position between devices  */
/* and merges their (O, LSE) partials (uwp/rkva/remote-attn-engine.cpp:     */
/* 2928-2978; the RANGE_ATTN reply, uwp/rkva/remote-attn-protocol.h:205-    */
/* 236).  Here the KV rows of every sequence are cut into fixed global     */
/* splits of rows_per_split rows and the splits into n_groups groups of    */
/* splits_per_group; rank r holds the groups [b, e) of a contiguous block   */
/* split (n_groups / world each, the first n_groups % world ranks one more) */
/* -- its k / v views start at row 0 of its first split -- and each step:   */
/*   xq_fa_shard_push    its splits' partial records, one (O, lse, 1)       */
/*                       record per group (in split order), stored with    */
/*                       NVLink peer stores into every rank's exchange      */
/*                       buffer;                                            */
/*   xq_fa_shard_finish  waits (bounded, 2 s) until every rank's records of */
/*                       this step arrived, merges all n_groups records in */
/*                       group order into out / lse (+ sinks).              */
/* The grouping and both merge orders depend only on the plan's global     */
/* numbers, so out is bit-identical for every world size.  Exchange       */
/* buffer: xq_shard_exchange_bytes(n_groups, n_rows, D) bytes from         */
/* xq_shard_exchange_alloc on each rank's GPU (zeroed); share it with      */
/* xq_ipc_export / xq_ipc_open (CUDA IPC; the caller moves the 64-byte      */
/* handles between processes) and list every rank's buffer as this rank    */
/* maps it in plan.exchange (its own at [rank]).  step: +1 per step on     */
/* every rank (its parity picks the buffer half; replays of a captured     */
/* sequence need an even number of steps).  After a timeout (NaN output)   */
/* re-create the exchange buffers on every rank.                           */
/* n_rows = n_seq * n_q * n_head.  No TMA and no multicast touch peer      */
/* memory: plain stores and one system-scope atomic per 16 KB chunk.       */
/* ------------------------------------------------------------------------ */
#define XQ_SHARD_MAX_RANKS 16
typedef struct {
    unsigned char bytes[64]; /* == cudaIpcMemHandle_t */
} xq_ipc_handle;
typedef struct {
    int64_t rows_per_split, splits_per_group, n_groups;
    int32_t rank, world;
    uint32_t step;
    int32_t reserved;
    void *exchange[XQ_SHARD_MAX_RANKS];
} xq_shard_plan;
size_t xq_shard_exchange_bytes(int64_t n_groups, int64_t n_rows, int64_t D);
int xq_shard_exchange_alloc(size_t bytes, void **exchange); /* setup: cudaMalloc + zero */
int xq_shard_exchange_free(void *exchange);
/* Host read of the exchange buffer's error word (synchronizes the stream):  */
/* 1 once a finish call's wait ran out (its output is NaN), else 0.          */
int xq_shard_exchange_error(const void *exchange, int64_t n_groups, int64_t n_rows, int64_t D,
                            xq_stream_t stream, int32_t *error);
int xq_ipc_export(const void *dev_ptr, xq_ipc_handle *handle);
int xq_ipc_open(const xq_ipc_handle *handle, void **dev_ptr);
int xq_ipc_close(void *dev_ptr);
size_t xq_fa_shard_workspace(const xq_fa_params *p, const xq_shard_plan *s);
int xq_fa_shard_push(const xq_fa_params *p, const xq_shard_plan *s, void *workspace,
                     size_t workspace_bytes, xq_stream_t stream);
int xq_fa_shard_finish(const xq_shard_plan *s, int64_t n_rows, int64_t D, const float *sinks,
                       int32_t n_head, float *out, float *lse, xq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* RKVA RANGE_ATTN: (O, LSE) over a compact KV range [0, active) whose row r */
/* holds absolute position origin + r.  k/v: [capacity][n_head_kv][D] in     */
/* storage type (F16/Q8_0/Q4_0); q: F32 [n_tokens][n_head][D]; positions:    */
/* int32 [n_tokens] absolute.  Query t attends rows                          */
/* [0, min(active, positions[t] - origin + 1)).  out F32 [n_tokens][n_head]  */
/* [D], lse F32 [n_tokens][n_head].  Empty => O = 0, LSE = -inf.             */
/* split_mode: 0 reference policy, 1/2/3 balanced/fine/coarse, 4 automatic.  */
/* positions must be device memory; workspace per                            */
/* xq_attend_range_workspace().                                              */
/* ------------------------------------------------------------------------ */
size_t xq_attend_range_workspace(int32_t storage, uint32_t n_tokens, uint32_t active,
                                 uint32_t n_head, uint32_t n_head_kv, uint32_t head_dim,
                                 uint32_t split_mode);
int xq_attend_range(int32_t storage, const void *k, const void *v, uint32_t n_head,
                    uint32_t n_head_kv, uint32_t head_dim, uint32_t origin, uint32_t active,
                    uint32_t n_tokens, const int32_t *positions, const float *q, float kq_scale,
                    uint32_t split_mode, float *out, float *lse, void *workspace,
                    size_t workspace_bytes, xq_stream_t stream);

/* Split count of the reference policies (host function, no GPU). */
uint32_t xq_split_k(uint32_t active, uint32_t mode);

/* ------------------------------------------------------------------------ */
/* RKVA native KVarN4 range attention (descriptor v1 resident image; the    */
/* reference's RemoteAttnEngine::attend_range over storage KVarN4,          */
/* docs/rkva-kvarn-range.md "Descriptor and records",                        */
/* shaders/rkva/rkva_range_attn_kvarn4.hlsl:64-150).  head_dim 256 = two     */
/* 128-dim physical slices per KV head.  Each plane (K, V), 16-byte aligned: */
/*   records [ceil(capacity/128)][2 n_head_kv][8960 B]: 4-bit values low     */
/*           nibble first as a 128 x 128 matrix (K [dim][token], V [token]  */
/*           [dim]), 128 F16 scales, 128 F16 zeros (per row), 128 F16        */
/*           factors (per column); value = (q * scale + zero) * factor       */
/*   stage   [384][n_head_kv][256] F16 rotated rows (slot 0 global group 0,  */
/*           1 + (g - 1) % 2 otherwise)                                     */
/*   tail    [128][n_head_kv][256] F16 original-domain rows (row % 128),     */
/*           present when precision_tail == 128                             */
/* Rows >= active - precision_tail come from the tail; global group 0 and  */
/* the incomplete live group from the stage; the rest from the records.    */
/* Rotated rows (WHT256 = Sylvester H256 / 16) meet WHT(q) and their value  */
/* numerator is rotated back.  Query t sees rows [0, min(active,           */
/* positions[t] - origin + 1)).  q F32 [n_tokens][n_head][256] original     */
/* domain; out F32 [n_tokens][n_head][256]; lse F32 [n_tokens][n_head]     */
/* (natural log; empty => O = 0, LSE = -inf; lse may be NULL).  q, out and */
/* lse may be in device or pinned host memory (q is then staged into the   */
/* workspace by a kernel, out / lse written over PCIe by the merge);       */
/* pageable host memory => XQ_ERR_INVALID.  positions: device memory.      */
/* The workspace holds the split partials and room to stage q.             */
/* ------------------------------------------------------------------------ */
typedef struct {
    int32_t origin;         /* global position of compact row 0, % 128 == 0 */
    int32_t capacity;       /* rows the planes hold */
    int32_t precision_tail; /* 0 or 128 */
    int32_t n_head_kv;
} xq_kvarn4_desc;
size_t xq_attend_range_kvarn4_workspace(const xq_kvarn4_desc *d, uint32_t n_head,
                                        uint32_t active, uint32_t n_tokens);
int xq_attend_range_kvarn4(const xq_kvarn4_desc *d, const void *k_plane, const void *v_plane,
                           uint32_t n_head, uint32_t active, uint32_t n_tokens,
                           const int32_t *positions, const float *q, float kq_scale, float *out,
                           float *lse, void *ws, size_t ws_bytes, xq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* GGML_OP_GATED_DELTA_NET                                                   */
/*   q, k  F32 [S, H_k, T, n_seq_qk]   (rows contiguous, any head/token      */
/*         stride); value head h reads key head h % H_k                      */
/*   v     F32 [S, H, T, n_seq]                                               */
/*   g, beta F32 [1, H, T, n_seq]  (scalar gates, already activated)         */
/*   state F32 [S, S, H, n_seq]    (state[seq][h][col][i])                    */
/*   dst   F32, contiguous: y [n_seq][T][H][S] then K snapshot slots, each  */
/*         [n_seq][H][S][S]; slot 0 = state after the last token, slot j =  */
/*         j tokens earlier; slots older than the first token are untouched. */
/* S = 128.  slots = op_params[0] in [1, 64].                                */
/* ------------------------------------------------------------------------ */
int xq_gated_delta_net(const xq_tensor *q, const xq_tensor *k, const xq_tensor *v,
                       const xq_tensor *g, const xq_tensor *beta, const xq_tensor *state,
                       float *dst, int32_t slots, xq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* GATED_DELTA_NET for long sequences (prefill), same contract as above, in  */
/* chunked (WY) form: 64-token chunks, the per-chunk products on the tensor  */
/* cores with TF32 operands and FP32 accumulation (error vs the sequential   */
/* FP32 recurrence ~1e-3 of max|y|, inside max-abs 2e-3 / rel 1e-2), the     */
/* state carried in FP32.  Used when T spans at least two chunks and q/k/v   */
/* rows are 16-byte aligned; otherwise (and for T <= 64) it runs exactly     */
/* xq_gated_delta_net.  workspace: device memory, 256-byte aligned, of       */
/* xq_gated_delta_net_workspace(v, slots) bytes (0: none needed); too small  */
/* => XQ_ERR_WORKSPACE.  With slots > 1 the last `slots` tokens run the      */
/* per-token kernel, which writes the snapshots.                             */
/* ------------------------------------------------------------------------ */
size_t xq_gated_delta_net_workspace(const xq_tensor *v, int32_t slots);
int xq_gated_delta_net_ws(const xq_tensor *q, const xq_tensor *k, const xq_tensor *v,
                          const xq_tensor *g, const xq_tensor *beta, const xq_tensor *state,
                          float *dst, int32_t slots, void *workspace, size_t workspace_bytes,
                          xq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* GATED_DELTA_NET over a block of value heads: the op sharded by value    */
/* head across GPUs (one process per GPU, no exchange step).  The block is */
/* value heads [head_begin, head_begin + v->ne[1]) of an op with            */
/* n_head_total value heads (n_head_total % H_k == 0): v, g, beta, state    */
/* and dst cover the block only (their head dims hold v->ne[1] heads; dst   */
/* is the block's y [n_seq][T][block][S] then its snapshot slots            */
/* [n_seq][block][S][S]); q and k are the op's full key-head tensors, and   */
/* block head j reads key head (head_begin + j) % H_k -- the mapping of the */
/* whole op (the reference's h mod H_k, src/bridge/ggml_d3d12.cpp:143), so  */
/* every block's outputs equal the whole op's outputs for its heads bit for */
/* bit.  Workspace and kernel choice as xq_gated_delta_net_ws, sized by    */
/* xq_gated_delta_net_workspace(v, slots) of the block's v.  The reference  */
/* runs the op on one device (Dispatch(32, 1, 16) over the value heads,     */
/* src/bridge/ggml_d3d12.cpp:1937); this is that dispatch cut by head.      */
/* ------------------------------------------------------------------------ */
int xq_gated_delta_net_heads(const xq_tensor *q, const xq_tensor *k, const xq_tensor *v,
                             const xq_tensor *g, const xq_tensor *beta, const xq_tensor *state,
                             float *dst, int32_t slots, int64_t head_begin, int64_t n_head_total,
                             void *workspace, size_t workspace_bytes, xq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* GGML_OP_SET_ROWS (quantize-on-append into the KV cache).  src F32         */
/* [ne0, ne1, ne2, ne3] with contiguous rows; idx I32 or I64 [ne1, i1, i2]   */
/* (ne2 % i1 == 0, ne3 % i2 == 0); dst F32/F16/Q8_0/Q4_0 [ne0, rows, ne2,    */
/* ne3] (ne0 % 32 == 0 for Q8_0/Q4_0).  Row (r, j, k) of src is written,     */
/* converted by ggml's reference quantizer (bit-exact with                   */
/* quantize_row_q8_0_ref / q4_0_ref and fp32->fp16 round-to-nearest-even),   */
/* to row idx[r, j % i1, k % i2] of dst plane (j, k).  An index outside      */
/* [0, rows) skips its row (ggml-cpu asserts instead).                        */
/* ------------------------------------------------------------------------ */
int xq_set_rows(const xq_tensor *src, const xq_tensor *idx, const xq_tensor *dst,
                xq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Block codecs.  n_per_row multiple of 32 for Q8_0/Q4_0.  Rows at byte      */
/* stride src_row_stride / dst_row_stride.                                   */
/* ------------------------------------------------------------------------ */
int xq_dequantize_rows(int32_t type, const void *src, uint64_t src_row_stride, float *dst,
                       uint64_t dst_row_stride, int64_t n_rows, int64_t n_per_row,
                       xq_stream_t stream);
int xq_quantize_rows(int32_t type, const float *src, uint64_t src_row_stride, void *dst,
                     uint64_t dst_row_stride, int64_t n_rows, int64_t n_per_row,
                     xq_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Allocation-free FLASH_ATTN_EXT (this entry point has no counterpart in   */
/* the reference).                                                           */
/*                                                                           */
/* Some callers cannot allocate device memory while attention runs: a host  */
/* whose device memory was fully planned ahead by its own allocator (ggml's */
/* graph allocator hands a backend only the tensors it planned), or a       */
/* thread that must not call cudaMalloc because cudaMalloc may synchronize  */
/* the device and stall every other stream.  Those callers cannot provide   */
/* the workspace xq_flash_attn_ext needs for its split partials.  This      */
/* variant takes the same parameters and instead uses a fixed scratch array */
/* compiled into the library: XQ_NOALLOC_SCRATCH_BYTES of device memory    */
/* that every GPU which loads the library holds until the process exits.    */
/*                                                                           */
/*  - It runs the split-KV decode kernels (never the tensor-core prefill     */
/*    kernel).  For every shape that xq_flash_attn_ext also sends to those  */
/*    kernels (decode and short multi-query calls) the results are bit for  */
/*    bit the same; F16 calls with 64 or more queries, which               */
/*    xq_flash_attn_ext sends to the prefill kernel, agree within the       */
/*    attention tolerance instead.                                          */
/*  - q and dst may be device memory or pinned host memory, as for          */
/*    xq_flash_attn_ext: a pinned q is copied into the scratch by a kernel  */
/*    and a pinned dst is written in place; pageable host memory returns    */
/*    XQ_ERR_INVALID before anything is launched.                           */
/*  - The first call on a device looks up the scratch address for that     */
/*    device (cudaGetSymbolAddress); make that first call before any stream */
/*    capture.  The address is kept for the life of the process: do not     */
/*    call this entry point again after cudaDeviceReset on that device.     */
/*  - A call whose split plan (plus the staged q) needs more scratch than   */
/*    the maximum returns XQ_ERR_WORKSPACE with the sizes in               */
/*    xq_last_error(); pass a smaller n_splits.                             */
/*  - All calls share the one array and it keeps the last call's contents;  */
/*    nothing in it has to start at zero (every partial record is written   */
/*    before it is read).  Calls that overlap on the GPU (other streams,    */
/*    other threads) race on the scratch: serialize them.                   */
/*  - It allocates nothing: no cudaMalloc, cudaFree or allocating library   */
/*    routine.                                                               */
/* ------------------------------------------------------------------------ */
#define XQ_NOALLOC_SCRATCH_BYTES (8u << 20)
int xq_flash_attn_ext_noalloc(const xq_fa_params *p, xq_stream_t stream);

/* Library identity and the last error message of this thread. */
const char *xq_version(void);
const char *xq_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* XQ_B200_H */
