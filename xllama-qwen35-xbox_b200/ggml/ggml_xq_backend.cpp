// The XQ_B200 ggml backend: ggml's plugin interface in front of the B200
// attention kernels (libxq_b200.so, include/xq_b200.h).
//
// Same plugin surface as the reference's D3D12 backend
// (src/bridge/ggml_d3d12.cpp): a registry (:2473-2478) with one device per
// GPU, a device (:2427-2446) whose supports_op claims FLASH_ATTN_EXT, SET_ROWS and
// GATED_DELTA_NET, a device buffer type (:1516-1527) and buffer (:1371-1383),
// and a backend (:2268-2285) whose graph_compute runs those three ops.  Unlike
// the reference (whose graph_compute is synchronous, synchronize = nullptr)
// work is queued on one CUDA stream per backend: set/get_tensor_async, the
// fork's 2-D strided copies, cpy_tensor_async between two of these backends,
// events and synchronize are implemented.  The registry's get_proc_address
// answers "ggml_backend_dev_get_extra_bufts" as the reference's does (:2462-
// 2471); the extra buffer type here is pinned host memory, which is also the
// device's host buffer type.  Nothing falls back to the CPU: an op the
// kernels cannot take is refused in supports_op, and a failing launch
// returns GGML_STATUS_FAILED.
//
// Build outside the fork: this file + ggml_abi_mirror.h (self-tests).  Inside
// the fork: -DXQ_GGML_REAL with the fork's ggml headers.
#ifdef XQ_GGML_REAL
#include "ggml-backend-impl.h"
#include "ggml-backend.h"
#include "ggml.h"
#else
#include "ggml_abi_mirror.h"
#endif

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "xq_b200.h"
#include "xq_ggml_backend.h"

namespace {

void log_err(const char *what, const char *detail) {
    std::fprintf(stderr, "[xq_b200] %s: %s\n", what, detail);
}

bool ok_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess)
        return true;
    log_err(what, cudaGetErrorString(e));
    return false;
}

// ---------------------------------------------------------------------------
// contract (pure host logic)

bool is_view_op(int op) {
    return op == GGML_OP_NONE || op == GGML_OP_RESHAPE || op == GGML_OP_VIEW ||
           op == GGML_OP_PERMUTE || op == GGML_OP_TRANSPOSE;
}

bool kv_type(int t) { return t == GGML_TYPE_F16 || t == GGML_TYPE_Q8_0 || t == GGML_TYPE_Q4_0; }

bool rows_aligned4(const ggml_tensor *t) {
    for (int i = 1; i < 4; ++i)
        if (t->nb[i] % 4)
            return false;
    return true;
}

bool dst_contiguous_f32(const ggml_tensor *t) {
    return t->type == GGML_TYPE_F32 && t->nb[0] == 4 && t->nb[1] == 4 * (size_t)t->ne[0] &&
           t->nb[2] == t->nb[1] * (size_t)t->ne[1] && t->nb[3] == t->nb[2] * (size_t)t->ne[2];
}

// FLASH_ATTN_EXT: src q (F32), k, v (equal F16/Q8_0/Q4_0), mask (F16, opt),
// sinks (F32, opt); op_params scale, max_bias, softcap; dst F32 [D, H, n_q, S].
bool fa_supported(const ggml_tensor *op) {
    const ggml_tensor *q = op->src[0], *k = op->src[1], *v = op->src[2];
    const ggml_tensor *m = op->src[3], *sk = op->src[4];
    if (!q || !k || !v || q->type != GGML_TYPE_F32 || q->nb[0] != 4 || !kv_type(k->type) ||
        k->type != v->type)
        return false;
    const int64_t D = q->ne[0];
    if ((D != 64 && D != 128 && D != 256) || k->ne[0] != D || v->ne[0] != D)
        return false;
    if (v->ne[1] != k->ne[1] || v->ne[2] != k->ne[2] || k->ne[2] <= 0 ||
        q->ne[2] % k->ne[2] || k->ne[3] <= 0 || v->ne[3] <= 0 || q->ne[3] % k->ne[3] ||
        q->ne[3] % v->ne[3])
        return false;
    if (!rows_aligned4(k) || !rows_aligned4(v))
        return false;
    if (m && (m->type != GGML_TYPE_F16 || m->ne[0] < k->ne[1] || m->ne[1] < q->ne[1]))
        return false;
    if (sk && (sk->type != GGML_TYPE_F32 || sk->ne[0] < q->ne[2]))
        return false;
    if (op->ne[0] != D || op->ne[1] != q->ne[2] || op->ne[2] != q->ne[1] ||
        op->ne[3] != q->ne[3] || !dst_contiguous_f32(op))
        return false;
    return k->ne[1] <= INT32_MAX && q->ne[1] * q->ne[2] <= INT32_MAX;
}

// GATED_DELTA_NET: q, k [128, H_k, T, S_qk]; v [128, H, T, S]; g, beta
// [1, H, T, S] (scalar, activated: op_params[1] == 0); state [128, 128, H, S];
// op_params[0] = K snapshot slots; dst [128 H, T S + K 128 S] contiguous.
bool gdn_supported(const ggml_tensor *op) {
    for (int i = 0; i < 6; ++i) {
        const ggml_tensor *t = op->src[i];
        if (!t || t->type != GGML_TYPE_F32 || (t->ne[0] != 1 && t->nb[0] != 4))
            return false;
    }
    if (op->src[6] || op->src[7] || op->src[8] || op->op_params[1] != 0)
        return false;
    const ggml_tensor *q = op->src[0], *k = op->src[1], *v = op->src[2], *g = op->src[3],
                      *b = op->src[4], *s = op->src[5];
    const int64_t S = v->ne[0], H = v->ne[1], T = v->ne[2], NS = v->ne[3];
    const int slots = op->op_params[0];
    if (S != 128 || q->ne[0] != S || k->ne[0] != S || q->ne[1] != k->ne[1] || q->ne[1] <= 0 ||
        H % q->ne[1] || q->ne[2] != T || k->ne[2] != T || NS % q->ne[3] || NS % k->ne[3])
        return false;
    for (const ggml_tensor *t : {g, b})
        if (t->ne[0] != 1 || t->ne[1] != H || t->ne[2] != T || t->ne[3] != NS)
            return false;
    if (s->ne[0] != S || s->ne[1] != S || s->ne[2] != H || s->ne[3] != NS)
        return false;
    if (slots < 1 || slots > 64)
        return false;
    return op->type == GGML_TYPE_F32 && op->ne[0] == S * H &&
           op->ne[1] == T * NS + (int64_t)slots * S * NS && op->ne[2] == 1 && op->ne[3] == 1 &&
           op->nb[0] == 4 && op->nb[1] == 4 * (size_t)op->ne[0];
}

// SET_ROWS (the KV-cache write): node = view of the cache (F32/F16/Q8_0/Q4_0,
// [ne0, rows, ne2, ne3]); src0 F32 rows [ne0, ne1, ne2, ne3]; src1 I32/I64
// indices [ne1, i1, i2] with ne2 % i1 == ne3 % i2 == 0 (ggml_set_rows' rules).
bool set_rows_supported(const ggml_tensor *op) {
    const ggml_tensor *b = op->src[0], *c = op->src[1];
    if (!b || !c || b->type != GGML_TYPE_F32 || b->nb[0] != 4)
        return false;
    if (c->type != GGML_TYPE_I32 && c->type != GGML_TYPE_I64)
        return false;
    const int t = op->type;
    if (t != GGML_TYPE_F32 && t != GGML_TYPE_F16 && t != GGML_TYPE_Q8_0 && t != GGML_TYPE_Q4_0)
        return false;
    if (op->ne[0] != b->ne[0] || op->ne[2] != b->ne[2] || op->ne[3] != b->ne[3] ||
        c->ne[0] != b->ne[1] || c->ne[1] <= 0 || c->ne[2] <= 0 || b->ne[2] % c->ne[1] ||
        b->ne[3] % c->ne[2] || c->ne[3] != 1)
        return false;
    return (t != GGML_TYPE_Q8_0 && t != GGML_TYPE_Q4_0) || op->ne[0] % 32 == 0;
}

xq_tensor xt(const ggml_tensor *t) {
    xq_tensor x;
    x.type = (int32_t)t->type;
    x.reserved = 0;
    x.data = t->data;
    for (int i = 0; i < 4; ++i) {
        x.ne[i] = t->ne[i];
        x.nb[i] = t->nb[i];
    }
    return x;
}

// ---------------------------------------------------------------------------
// buffers (device memory of one GPU)

struct BufCtx {
    void *base;
    int device;
};

struct DevCtx {
    int device;
    std::string name, description;
    ggml_backend_buffer_type buft;
};

void buf_free(ggml_backend_buffer_t b) {
    auto *c = static_cast<BufCtx *>(b->context);
    cudaSetDevice(c->device);
    cudaFree(c->base);
    delete c;
}
void *buf_base(ggml_backend_buffer_t b) { return static_cast<BufCtx *>(b->context)->base; }
ggml_status buf_init_tensor(ggml_backend_buffer_t, ggml_tensor *) { return GGML_STATUS_SUCCESS; }
void buf_memset(ggml_backend_buffer_t b, ggml_tensor *t, uint8_t value, size_t off, size_t size) {
    cudaSetDevice(static_cast<BufCtx *>(b->context)->device);
    ok_cuda(cudaMemset(static_cast<char *>(t->data) + off, value, size), "memset_tensor");
}
void buf_set(ggml_backend_buffer_t b, ggml_tensor *t, const void *data, size_t off, size_t size) {
    cudaSetDevice(static_cast<BufCtx *>(b->context)->device);
    ok_cuda(cudaMemcpy(static_cast<char *>(t->data) + off, data, size, cudaMemcpyHostToDevice),
            "set_tensor");
}
void buf_get(ggml_backend_buffer_t b, const ggml_tensor *t, void *data, size_t off, size_t size) {
    cudaSetDevice(static_cast<BufCtx *>(b->context)->device);
    ok_cuda(cudaMemcpy(data, static_cast<const char *>(t->data) + off, size,
                       cudaMemcpyDeviceToHost),
            "get_tensor");
}
// n_copies rows of `size` bytes between a tensor (row i at byte offset
// offset + i * stride_tensor) and host memory (row i at data + i *
// stride_data), the fork's ggml_backend_tensor_{set,get}_2d contract
// (ggml/src/ggml-backend.cpp:367-409 of the fork).  One strided copy when
// both strides are pitches cudaMemcpy2D takes, else one copy per row in row
// order, so that where rows overlap the later one wins as in ggml's loop.
bool copy_rows(int device, void *dst, size_t dpitch, const void *src, size_t spitch,
               size_t size, size_t n, cudaMemcpyKind kind, cudaStream_t st, bool async,
               const char *what) {
    if (size == 0 || n == 0)
        return true;
    int max_pitch = 0;
    if (cudaDeviceGetAttribute(&max_pitch, cudaDevAttrMaxPitch, device) != cudaSuccess)
        max_pitch = 0;
    if (dpitch >= size && spitch >= size && dpitch <= (size_t)max_pitch &&
        spitch <= (size_t)max_pitch) {
        return ok_cuda(async ? cudaMemcpy2DAsync(dst, dpitch, src, spitch, size, n, kind, st)
                             : cudaMemcpy2D(dst, dpitch, src, spitch, size, n, kind),
                       what);
    }
    for (size_t i = 0; i < n; ++i) {
        char *d = static_cast<char *>(dst) + i * dpitch;
        const char *s = static_cast<const char *>(src) + i * spitch;
        if (!ok_cuda(async ? cudaMemcpyAsync(d, s, size, kind, st) : cudaMemcpy(d, s, size, kind),
                     what))
            return false;
    }
    return true;
}
void buf_set_2d(ggml_backend_buffer_t b, ggml_tensor *t, const void *data, size_t off,
                size_t size, size_t n, size_t stride_tensor, size_t stride_data) {
    const int dev = static_cast<BufCtx *>(b->context)->device;
    cudaSetDevice(dev);
    copy_rows(dev, static_cast<char *>(t->data) + off, stride_tensor, data, stride_data, size, n,
              cudaMemcpyHostToDevice, nullptr, false, "set_tensor_2d");
}
void buf_get_2d(ggml_backend_buffer_t b, const ggml_tensor *t, void *data, size_t off,
                size_t size, size_t n, size_t stride_tensor, size_t stride_data) {
    const int dev = static_cast<BufCtx *>(b->context)->device;
    cudaSetDevice(dev);
    copy_rows(dev, data, stride_data, static_cast<const char *>(t->data) + off, stride_tensor,
              size, n, cudaMemcpyDeviceToHost, nullptr, false, "get_tensor_2d");
}
bool buf_cpy(ggml_backend_buffer_t b, const ggml_tensor *src, ggml_tensor *dst);
void buf_clear(ggml_backend_buffer_t b, uint8_t value) {
    cudaSetDevice(static_cast<BufCtx *>(b->context)->device);
    ok_cuda(cudaMemset(buf_base(b), value, b->size), "clear");
}

ggml_backend_buffer_i make_buf_iface() {
    ggml_backend_buffer_i i;
    std::memset(&i, 0, sizeof(i));
    i.free_buffer = buf_free;
    i.get_base = buf_base;
    i.init_tensor = buf_init_tensor;
    i.memset_tensor = buf_memset;
    i.set_tensor = buf_set;
    i.get_tensor = buf_get;
    i.set_tensor_2d = buf_set_2d;
    i.get_tensor_2d = buf_get_2d;
    i.cpy_tensor = buf_cpy;
    i.clear = buf_clear;
    return i;
}

const char *buft_name(ggml_backend_buffer_type_t) { return "XQ_B200"; }
ggml_backend_buffer_t buft_alloc(ggml_backend_buffer_type_t buft, size_t size) {
    auto *dc = static_cast<DevCtx *>(buft->context);
    if (size == 0)
        size = 256;
    void *p = nullptr;
    if (!ok_cuda(cudaSetDevice(dc->device), "alloc_buffer") ||
        !ok_cuda(cudaMalloc(&p, size), "alloc_buffer"))
        return nullptr;
    auto *c = new BufCtx{p, dc->device};
    return ggml_backend_buffer_init(buft, make_buf_iface(), c, size);
}
size_t buft_align(ggml_backend_buffer_type_t) { return 256; }

bool is_ours(ggml_backend_buffer_type_t buft) {
    return buft && buft->iface.get_name == buft_name;
}

bool buf_cpy(ggml_backend_buffer_t b, const ggml_tensor *src, ggml_tensor *dst) {
    if (!src->buffer || !is_ours(src->buffer->buft))
        return false;
    cudaSetDevice(static_cast<BufCtx *>(b->context)->device);
    return ok_cuda(cudaMemcpy(dst->data, src->data, ggml_nbytes(src), cudaMemcpyDeviceToDevice),
                   "cpy_tensor");
}

// ---------------------------------------------------------------------------
// pinned host buffers: the device's host buffer type (staging for the
// async copies) and its one extra buffer type

struct HostBufCtx {
    void *base;
};

bool buft_is_host(ggml_backend_buffer_type_t buft) {
    return buft && buft->iface.is_host && buft->iface.is_host(buft);
}

void hbuf_free(ggml_backend_buffer_t b) {
    auto *c = static_cast<HostBufCtx *>(b->context);
    cudaFreeHost(c->base);
    delete c;
}
void *hbuf_base(ggml_backend_buffer_t b) { return static_cast<HostBufCtx *>(b->context)->base; }
void hbuf_memset(ggml_backend_buffer_t, ggml_tensor *t, uint8_t value, size_t off, size_t size) {
    std::memset(static_cast<char *>(t->data) + off, value, size);
}
void hbuf_set(ggml_backend_buffer_t, ggml_tensor *t, const void *data, size_t off, size_t size) {
    std::memcpy(static_cast<char *>(t->data) + off, data, size);
}
void hbuf_get(ggml_backend_buffer_t, const ggml_tensor *t, void *data, size_t off, size_t size) {
    std::memcpy(data, static_cast<const char *>(t->data) + off, size);
}
bool hbuf_cpy(ggml_backend_buffer_t, const ggml_tensor *src, ggml_tensor *dst) {
    if (!src->buffer || !buft_is_host(src->buffer->buft))
        return false;
    std::memcpy(dst->data, src->data, ggml_nbytes(src));
    return true;
}
void hbuf_clear(ggml_backend_buffer_t b, uint8_t value) { std::memset(hbuf_base(b), value, b->size); }

ggml_backend_buffer_i make_host_buf_iface() {
    ggml_backend_buffer_i i;
    std::memset(&i, 0, sizeof(i));
    i.free_buffer = hbuf_free;
    i.get_base = hbuf_base;
    i.init_tensor = buf_init_tensor;
    i.memset_tensor = hbuf_memset;
    i.set_tensor = hbuf_set;
    i.get_tensor = hbuf_get;
    i.cpy_tensor = hbuf_cpy;
    i.clear = hbuf_clear;
    return i;
}

const char *hbuft_name(ggml_backend_buffer_type_t) { return "XQ_B200_Host"; }
ggml_backend_buffer_t hbuft_alloc(ggml_backend_buffer_type_t buft, size_t size) {
    if (size == 0)
        size = 64;
    void *p = nullptr;
    // portable: the pages are pinned for every device of the process
    if (!ok_cuda(cudaHostAlloc(&p, size, cudaHostAllocPortable), "host alloc_buffer"))
        return nullptr;
    return ggml_backend_buffer_init(buft, make_host_buf_iface(), new HostBufCtx{p}, size);
}
size_t hbuft_align(ggml_backend_buffer_type_t) { return 64; }
bool hbuft_is_host(ggml_backend_buffer_type_t) { return true; }

// ---------------------------------------------------------------------------
// backend (one CUDA stream)

// Per-op GPU time of a backend created with XQ_GGML_TIMING=1: CUDA events
// around every node on the backend's stream, read back at synchronize (the
// reference backend's timestamp accounting, ggml_d3d12.cpp:1897-1903,
// 2148-2151, 2202-2221).  Ops: 0 FLASH_ATTN_EXT, 1 GATED_DELTA_NET, 2 SET_ROWS.
constexpr int kTimedOps = 3;
const char *const kOpNames[kTimedOps] = {"FLASH_ATTN_EXT", "GATED_DELTA_NET", "SET_ROWS"};
struct OpTime {
    uint64_t nodes = 0, untimed = 0;
    double ms = 0.0;
};
struct PendingTime {
    int op;
    cudaEvent_t begin, end;
};

struct BackendCtx {
    int device = 0;
    cudaStream_t stream = nullptr;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    std::string name;
    cudaEvent_t order = nullptr; // orders this stream against another backend's (cpy_tensor_async)
    bool timing = false;
    OpTime times[kTimedOps];
    std::vector<PendingTime> pending; // timed nodes not read back yet
    std::vector<cudaEvent_t> pool;    // timing events for reuse
};

cudaEvent_t take_event(BackendCtx *c) {
    if (!c->pool.empty()) {
        cudaEvent_t e = c->pool.back();
        c->pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    return cudaEventCreate(&e) == cudaSuccess ? e : nullptr;
}

// Read back the timed nodes whose end event has completed, in order (all of
// them after a stream synchronize).
void drain_times(BackendCtx *c) {
    size_t done = 0;
    for (; done < c->pending.size(); ++done) {
        PendingTime &p = c->pending[done];
        const cudaError_t q = cudaEventQuery(p.end);
        if (q == cudaErrorNotReady)
            break;
        float ms = 0.0f;
        if (q == cudaSuccess && cudaEventElapsedTime(&ms, p.begin, p.end) == cudaSuccess) {
            c->times[p.op].nodes++;
            c->times[p.op].ms += ms;
        } else {
            cudaGetLastError();
            c->times[p.op].untimed++;
        }
        c->pool.push_back(p.begin);
        c->pool.push_back(p.end);
    }
    c->pending.erase(c->pending.begin(), c->pending.begin() + (std::ptrdiff_t)done);
}

const char *be_name(ggml_backend_t b) { return static_cast<BackendCtx *>(b->context)->name.c_str(); }
void be_free(ggml_backend_t b) {
    auto *c = static_cast<BackendCtx *>(b->context);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    drain_times(c);
    if (c->timing)
        for (int i = 0; i < kTimedOps; ++i)
            if (c->times[i].nodes || c->times[i].untimed)
                std::fprintf(stderr, "[xq_b200] %s %s: %llu nodes, %.3f ms GPU, %llu untimed\n",
                             c->name.c_str(), kOpNames[i], (unsigned long long)c->times[i].nodes,
                             c->times[i].ms, (unsigned long long)c->times[i].untimed);
    for (const PendingTime &p : c->pending) {
        cudaEventDestroy(p.begin);
        cudaEventDestroy(p.end);
    }
    for (cudaEvent_t e : c->pool)
        cudaEventDestroy(e);
    if (c->ws)
        cudaFree(c->ws);
    cudaEventDestroy(c->order);
    cudaStreamDestroy(c->stream);
    delete c;
    delete b;
}
void be_set_async(ggml_backend_t b, ggml_tensor *t, const void *data, size_t off, size_t size) {
    auto *c = static_cast<BackendCtx *>(b->context);
    ok_cuda(cudaMemcpyAsync(static_cast<char *>(t->data) + off, data, size,
                            cudaMemcpyHostToDevice, c->stream),
            "set_tensor_async");
}
void be_get_async(ggml_backend_t b, const ggml_tensor *t, void *data, size_t off, size_t size) {
    auto *c = static_cast<BackendCtx *>(b->context);
    ok_cuda(cudaMemcpyAsync(data, static_cast<const char *>(t->data) + off, size,
                            cudaMemcpyDeviceToHost, c->stream),
            "get_tensor_async");
}
void be_set_2d_async(ggml_backend_t b, ggml_tensor *t, const void *data, size_t off,
                     size_t size, size_t n, size_t stride_tensor, size_t stride_data) {
    auto *c = static_cast<BackendCtx *>(b->context);
    copy_rows(c->device, static_cast<char *>(t->data) + off, stride_tensor, data, stride_data,
              size, n, cudaMemcpyHostToDevice, c->stream, true, "set_tensor_2d_async");
}
void be_get_2d_async(ggml_backend_t b, const ggml_tensor *t, void *data, size_t off,
                     size_t size, size_t n, size_t stride_tensor, size_t stride_data) {
    auto *c = static_cast<BackendCtx *>(b->context);
    copy_rows(c->device, data, stride_data, static_cast<const char *>(t->data) + off,
              stride_tensor, size, n, cudaMemcpyDeviceToHost, c->stream, true,
              "get_tensor_2d_async");
}
void be_sync(ggml_backend_t b) {
    auto *c = static_cast<BackendCtx *>(b->context);
    ok_cuda(cudaStreamSynchronize(c->stream), "synchronize");
    drain_times(c);
}
bool is_our_backend(ggml_backend_t b);

// A copy between two tensors in this backend's device buffers, queued on the
// source backend's stream behind the work both streams already hold; the
// destination stream then waits for it.  Across GPUs it is a peer copy.
// Anything else (a host buffer, another backend) answers false and ggml
// falls back to its synchronous copy.
bool be_cpy_async(ggml_backend_t bs, ggml_backend_t bd, const ggml_tensor *src,
                  ggml_tensor *dst) {
    if (!is_our_backend(bs) || !is_our_backend(bd) || !src->buffer || !dst->buffer ||
        !is_ours(src->buffer->buft) || !is_ours(dst->buffer->buft))
        return false;
    auto *cs = static_cast<BackendCtx *>(bs->context);
    auto *cd = static_cast<BackendCtx *>(bd->context);
    const size_t n = ggml_nbytes(src);
    if (bs != bd) {
        cudaSetDevice(cd->device);
        if (!ok_cuda(cudaEventRecord(cd->order, cd->stream), "cpy_tensor_async"))
            return false;
        cudaSetDevice(cs->device);
        if (!ok_cuda(cudaStreamWaitEvent(cs->stream, cd->order, 0), "cpy_tensor_async"))
            return false;
    }
    cudaSetDevice(cs->device);
    const cudaError_t e =
        cs->device == cd->device
            ? cudaMemcpyAsync(dst->data, src->data, n, cudaMemcpyDeviceToDevice, cs->stream)
            : cudaMemcpyPeerAsync(dst->data, cd->device, src->data, cs->device, n, cs->stream);
    if (!ok_cuda(e, "cpy_tensor_async"))
        return false;
    if (bs != bd) {
        if (!ok_cuda(cudaEventRecord(cs->order, cs->stream), "cpy_tensor_async"))
            return false;
        cudaSetDevice(cd->device);
        if (!ok_cuda(cudaStreamWaitEvent(cd->stream, cs->order, 0), "cpy_tensor_async"))
            return false;
    }
    return true;
}

// events: a CUDA event of the device the ggml event was made for
cudaEvent_t cuda_event(ggml_backend_event_t ev) { return static_cast<cudaEvent_t>(ev->context); }
void be_event_record(ggml_backend_t b, ggml_backend_event_t ev) {
    auto *c = static_cast<BackendCtx *>(b->context);
    cudaSetDevice(c->device);
    ok_cuda(cudaEventRecord(cuda_event(ev), c->stream), "event_record");
}
void be_event_wait(ggml_backend_t b, ggml_backend_event_t ev) {
    auto *c = static_cast<BackendCtx *>(b->context);
    cudaSetDevice(c->device);
    ok_cuda(cudaStreamWaitEvent(c->stream, cuda_event(ev), 0), "event_wait");
}

bool ensure_ws(BackendCtx *c, size_t need) {
    if (need <= c->ws_bytes)
        return true;
    // the stream may still read the old workspace: wait before replacing it
    if (c->ws) {
        cudaStreamSynchronize(c->stream);
        cudaFree(c->ws);
        c->ws = nullptr;
        c->ws_bytes = 0;
    }
    if (!ok_cuda(cudaMalloc(&c->ws, need), "workspace"))
        return false;
    c->ws_bytes = need;
    return true;
}

ggml_status run_fa(BackendCtx *c, ggml_tensor *op) {
    xq_fa_params p;
    std::memset(&p, 0, sizeof(p));
    p.q = xt(op->src[0]);
    p.k = xt(op->src[1]);
    p.v = xt(op->src[2]);
    if (op->src[3])
        p.mask = xt(op->src[3]);
    p.sinks = op->src[4] ? static_cast<const float *>(op->src[4]->data) : nullptr;
    p.dst = static_cast<float *>(op->data);
    std::memcpy(&p.scale, &op->op_params[0], 4);
    std::memcpy(&p.max_bias, &op->op_params[1], 4);
    std::memcpy(&p.softcap, &op->op_params[2], 4);
    // one planned call with the backend's workspace as it is; a call that
    // needs more returns XQ_ERR_WORKSPACE before launching anything, and only
    // then is the size asked for and the workspace grown
    xq_stream_t st = reinterpret_cast<xq_stream_t>(c->stream);
    int rc = xq_flash_attn_ext(&p, c->ws, c->ws_bytes, st);
    if (rc == XQ_ERR_WORKSPACE) {
        if (!ensure_ws(c, xq_flash_attn_ext_workspace(&p)))
            return GGML_STATUS_ALLOC_FAILED;
        rc = xq_flash_attn_ext(&p, c->ws, c->ws_bytes, st);
    }
    if (rc) {
        log_err("FLASH_ATTN_EXT", xq_last_error());
        return GGML_STATUS_FAILED;
    }
    return GGML_STATUS_SUCCESS;
}

ggml_status run_gdn(BackendCtx *c, ggml_tensor *op) {
    xq_tensor t[6];
    for (int i = 0; i < 6; ++i)
        t[i] = xt(op->src[i]);
    // long prefill runs the chunked tensor-core form (workspace on the backend)
    const size_t need = xq_gated_delta_net_workspace(&t[2], op->op_params[0]);
    if (!ensure_ws(c, need))
        return GGML_STATUS_ALLOC_FAILED;
    if (xq_gated_delta_net_ws(&t[0], &t[1], &t[2], &t[3], &t[4], &t[5],
                              static_cast<float *>(op->data), op->op_params[0], c->ws,
                              c->ws_bytes, reinterpret_cast<xq_stream_t>(c->stream))) {
        log_err("GATED_DELTA_NET", xq_last_error());
        return GGML_STATUS_FAILED;
    }
    return GGML_STATUS_SUCCESS;
}

ggml_status run_set_rows(BackendCtx *c, ggml_tensor *op) {
    const xq_tensor src = xt(op->src[0]), idx = xt(op->src[1]), dst = xt(op);
    if (xq_set_rows(&src, &idx, &dst, reinterpret_cast<xq_stream_t>(c->stream))) {
        log_err("SET_ROWS", xq_last_error());
        return GGML_STATUS_FAILED;
    }
    return GGML_STATUS_SUCCESS;
}

ggml_status be_graph_compute(ggml_backend_t b, ggml_cgraph *g) {
    auto *c = static_cast<BackendCtx *>(b->context);
    if (!ok_cuda(cudaSetDevice(c->device), "graph_compute"))
        return GGML_STATUS_FAILED;
    const int n = ggml_graph_n_nodes(g);
    for (int i = 0; i < n; ++i) {
        ggml_tensor *node = ggml_graph_node(g, i);
        if (is_view_op(node->op) || !(node->flags & GGML_TENSOR_FLAG_COMPUTE))
            continue;
        const int oi = node->op == GGML_OP_FLASH_ATTN_EXT    ? 0
                       : node->op == GGML_OP_GATED_DELTA_NET ? 1
                       : node->op == GGML_OP_SET_ROWS        ? 2
                                                             : -1;
        // one NVTX range per node (free unless a profiler is attached)
        nvtxRangePushA(oi >= 0 ? kOpNames[oi] : "unclaimed");
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        if (c->timing && oi >= 0) {
            if (c->pending.size() >= 1024)
                drain_times(c); // completed nodes only: never blocks
            e0 = take_event(c);
            e1 = take_event(c);
            if (e0 && cudaEventRecord(e0, c->stream) != cudaSuccess) {
                cudaGetLastError();
                c->pool.push_back(e0);
                e0 = nullptr;
            }
        }
        ggml_status st;
        if (node->op == GGML_OP_FLASH_ATTN_EXT && fa_supported(node))
            st = run_fa(c, node);
        else if (node->op == GGML_OP_GATED_DELTA_NET && gdn_supported(node))
            st = run_gdn(c, node);
        else if (node->op == GGML_OP_SET_ROWS && set_rows_supported(node))
            st = run_set_rows(c, node);
        else {
            log_err("graph_compute", "node outside the supports_op contract");
            st = GGML_STATUS_FAILED;
        }
        if (c->timing && oi >= 0) {
            if (st == GGML_STATUS_SUCCESS && e0 && e1 &&
                cudaEventRecord(e1, c->stream) == cudaSuccess) {
                c->pending.push_back({oi, e0, e1});
            } else {
                cudaGetLastError();
                c->times[oi].untimed++;
                if (e0)
                    c->pool.push_back(e0);
                if (e1)
                    c->pool.push_back(e1);
            }
        }
        nvtxRangePop();
        if (st != GGML_STATUS_SUCCESS)
            return st;
    }
    return GGML_STATUS_SUCCESS;
}

ggml_guid_t backend_guid() {
    static ggml_guid guid = {0x78, 0x71, 0x2d, 0x62, 0x32, 0x30, 0x30, 0x2d,
                             0x61, 0x74, 0x74, 0x6e, 0x2d, 0x76, 0x30, 0x31};
    return &guid;
}

ggml_backend_i make_backend_iface() {
    ggml_backend_i i;
    std::memset(&i, 0, sizeof(i));
    i.get_name = be_name;
    i.free = be_free;
    i.set_tensor_async = be_set_async;
    i.get_tensor_async = be_get_async;
    i.set_tensor_2d_async = be_set_2d_async;
    i.get_tensor_2d_async = be_get_2d_async;
    i.cpy_tensor_async = be_cpy_async;
    i.synchronize = be_sync;
    i.graph_compute = be_graph_compute;
    i.event_record = be_event_record;
    i.event_wait = be_event_wait;
    return i;
}

bool is_our_backend(ggml_backend_t b) { return b && b->iface.get_name == be_name; }

// ---------------------------------------------------------------------------
// device + registry

const char *dev_name(ggml_backend_dev_t d) {
    return static_cast<DevCtx *>(d->context)->name.c_str();
}
const char *dev_desc(ggml_backend_dev_t d) {
    return static_cast<DevCtx *>(d->context)->description.c_str();
}
void dev_memory(ggml_backend_dev_t d, size_t *free_b, size_t *total_b) {
    *free_b = *total_b = 0;
    if (cudaSetDevice(static_cast<DevCtx *>(d->context)->device) == cudaSuccess)
        cudaMemGetInfo(free_b, total_b);
}
ggml_backend_dev_type dev_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_GPU; }
void dev_props(ggml_backend_dev_t d, ggml_backend_dev_props *p) {
    p->name = dev_name(d);
    p->description = dev_desc(d);
    dev_memory(d, &p->memory_free, &p->memory_total);
    p->type = GGML_BACKEND_DEVICE_TYPE_GPU;
    p->device_id = nullptr;
    p->caps.async = true;
    p->caps.host_buffer = true;
    p->caps.buffer_from_host_ptr = false;
    p->caps.events = true;
}
ggml_backend_t dev_init(ggml_backend_dev_t d, const char *) {
    auto *dc = static_cast<DevCtx *>(d->context);
    if (!ok_cuda(cudaSetDevice(dc->device), "init_backend"))
        return nullptr;
    auto *c = new BackendCtx;
    c->device = dc->device;
    c->name = dc->name;
    const char *tm = std::getenv("XQ_GGML_TIMING");
    c->timing = tm && tm[0] && tm[0] != '0';
    if (!ok_cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "init_backend")) {
        delete c;
        return nullptr;
    }
    if (!ok_cuda(cudaEventCreateWithFlags(&c->order, cudaEventDisableTiming), "init_backend")) {
        cudaStreamDestroy(c->stream);
        delete c;
        return nullptr;
    }
    return new ggml_backend{backend_guid(), make_backend_iface(), d, c};
}
ggml_backend_buffer_type_t dev_buft(ggml_backend_dev_t d) {
    return &static_cast<DevCtx *>(d->context)->buft;
}
bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor *op) {
    return ggml_xq_b200_supports_op(op);
}
bool dev_supports_buft(ggml_backend_dev_t d, ggml_backend_buffer_type_t buft) {
    return buft == dev_buft(d);
}
ggml_backend_event_t dev_event_new(ggml_backend_dev_t d) {
    cudaEvent_t e = nullptr;
    if (!ok_cuda(cudaSetDevice(static_cast<DevCtx *>(d->context)->device), "event_new") ||
        !ok_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event_new"))
        return nullptr;
    return new ggml_backend_event{d, e};
}
void dev_event_free(ggml_backend_dev_t, ggml_backend_event_t ev) {
    if (!ev)
        return;
    cudaSetDevice(static_cast<DevCtx *>(ev->device->context)->device);
    cudaEventDestroy(cuda_event(ev));
    delete ev;
}
void dev_event_sync(ggml_backend_dev_t, ggml_backend_event_t ev) {
    ok_cuda(cudaEventSynchronize(cuda_event(ev)), "event_synchronize");
}

struct Registry {
    std::vector<DevCtx *> ctx;
    std::vector<ggml_backend_device> devices;
    ggml_backend_reg reg;
    ggml_backend_buffer_type host_buft; // pinned, shared by every device
};

const char *reg_name(ggml_backend_reg_t) { return "XQ_B200"; }
Registry &registry();
size_t reg_count(ggml_backend_reg_t) { return registry().devices.size(); }
ggml_backend_dev_t reg_device(ggml_backend_reg_t, size_t i) {
    Registry &r = registry();
    return i < r.devices.size() ? &r.devices[i] : nullptr;
}
ggml_backend_buffer_type_t dev_host_buft(ggml_backend_dev_t) { return &registry().host_buft; }
// ggml_backend_dev_get_extra_bufts_t: a null-terminated list of the buffer
// types this device offers besides its own (the reference's answer lists its
// weights buffer type; here it is the pinned host type)
ggml_backend_buffer_type_t *dev_extra_bufts(ggml_backend_dev_t) {
    static ggml_backend_buffer_type_t list[2] = {&registry().host_buft, nullptr};
    return list;
}
void *reg_proc(ggml_backend_reg_t, const char *name) {
    if (name && std::strcmp(name, "ggml_backend_dev_get_extra_bufts") == 0)
        return reinterpret_cast<void *>(dev_extra_bufts);
    return nullptr;
}

Registry &registry() {
    static Registry r;
    static std::once_flag once;
    std::call_once(once, [] {
        r.reg.api_version = GGML_BACKEND_API_VERSION;
        r.reg.iface = {reg_name, reg_count, reg_device, reg_proc};
        r.reg.context = nullptr;
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess)
            n = 0;
        r.ctx.resize(n);
        r.devices.resize(n);
        r.host_buft.iface = {hbuft_name, hbuft_alloc, hbuft_align, nullptr, nullptr,
                             hbuft_is_host};
        r.host_buft.device = n > 0 ? &r.devices[0] : nullptr;
        r.host_buft.context = nullptr;
        for (int i = 0; i < n; ++i) {
            cudaDeviceProp prop;
            std::memset(&prop, 0, sizeof(prop));
            cudaGetDeviceProperties(&prop, i);
            auto *dc = new DevCtx;
            dc->device = i;
            dc->name = "XQ_B200" + std::to_string(i);
            dc->description = std::string(prop.name) + " (FLASH_ATTN_EXT, GATED_DELTA_NET)";
            dc->buft.iface = {buft_name, buft_alloc, buft_align, nullptr, nullptr, nullptr};
            dc->buft.device = &r.devices[i];
            dc->buft.context = dc;
            r.ctx[i] = dc;
            ggml_backend_device_i di;
            std::memset(&di, 0, sizeof(di));
            di.get_name = dev_name;
            di.get_description = dev_desc;
            di.get_memory = dev_memory;
            di.get_type = dev_type;
            di.get_props = dev_props;
            di.init_backend = dev_init;
            di.get_buffer_type = dev_buft;
            di.get_host_buffer_type = dev_host_buft;
            di.supports_op = dev_supports_op;
            di.supports_buft = dev_supports_buft;
            di.event_new = dev_event_new;
            di.event_free = dev_event_free;
            di.event_synchronize = dev_event_sync;
            r.devices[i].iface = di;
            r.devices[i].reg = &r.reg;
            r.devices[i].context = dc;
        }
    });
    return r;
}

} // namespace

extern "C" {

bool ggml_xq_b200_supports_op(const ggml_tensor *op) {
    if (!op)
        return false;
    if (is_view_op(op->op))
        return true;
    if (op->op == GGML_OP_FLASH_ATTN_EXT)
        return fa_supported(op);
    if (op->op == GGML_OP_GATED_DELTA_NET)
        return gdn_supported(op);
    if (op->op == GGML_OP_SET_ROWS)
        return set_rows_supported(op);
    return false;
}

ggml_backend_reg_t ggml_backend_xq_b200_reg(void) { return &registry().reg; }

bool ggml_xq_b200_backend_op_time(ggml_backend_t backend, int op, uint64_t *nodes, double *ms,
                                  uint64_t *untimed) {
    if (!is_our_backend(backend) || op < 0 || op >= kTimedOps)
        return false;
    auto *c = static_cast<BackendCtx *>(backend->context);
    if (!c->timing)
        return false;
    drain_times(c);
    if (nodes)
        *nodes = c->times[op].nodes;
    if (ms)
        *ms = c->times[op].ms;
    if (untimed)
        *untimed = c->times[op].untimed;
    return true;
}

bool ggml_xq_b200_register(void) {
    static std::once_flag once;
    static bool done = false;
    std::call_once(once, [] {
        Registry &r = registry();
        if (r.devices.empty()) {
            log_err("register", "no CUDA device visible; backend not registered");
            return;
        }
        ggml_backend_register(&r.reg);
        done = true;
    });
    return done;
}

} // extern "C"
