// extern "C" entry points of libxq_b200.so (declared in include/xq_b200.h):
// argument contracts, launch planning and error reporting.  No allocation
// happens here: scratch comes from the caller's workspace.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>

#include "xq_common.cuh"
#include "xq_internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess)
        return XQ_OK;
    return fail(XQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// SM count of the current device, queried once per device.
int sm_count() {
    static std::atomic<int> cache[64];
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return 148;
    if (dev >= 0 && dev < 64 && (n = cache[dev].load(std::memory_order_relaxed)) > 0)
        return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return 148;
    if (dev >= 0 && dev < 64)
        cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

bool kv_type_ok(int t) { return t == XQ_TYPE_F16 || t == XQ_TYPE_Q8_0 || t == XQ_TYPE_Q4_0; }

struct FaPlan {
    xq::DecodeArgs a;
    xq::DecodeConfig cfg;
    int D, n_qblocks;
    bool mma; // warp-MMA decode kernel (8 q-rows per CTA)
    int64_t n_rows, n_splits;
};

bool mma_disabled() {
    static const int off = [] {
        const char *e = getenv("XQ_DECODE_MMA");
        return e && e[0] == '0';
    }();
    return off != 0;
}

cudaError_t run_decode(const FaPlan &pl, dim3 grid, cudaStream_t st) {
    if (pl.mma)
        return xq::launch_decode_mma(pl.a, pl.cfg.type, pl.D, pl.cfg.VW, grid, st);
    return xq::launch_decode(pl.a, pl.cfg, grid, st);
}

// Validate a FLASH_ATTN_EXT call and fill the decode arguments (without
// choosing splits).
int fa_prepare(const xq_fa_params *p, FaPlan *pl) {
    if (!p)
        return fail(XQ_ERR_INVALID, "flash_attn_ext: null params");
    const xq_tensor &q = p->q, &k = p->k, &v = p->v, &m = p->mask;
    if (q.type != XQ_TYPE_F32 || q.nb[0] != 4)
        return fail(XQ_ERR_UNSUPPORTED, "flash_attn_ext: q must be F32 with contiguous rows");
    if (!kv_type_ok(k.type) || k.type != v.type)
        return fail(XQ_ERR_UNSUPPORTED,
                    "flash_attn_ext: K/V types %d/%d (supported: equal F16, Q8_0 or Q4_0)",
                    k.type, v.type);
    const int64_t D = q.ne[0];
    if (k.ne[0] != D || v.ne[0] != D || (D != 64 && D != 128 && D != 256))
        return fail(XQ_ERR_UNSUPPORTED, "flash_attn_ext: head dim %lld/%lld/%lld",
                    (long long)D, (long long)k.ne[0], (long long)v.ne[0]);
    const int64_t n_q = q.ne[1], n_head = q.ne[2], n_seq = q.ne[3];
    const int64_t n_kv = k.ne[1], n_hkv = k.ne[2];
    if (v.ne[1] != n_kv || v.ne[2] != n_hkv || n_hkv <= 0 || n_head % n_hkv ||
        k.ne[3] <= 0 || v.ne[3] <= 0 || n_seq % k.ne[3] || n_seq % v.ne[3] || n_q <= 0)
        return fail(XQ_ERR_INVALID, "flash_attn_ext: inconsistent q/k/v shapes");
    if (n_kv > INT32_MAX || n_q * n_head > INT32_MAX)
        return fail(XQ_ERR_UNSUPPORTED, "flash_attn_ext: sizes beyond int32");
    if (!q.data || !k.data || !v.data || !p->dst)
        return fail(XQ_ERR_INVALID, "flash_attn_ext: null tensor data");
    if (m.data) {
        if (m.type != XQ_TYPE_F16 || m.nb[0] != 2 || m.ne[0] < n_kv || m.ne[1] < n_q ||
            m.ne[2] <= 0 || m.ne[3] <= 0)
            return fail(XQ_ERR_INVALID, "flash_attn_ext: mask must be F16 [n_kv, >=n_q, ...]");
    }
    xq::DecodeArgs &a = pl->a;
    memset(&a, 0, sizeof(a));
    a.q = static_cast<const uint8_t *>(q.data);
    a.q_nb1 = (int64_t)q.nb[1];
    a.q_nb2 = (int64_t)q.nb[2];
    a.q_nb3 = (int64_t)q.nb[3];
    a.k = static_cast<const uint8_t *>(k.data);
    a.k_nb1 = (int64_t)k.nb[1];
    a.k_nb2 = (int64_t)k.nb[2];
    a.k_nb3 = (int64_t)k.nb[3];
    a.v = static_cast<const uint8_t *>(v.data);
    a.v_nb1 = (int64_t)v.nb[1];
    a.v_nb2 = (int64_t)v.nb[2];
    a.v_nb3 = (int64_t)v.nb[3];
    if (m.data) {
        a.mask = static_cast<const uint8_t *>(m.data);
        a.m_nb1 = (int64_t)m.nb[1];
        a.m_nb2 = (int64_t)m.nb[2];
        a.m_nb3 = (int64_t)m.nb[3];
        a.m_ne2 = (int)m.ne[2];
        a.m_ne3 = (int)m.ne[3];
    } else {
        a.m_ne2 = a.m_ne3 = 1;
    }
    a.dst = p->dst;
    a.sinks = p->sinks;
    a.n_q = (int)n_q;
    a.n_head = (int)n_head;
    a.n_head_kv = (int)n_hkv;
    a.n_seq = (int)n_seq;
    a.n_kv = (int)n_kv;
    a.G = (int)(n_head / n_hkv);
    a.rk3 = (int)(n_seq / k.ne[3]);
    a.rv3 = (int)(n_seq / v.ne[3]);
    a.n_qrows = (int)(n_q * a.G);
    a.q_convert = 1;
    a.softcap = p->softcap;
    a.scale = p->softcap != 0.0f ? p->scale / p->softcap : p->scale;
    a.alibi = p->max_bias > 0.0f;
    const uint32_t nh_log2 = 1u << (uint32_t)floor(log2((double)n_head));
    a.n_head_log2 = (int)nh_log2;
    a.m0 = powf(2.0f, -(p->max_bias) / (float)nh_log2);
    a.m1 = powf(2.0f, -(p->max_bias / 2.0f) / (float)nh_log2);
    if (!xq::decode_config(k.type, (int)D, a.n_qrows, a, &pl->cfg))
        return fail(XQ_ERR_UNSUPPORTED, "flash_attn_ext: K/V rows not 4-byte aligned");
    pl->D = (int)D;
    pl->mma = !mma_disabled() && xq::decode_mma_ok(k.type, (int)D, a);
    const int per_block = pl->mma ? xq::decode_mma_rows_per_cta(a.n_qrows) : pl->cfg.NR;
    pl->n_qblocks = (a.n_qrows + per_block - 1) / per_block;
    pl->n_rows = n_seq * n_q * n_head;
    return XQ_OK;
}

bool prefill_disabled() {
    static const int off = [] {
        const char *e = getenv("XQ_PREFILL");
        return e && e[0] == '0';
    }();
    return off != 0;
}

// The tensor-core prefill kernel takes F16 K/V -- or Q8_0 / Q4_0 K/V, which a
// pre-pass widens to f16 in the workspace -- D 128/256, many queries and no
// softcap / ALiBi / sinks, with TMA-compatible (16-byte) strides for what it
// reads through tensor maps (q always, K/V when F16).
bool prefill_shape(const xq_fa_params *p, const FaPlan &pl, xq::PrefillShape *ps) {
    const xq_tensor &q = p->q, &k = p->k, &v = p->v, &m = p->mask;
    const bool quant = k.type == XQ_TYPE_Q8_0 || k.type == XQ_TYPE_Q4_0;
    if (prefill_disabled() || !(k.type == XQ_TYPE_F16 || quant) || v.type != k.type ||
        (pl.D != 128 && pl.D != 256) || q.ne[1] < 64 || p->softcap != 0.0f ||
        p->max_bias > 0.0f || p->sinks)
        return false;
    auto a16 = [](uint64_t x) { return x % 16 == 0; };
    auto a2 = [](uint64_t x) { return x % 2 == 0; };
    const auto kv_ok = quant ? +a2 : +a16; // quantized rows are read by the pre-pass
    if (!kv_ok((uint64_t)(uintptr_t)k.data) || !kv_ok((uint64_t)(uintptr_t)v.data) ||
        !a16((uint64_t)(uintptr_t)q.data) || !kv_ok(k.nb[1]) || !kv_ok(k.nb[2]) ||
        !kv_ok(k.nb[3]) || !kv_ok(v.nb[1]) || !kv_ok(v.nb[2]) || !kv_ok(v.nb[3]) ||
        !a16(q.nb[1]) || !a16(q.nb[2]) || !a16(q.nb[3]) || k.ne[3] != v.ne[3])
        return false;
    ps->kv_type = k.type;
    ps->q = static_cast<const uint8_t *>(q.data);
    for (int i = 0; i < 4; ++i) {
        ps->q_nb[i] = (int64_t)q.nb[i];
        ps->k_nb[i] = (int64_t)k.nb[i];
        ps->v_nb[i] = (int64_t)v.nb[i];
    }
    ps->k = k.data;
    ps->v = v.data;
    ps->mask = static_cast<const uint8_t *>(m.data);
    ps->m_nb1 = (int64_t)m.nb[1];
    ps->m_nb2 = (int64_t)m.nb[2];
    ps->m_nb3 = (int64_t)m.nb[3];
    ps->m_ne2 = m.data ? (int)m.ne[2] : 1;
    ps->m_ne3 = m.data ? (int)m.ne[3] : 1;
    ps->m_planes = ps->m_ne2 * ps->m_ne3;
    ps->dst = p->dst;
    ps->D = pl.D;
    ps->n_q = (int)q.ne[1];
    ps->n_head = (int)q.ne[2];
    ps->n_head_kv = (int)k.ne[2];
    ps->n_seq = (int)q.ne[3];
    ps->n_seq_kv = (int)k.ne[3];
    ps->n_kv = (int)k.ne[1];
    ps->scale = p->scale;
    return true;
}

// Automatic split count: about `per_sm` CTAs per SM in one wave.
int64_t auto_splits(int64_t n_kv, int64_t ctas_per_split, int64_t min_rows, int per_sm = 2) {
    const int64_t target = per_sm * (int64_t)sm_count();
    int64_t s = (target + ctas_per_split - 1) / ctas_per_split;
    const int64_t cap = (n_kv + min_rows - 1) / min_rows;
    if (s > cap)
        s = cap;
    return s < 1 ? 1 : s;
}

void plan_splits(FaPlan *pl, int64_t requested) {
    const int64_t n_kv = pl->a.n_kv;
    const int64_t per = (int64_t)pl->a.n_head_kv * pl->n_qblocks * pl->a.n_seq;
    // the warp-MMA kernel fills every CTA slot its variant has on an SM; the
    // CUDA-core kernel two
    const int per_sm =
        pl->mma ? xq::decode_mma_occupancy(pl->cfg.type, pl->D, pl->cfg.VW, pl->a.n_qrows) : 2;
    int64_t s = requested > 0 ? requested : auto_splits(n_kv, per, 64, per_sm);
    if (n_kv == 0)
        s = 1;
    int64_t rows = s > 0 ? (n_kv + s - 1) / s : n_kv;
    if (requested <= 0 && pl->mma) {
        // automatic plan for the warp-MMA kernel: whole rounds of 64 rows (each
        // of the 4 warps one 16-key group per round, so no warp idles through
        // the last round) and at least 128 rows, which leaves fewer records
        // to merge on small caches -- at two CTAs per SM: config 2 128 splits
        // of 256 rows, 14.5 against 14.8 us (148 x 222), Q4_0 14.2 against
        // 14.7 us; config 1: 32 splits of 128 rows, 9.95 against 10.7 us (74 x 56)
        rows = (rows + 63) / 64 * 64;
        if (rows < 128)
            rows = 128;
    }
    if (rows < 1)
        rows = 1;
    pl->a.rows_per_split = rows;
    pl->n_splits = n_kv == 0 ? 1 : (n_kv + rows - 1) / rows;
}

// Where a caller's pointer lives: 0 device (or managed) memory, 1 pinned host
// memory (dev = its device-side address), -1 pageable host memory.
struct HostView {
    void *dev;
};
int host_view(const void *ptr, HostView *v) {
    v->dev = const_cast<void *>(ptr);
    if (!ptr)
        return 0;
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, ptr) != cudaSuccess) {
        cudaGetLastError(); // clear: treated as unknown (device) memory
        return 0;
    }
    if (at.type == cudaMemoryTypeHost) {
        v->dev = at.devicePointer;
        return v->dev ? 1 : -1;
    }
    return at.type == cudaMemoryTypeUnregistered ? -1 : 0;
}

size_t q_stage_bytes(const xq_tensor &q) {
    return (size_t)q.ne[0] * q.ne[1] * q.ne[2] * q.ne[3] * sizeof(float);
}

// Strided F32 [ne0, ne1, ne2, ne3] (ggml view, any byte strides) -> contiguous,
// one warp per row, every element of a lane's row loaded before any store (one
// PCIe round trip for host memory).  Launched as a programmatic dependent that
// releases its own dependent at once, so the attention kernel after it sets up
// and prefetches K/V into L2 while the rows cross PCIe; both the source (which
// the kernel before this one may have written) and the destination (which it
// may still be reading) are touched only after griddepcontrol.wait.
__global__ void stage_rows_kernel(const uint8_t *__restrict__ src, int64_t nb1, int64_t nb2,
                                  int64_t nb3, int64_t ne0, int64_t ne1, int64_t ne2,
                                  int64_t n_rows, float *__restrict__ dst) {
    constexpr int VR = 8; // elements per lane loaded at once (ne0 <= 256)
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    const int64_t row = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (row >= n_rows)
        return;
    const int64_t i1 = row % ne1, i2 = (row / ne1) % ne2, i3 = row / (ne1 * ne2);
    const float *s = reinterpret_cast<const float *>(src + i1 * nb1 + i2 * nb2 + i3 * nb3);
    float *d = dst + row * ne0;
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    if (ne0 <= 32 * VR) {
        float v[VR];
#pragma unroll
        for (int k = 0; k < VR; ++k)
            v[k] = lane + 32 * k < ne0 ? s[lane + 32 * k] : 0.0f;
#pragma unroll
        for (int k = 0; k < VR; ++k)
            if (lane + 32 * k < ne0)
                d[lane + 32 * k] = v[k];
    } else {
        for (int64_t i = lane; i < ne0; i += 32)
            d[i] = s[i];
    }
}

int stage_q(const xq_tensor &q, const void *src, float *dst, cudaStream_t st) {
    if (q.type != XQ_TYPE_F32 || q.nb[0] != 4)
        return fail(XQ_ERR_UNSUPPORTED, "flash_attn_ext: q must be F32 with contiguous rows");
    const int64_t n_rows = q.ne[1] * q.ne[2] * q.ne[3];
    if (n_rows <= 0)
        return XQ_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n_rows + 7) / 8), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, stage_rows_kernel,
                                          static_cast<const uint8_t *>(src), q.nb[1], q.nb[2],
                                          q.nb[3], q.ne[0], q.ne[1], q.ne[2], n_rows, dst),
                       "flash_attn_ext: staging q");
}

} // namespace

extern "C" {

const char *xq_version(void) { return "xq_b200 0.1 sm_100a"; }

const char *xq_last_error(void) { return g_last_error.c_str(); }

uint32_t xq_split_k(uint32_t active, uint32_t mode) {
    if (mode == 0) {
        const uint32_t k = (active + 255u) / 256u;
        return k < 1 ? 1 : (k > 32 ? 32 : k);
    }
    uint32_t target = 128, max_splits = 128;
    if (mode == 2) {
        target = 32;
        max_splits = 256;
    } else if (mode == 3) {
        target = 512;
        max_splits = 64;
    }
    const uint32_t wanted = (active + target - 1) / target;
    uint32_t k = wanted < max_splits ? wanted : max_splits;
    if (k > 256)
        k = 256;
    return k < 1 ? 1 : k;
}


// One planned call: the prefill kernel (pre) or the split-KV decode (+ merge).
static int fa_execute(const xq_fa_params *p, FaPlan &pl, bool pre, const xq::PrefillShape &ps,
                      void *ws, size_t ws_bytes, cudaStream_t st) {
    if (pre) {
        const size_t need = xq::prefill_ws_bytes(ps);
        if (!ws || ws_bytes < need)
            return fail(XQ_ERR_WORKSPACE, "flash_attn_ext: workspace %zu < %zu bytes", ws_bytes,
                        need);
        if (reinterpret_cast<uintptr_t>(ws) % 16)
            return fail(XQ_ERR_WORKSPACE, "flash_attn_ext: workspace must be 16-byte aligned");
        const char *why = "";
        cudaError_t e = xq::launch_prefill(ps, ws, st, &why);
        if (e != cudaSuccess)
            return fail(XQ_ERR_CUDA, "flash_attn_ext prefill: %s (%s)", cudaGetErrorString(e),
                        why);
        return XQ_OK;
    }
    dim3 grid((unsigned)pl.n_splits, (unsigned)(pl.a.n_head_kv * pl.n_qblocks),
              (unsigned)pl.a.n_seq);
    if (pl.n_splits == 1) {
        pl.a.direct = 1;
        return cuda_status(run_decode(pl, grid, st), "flash_attn_ext decode");
    }
    const size_t need = (size_t)pl.n_splits * (size_t)pl.n_rows * (size_t)(pl.D + 2) * 4;
    if (!ws || ws_bytes < need)
        return fail(XQ_ERR_WORKSPACE, "flash_attn_ext: workspace %zu < %zu bytes", ws_bytes, need);
    pl.a.direct = 0;
    pl.a.partials = static_cast<float *>(ws);
    int rc = cuda_status(run_decode(pl, grid, st), "flash_attn_ext decode");
    if (rc)
        return rc;
    return cuda_status(xq::launch_merge(pl.a.partials, pl.n_splits, pl.n_rows, pl.D, p->dst,
                                        nullptr, p->sinks, pl.a.n_head, st, 1, false, pl.mma),
                       "flash_attn_ext merge");
}

// Validate and plan once: the kernels' own workspace bytes in *main.
static int fa_plan(const xq_fa_params *p, FaPlan *pl, bool *pre, xq::PrefillShape *ps,
                   size_t *main) {
    int rc = fa_prepare(p, pl);
    if (rc)
        return rc;
    *pre = prefill_shape(p, *pl, ps);
    if (*pre) {
        *main = xq::prefill_ws_bytes(*ps);
        return XQ_OK;
    }
    plan_splits(pl, p->n_splits);
    *main = pl->n_splits <= 1
                ? 0
                : (size_t)pl->n_splits * (size_t)pl->n_rows * (size_t)(pl->D + 2) * sizeof(float);
    return XQ_OK;
}

int xq_flash_attn_ext(const xq_fa_params *p, void *ws, size_t ws_bytes, xq_stream_t stream) {
    if (!p)
        return fail(XQ_ERR_INVALID, "flash_attn_ext: null params");
    HostView hq, hd;
    const int kq = host_view(p->q.data, &hq), kd = host_view(p->dst, &hd);
    if (kq < 0 || kd < 0)
        return fail(XQ_ERR_INVALID,
                    "flash_attn_ext: q / dst in pageable host memory (pin it or use the device)");
    // pinned host dst: written in place by the kernels through its device view
    xq_fa_params p2 = *p;
    if (kd == 1)
        p2.dst = static_cast<float *>(hd.dev);
    FaPlan pl;
    bool pre = false;
    xq::PrefillShape ps;
    size_t main = 0;
    int rc = fa_plan(&p2, &pl, &pre, &ps, &main);
    if (rc)
        return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (kq == 1) {
        // pinned host q: copied into the tail of the workspace by a kernel,
        // then read from there (contiguous rows)
        const size_t off = (main + 255) / 256 * 256, need = off + q_stage_bytes(p->q);
        if (!ws || ws_bytes < need)
            return fail(XQ_ERR_WORKSPACE, "flash_attn_ext: workspace %zu < %zu bytes", ws_bytes,
                        need);
        float *staged = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + off);
        rc = stage_q(p->q, hq.dev, staged, st);
        if (rc)
            return rc;
        const int64_t nb1 = 4 * p->q.ne[0], nb2 = nb1 * p->q.ne[1], nb3 = nb2 * p->q.ne[2];
        pl.a.q = reinterpret_cast<const uint8_t *>(staged);
        pl.a.q_nb1 = nb1;
        pl.a.q_nb2 = nb2;
        pl.a.q_nb3 = nb3;
        ps.q = pl.a.q;
        ps.q_nb[0] = 4;
        ps.q_nb[1] = nb1;
        ps.q_nb[2] = nb2;
        ps.q_nb[3] = nb3;
        ws_bytes = off;
    }
    return fa_execute(&p2, pl, pre, ps, ws, ws_bytes, st);
}

int xq_flash_attn_ext_plan(const xq_fa_params *p, int32_t *kernel, int64_t *n_splits,
                           int64_t *rows_per_split) {
    FaPlan pl;
    bool pre = false;
    xq::PrefillShape ps;
    size_t main = 0;
    const int rc = fa_plan(p, &pl, &pre, &ps, &main);
    if (rc)
        return rc;
    if (kernel)
        *kernel = pre ? 2 : (pl.mma ? 1 : 0);
    if (n_splits)
        *n_splits = pre ? 0 : pl.n_splits;
    if (rows_per_split)
        *rows_per_split = pre ? 0 : pl.a.rows_per_split;
    return XQ_OK;
}

size_t xq_flash_attn_ext_workspace(const xq_fa_params *p) {
    FaPlan pl;
    bool pre = false;
    xq::PrefillShape ps;
    size_t main = 0;
    if (!p || fa_plan(p, &pl, &pre, &ps, &main) != XQ_OK)
        return 0;
    HostView hq;
    if (host_view(p->q.data, &hq) != 1)
        return main;
    return (main + 255) / 256 * 256 + q_stage_bytes(p->q);
}

int xq_fa_partials(const xq_fa_params *p, int64_t rows_per_split, int64_t split_begin,
                   int64_t split_end, float *partials, xq_stream_t stream) {
    FaPlan pl;
    int rc = fa_prepare(p, &pl);
    if (rc)
        return rc;
    if (p->sinks)
        return fail(XQ_ERR_UNSUPPORTED, "fa_partials: sinks belong to the merge");
    if (rows_per_split <= 0 || split_begin < 0 || split_end < split_begin || !partials)
        return fail(XQ_ERR_INVALID, "fa_partials: bad split range");
    if (split_end == split_begin)
        return XQ_OK;
    pl.a.rows_per_split = rows_per_split;
    pl.a.split_begin = split_begin;
    pl.a.direct = 0;
    pl.a.partials = partials;
    dim3 grid((unsigned)(split_end - split_begin), (unsigned)(pl.a.n_head_kv * pl.n_qblocks),
              (unsigned)pl.a.n_seq);
    return cuda_status(run_decode(pl, grid, reinterpret_cast<cudaStream_t>(stream)),
                       "fa_partials decode");
}

int xq_lse_merge(const float *partials, int64_t n_splits, int64_t n_rows, int64_t D, float *out,
                 float *lse, xq_stream_t stream) {
    if (!partials || !out || n_splits <= 0 || n_rows < 0 || (D != 64 && D != 128 && D != 256))
        return fail(XQ_ERR_INVALID, "lse_merge: bad arguments (D must be 64/128/256)");
    return cuda_status(xq::launch_merge(partials, n_splits, n_rows, (int)D, out, lse, nullptr, 1,
                                        reinterpret_cast<cudaStream_t>(stream)),
                       "lse_merge");
}

int xq_lse_merge_records(const float *partials, int64_t n_groups, int64_t splits_per_group,
                         int64_t n_rows, int64_t D, float *records, xq_stream_t stream) {
    if (!partials || !records || n_groups <= 0 || splits_per_group <= 0 || n_rows < 0 ||
        (D != 64 && D != 128 && D != 256))
        return fail(XQ_ERR_INVALID, "lse_merge_records: bad arguments (D must be 64/128/256)");
    return cuda_status(xq::launch_merge(partials, splits_per_group, n_rows, (int)D, records,
                                        nullptr, nullptr, 1,
                                        reinterpret_cast<cudaStream_t>(stream), n_groups, true),
                       "lse_merge_records");
}

// ---------------------------------------------------------------------------
// KV-sharded decode across GPUs (one process per GPU).

size_t xq_shard_exchange_bytes(int64_t n_groups, int64_t n_rows, int64_t D) {
    if (n_groups <= 0 || n_rows <= 0 || (D != 64 && D != 128 && D != 256))
        return 0;
    return xq::shard_exchange_bytes(n_groups, n_rows, (int)D);
}

int xq_shard_exchange_alloc(size_t bytes, void **exchange) {
    if (!exchange || bytes == 0)
        return fail(XQ_ERR_INVALID, "shard_exchange_alloc: bad arguments");
    *exchange = nullptr;
    void *p = nullptr;
    int rc = cuda_status(cudaMalloc(&p, bytes), "shard_exchange_alloc: cudaMalloc");
    if (rc)
        return rc;
    rc = cuda_status(cudaMemset(p, 0, bytes), "shard_exchange_alloc: cudaMemset");
    if (rc) {
        cudaFree(p);
        return rc;
    }
    *exchange = p;
    return XQ_OK;
}

int xq_shard_exchange_error(const void *exchange, int64_t n_groups, int64_t n_rows, int64_t D,
                            xq_stream_t stream, int32_t *error) {
    if (!exchange || !error || xq_shard_exchange_bytes(n_groups, n_rows, D) == 0)
        return fail(XQ_ERR_INVALID, "shard_exchange_error: bad arguments");
    const uint8_t *w = static_cast<const uint8_t *>(exchange) +
                       xq::shard_ctl_off(n_groups, n_rows, (int)D) + 2 * sizeof(unsigned);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned v = 0;
    int rc = cuda_status(cudaMemcpyAsync(&v, w, sizeof(v), cudaMemcpyDeviceToHost, st),
                         "shard_exchange_error: copy");
    if (!rc)
        rc = cuda_status(cudaStreamSynchronize(st), "shard_exchange_error: synchronize");
    *error = (int32_t)v;
    return rc;
}

int xq_shard_exchange_free(void *exchange) {
    return cuda_status(cudaFree(exchange), "shard_exchange_free");
}

int xq_ipc_export(const void *dev_ptr, xq_ipc_handle *handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(handle->bytes), "IPC handle size");
    if (!dev_ptr || !handle)
        return fail(XQ_ERR_INVALID, "ipc_export: null argument");
    cudaIpcMemHandle_t h;
    const int rc = cuda_status(cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr)),
                               "ipc_export: cudaIpcGetMemHandle");
    if (!rc)
        memcpy(handle->bytes, &h, sizeof(h));
    return rc;
}

int xq_ipc_open(const xq_ipc_handle *handle, void **dev_ptr) {
    if (!handle || !dev_ptr)
        return fail(XQ_ERR_INVALID, "ipc_open: null argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle->bytes, sizeof(h));
    return cuda_status(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess),
                       "ipc_open: cudaIpcOpenMemHandle");
}

int xq_ipc_close(void *dev_ptr) {
    return cuda_status(cudaIpcCloseMemHandle(dev_ptr), "ipc_close: cudaIpcCloseMemHandle");
}

namespace {

// [begin, end) of the groups rank r holds: contiguous blocks, the first
// n % world ranks one group longer.
void group_block(int64_t n, int world, int r, int64_t *b, int64_t *e) {
    const int64_t base = n / world, extra = n % world;
    *b = r * base + (r < extra ? r : extra);
    *e = *b + base + (r < extra ? 1 : 0);
}

int shard_check(const xq_shard_plan *s, const char *who) {
    if (!s || s->world < 1 || s->world > XQ_SHARD_MAX_RANKS || s->rank < 0 ||
        s->rank >= s->world || s->rows_per_split <= 0 || s->splits_per_group <= 0 ||
        s->n_groups < s->world)
        return fail(XQ_ERR_INVALID, "%s: bad shard plan (1 <= world <= %d, n_groups >= world)",
                    who, XQ_SHARD_MAX_RANKS);
    for (int r = 0; r < s->world; ++r)
        if (!s->exchange[r] || reinterpret_cast<uintptr_t>(s->exchange[r]) % 256)
            return fail(XQ_ERR_INVALID, "%s: exchange buffer of rank %d missing or unaligned", who,
                        r);
    return XQ_OK;
}

// Local split partials, then local group records (256-byte aligned after them).
size_t shard_ws_layout(const FaPlan &pl, const xq_shard_plan *s, size_t *rec_off) {
    int64_t g0, g1;
    group_block(s->n_groups, s->world, s->rank, &g0, &g1);
    const size_t rec = (size_t)pl.n_rows * (size_t)(pl.D + 2) * sizeof(float);
    *rec_off = ((size_t)(g1 - g0) * s->splits_per_group * rec + 255) / 256 * 256;
    return *rec_off + (size_t)(g1 - g0) * rec;
}

} // namespace

size_t xq_fa_shard_workspace(const xq_fa_params *p, const xq_shard_plan *s) {
    FaPlan pl;
    if (!p || shard_check(s, "fa_shard_workspace") || fa_prepare(p, &pl))
        return 0;
    size_t rec_off;
    return shard_ws_layout(pl, s, &rec_off);
}

int xq_fa_shard_push(const xq_fa_params *p, const xq_shard_plan *s, void *ws, size_t ws_bytes,
                     xq_stream_t stream) {
    int rc = shard_check(s, "fa_shard_push");
    if (rc)
        return rc;
    FaPlan pl;
    if ((rc = fa_prepare(p, &pl)))
        return rc;
    if (p->sinks)
        return fail(XQ_ERR_UNSUPPORTED, "fa_shard_push: sinks belong to xq_fa_shard_finish");
    size_t rec_off;
    const size_t need = shard_ws_layout(pl, s, &rec_off);
    if (!ws || ws_bytes < need || reinterpret_cast<uintptr_t>(ws) % 256)
        return fail(XQ_ERR_WORKSPACE, "fa_shard_push: workspace %zu < %zu bytes (256-aligned)",
                    ws_bytes, need);
    int64_t g0, g1;
    group_block(s->n_groups, s->world, s->rank, &g0, &g1);
    const int64_t n_local = (g1 - g0) * s->splits_per_group;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // 1. this rank's splits (its k / v views start at its first split's row 0)
    pl.a.rows_per_split = s->rows_per_split;
    pl.a.split_begin = 0;
    pl.a.direct = 0;
    pl.a.partials = static_cast<float *>(ws);
    dim3 grid((unsigned)n_local, (unsigned)(pl.a.n_head_kv * pl.n_qblocks), (unsigned)pl.a.n_seq);
    if ((rc = cuda_status(run_decode(pl, grid, st), "fa_shard_push decode")))
        return rc;
    // 2. one (O, lse, 1) record per local group, in split order
    float *recs = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + rec_off);
    if ((rc = cuda_status(xq::launch_merge(pl.a.partials, s->splits_per_group, pl.n_rows, pl.D,
                                           recs, nullptr, nullptr, 1, st, g1 - g0, true),
                          "fa_shard_push group records")))
        return rc;
    // 3. the records into every rank's exchange half of this step
    xq::ShardPushArgs a;
    memset(&a, 0, sizeof(a));
    const size_t rec_bytes = (size_t)pl.n_rows * (size_t)(pl.D + 2) * sizeof(float);
    a.src = reinterpret_cast<const float2 *>(recs);
    a.n8 = (int64_t)((g1 - g0) * rec_bytes / 8);
    a.dst_off8 = (int64_t)(g0 * rec_bytes / 8);
    a.parity = (int)(s->step & 1u);
    a.half_off = (size_t)a.parity * xq::shard_records_bytes(s->n_groups, pl.n_rows, pl.D);
    a.ctl_off = xq::shard_ctl_off(s->n_groups, pl.n_rows, pl.D);
    for (int r = 0; r < s->world; ++r)
        a.peers[r] = static_cast<uint8_t *>(s->exchange[r]);
    return cuda_status(xq::launch_shard_push(a, s->world, st), "fa_shard_push exchange");
}

int xq_fa_shard_finish(const xq_shard_plan *s, int64_t n_rows, int64_t D, const float *sinks,
                       int32_t n_head, float *out, float *lse, xq_stream_t stream) {
    int rc = shard_check(s, "fa_shard_finish");
    if (rc)
        return rc;
    if (!out || n_rows <= 0 || (D != 64 && D != 128 && D != 256) || (sinks && n_head <= 0))
        return fail(XQ_ERR_INVALID, "fa_shard_finish: bad arguments");
    // every rank's chunks, as each pushes its block of groups
    const size_t rec_bytes = (size_t)n_rows * (size_t)(D + 2) * sizeof(float);
    int64_t expected = 0;
    for (int r = 0; r < s->world; ++r) {
        int64_t b, e;
        group_block(s->n_groups, s->world, r, &b, &e);
        expected += xq::shard_chunks((size_t)(e - b) * rec_bytes);
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int parity = (int)(s->step & 1u);
    void *own = s->exchange[s->rank];
    if ((rc = cuda_status(xq::launch_shard_wait(own, s->n_groups, n_rows, (int)D, parity,
                                                (unsigned)expected, st),
                          "fa_shard_finish wait")))
        return rc;
    const float *half = reinterpret_cast<const float *>(
        static_cast<const uint8_t *>(own) +
        (size_t)parity * xq::shard_records_bytes(s->n_groups, n_rows, (int)D));
    return cuda_status(xq::launch_merge(half, s->n_groups, n_rows, (int)D, out, lse, sinks,
                                        sinks ? n_head : 1, st),
                       "fa_shard_finish merge");
}

// ---------------------------------------------------------------------------
// RKVA range attention.

static int range_prepare(int32_t storage, const void *k, const void *v, uint32_t n_head,
                         uint32_t n_hkv, uint32_t D, uint32_t origin, uint32_t active,
                         uint32_t n_tokens, const int32_t *positions, const float *q,
                         float kq_scale, float *out, float *lse, xq_fa_params *fp, FaPlan *pl) {
    if (!kv_type_ok(storage))
        return fail(XQ_ERR_UNSUPPORTED, "attend_range: storage %d", storage);
    if (!n_tokens || !positions || !q || !out || !lse || !n_hkv || n_head % n_hkv ||
        (active && (!k || !v)))
        return fail(XQ_ERR_INVALID, "attend_range: invalid arguments");
    memset(fp, 0, sizeof(*fp));
    const uint64_t rec = (uint64_t)xq::rec_bytes(storage, (int)D);
    fp->q = {XQ_TYPE_F32, 0, q, {D, n_tokens, n_head, 1},
             {4, (uint64_t)n_head * D * 4, (uint64_t)D * 4, (uint64_t)n_tokens * n_head * D * 4}};
    const void *kd = active ? k : q; // any valid pointer: no rows are read
    const void *vd = active ? v : q;
    fp->k = {storage, 0, kd, {D, active, n_hkv, 1},
             {0, n_hkv * rec, rec, (uint64_t)active * n_hkv * rec}};
    fp->v = {storage, 0, vd, {D, active, n_hkv, 1},
             {0, n_hkv * rec, rec, (uint64_t)active * n_hkv * rec}};
    fp->dst = out;
    fp->scale = kq_scale;
    int rc = fa_prepare(fp, pl);
    if (rc)
        return rc;
    // RKVA multiplies raw F32 q; only the CUDA-core kernel implements that
    pl->a.q_convert = 0;
    pl->mma = false;
    pl->n_qblocks = (pl->a.n_qrows + pl->cfg.NR - 1) / pl->cfg.NR;
    pl->a.positions = positions;
    pl->a.origin = (int)origin;
    pl->a.active = (int)active;
    pl->a.lse = lse;
    return XQ_OK;
}

static int64_t range_splits(uint32_t active, uint32_t mode, const FaPlan &pl) {
    if (mode <= 3)
        return xq_split_k(active, mode);
    const int64_t per = (int64_t)pl.a.n_head_kv * pl.n_qblocks;
    return auto_splits(active, per, 64);
}

size_t xq_attend_range_workspace(int32_t storage, uint32_t n_tokens, uint32_t active,
                                 uint32_t n_head, uint32_t n_head_kv, uint32_t head_dim,
                                 uint32_t split_mode) {
    if (!n_head_kv || !n_tokens)
        return 0;
    const uint32_t G = n_head / n_head_kv;
    const int NR = n_tokens * G <= 4 ? 4 : n_tokens * G <= 8 ? 8 : 16;
    FaPlan pl;
    pl.a.n_head_kv = (int)n_head_kv;
    pl.n_qblocks = (int)((n_tokens * G + NR - 1) / NR);
    const int64_t s = range_splits(active, split_mode, pl);
    if (s <= 1)
        return 0;
    (void)storage;
    return (size_t)s * n_tokens * n_head * (head_dim + 2) * sizeof(float);
}

int xq_attend_range(int32_t storage, const void *k, const void *v, uint32_t n_head,
                    uint32_t n_head_kv, uint32_t head_dim, uint32_t origin, uint32_t active,
                    uint32_t n_tokens, const int32_t *positions, const float *q, float kq_scale,
                    uint32_t split_mode, float *out, float *lse, void *ws, size_t ws_bytes,
                    xq_stream_t stream) {
    xq_fa_params fp;
    FaPlan pl;
    int rc = range_prepare(storage, k, v, n_head, n_head_kv, head_dim, origin, active, n_tokens,
                           positions, q, kq_scale, out, lse, &fp, &pl);
    if (rc)
        return rc;
    if (split_mode > 4)
        return fail(XQ_ERR_INVALID, "attend_range: split mode %u", split_mode);
    int64_t s = range_splits(active, split_mode, pl);
    const int64_t rows = active ? (active + s - 1) / s : 1;
    pl.a.rows_per_split = rows;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    dim3 grid((unsigned)s, (unsigned)(pl.a.n_head_kv * pl.n_qblocks), 1);
    if (s == 1) {
        pl.a.direct = 1;
        return cuda_status(run_decode(pl, grid, st), "attend_range decode");
    }
    const size_t need = (size_t)s * pl.n_rows * (head_dim + 2) * 4;
    if (!ws || ws_bytes < need)
        return fail(XQ_ERR_WORKSPACE, "attend_range: workspace %zu < %zu bytes", ws_bytes, need);
    pl.a.direct = 0;
    pl.a.lse = nullptr;
    pl.a.partials = static_cast<float *>(ws);
    rc = cuda_status(run_decode(pl, grid, st), "attend_range decode");
    if (rc)
        return rc;
    return cuda_status(xq::launch_merge(pl.a.partials, s, pl.n_rows, (int)head_dim, out, lse,
                                        nullptr, 1, st),
                       "attend_range merge");
}

// ---------------------------------------------------------------------------
// Native KVarN4 range attention.

// Split plan: body splits of whole 128-row groups over rows [0, active - tail)
// (about two CTAs per SM in all, at most one split per group) and one split
// for the precision tail rows.
struct Kvarn4Plan {
    int64_t rows; // rows per body split
    int n_body, n_splits;
};
static Kvarn4Plan kvarn4_plan(uint32_t active, uint32_t tail, uint32_t n_head_kv,
                              uint32_t n_tokens) {
    const int64_t tail_rows = active < tail ? active : tail;
    const int64_t body = (int64_t)active - tail_rows;
    const int64_t groups = (body + 127) / 128;
    const int64_t per = (int64_t)n_head_kv * n_tokens;
    int64_t s = (2 * (int64_t)sm_count() + per - 1) / per - (tail_rows ? 1 : 0);
    s = s < 1 ? 1 : s > groups ? groups : s;
    Kvarn4Plan pl;
    pl.rows = groups ? 128 * ((groups + s - 1) / s) : 128;
    pl.n_body = groups ? (int)((body + pl.rows - 1) / pl.rows) : 0;
    pl.n_splits = pl.n_body + (tail_rows ? 1 : 0);
    if (pl.n_splits == 0)
        pl.n_splits = 1; // nothing active: one empty split (O = 0, LSE = -inf)
    return pl;
}

// Workspace: the split partials, then (256-byte aligned) room for q when the
// caller's q is in pinned host memory and is staged to the device first.
static size_t kvarn4_q_offset(const Kvarn4Plan &pl, uint32_t n_head, uint32_t n_tokens) {
    return ((size_t)pl.n_splits * n_tokens * n_head * 258 * sizeof(float) + 255) / 256 * 256;
}

size_t xq_attend_range_kvarn4_workspace(const xq_kvarn4_desc *d, uint32_t n_head,
                                        uint32_t active, uint32_t n_tokens) {
    if (!d || d->n_head_kv <= 0 || !n_tokens || d->precision_tail < 0)
        return 0;
    const Kvarn4Plan pl =
        kvarn4_plan(active, (uint32_t)d->precision_tail, (uint32_t)d->n_head_kv, n_tokens);
    return kvarn4_q_offset(pl, n_head, n_tokens) + (size_t)n_tokens * n_head * 256 * sizeof(float);
}

int xq_attend_range_kvarn4(const xq_kvarn4_desc *d, const void *k_plane, const void *v_plane,
                           uint32_t n_head, uint32_t active, uint32_t n_tokens,
                           const int32_t *positions, const float *q, float kq_scale, float *out,
                           float *lse, void *ws, size_t ws_bytes, xq_stream_t stream) {
    if (!d || !k_plane || !v_plane || !positions || !q || !out)
        return fail(XQ_ERR_INVALID, "attend_range_kvarn4: null argument");
    if (d->origin < 0 || d->origin % 128 || d->capacity <= 0 ||
        (d->precision_tail != 0 && d->precision_tail != 128) || d->n_head_kv <= 0)
        return fail(XQ_ERR_INVALID,
                    "attend_range_kvarn4: descriptor (origin %% 128, capacity > 0, tail 0/128)");
    if (active > (uint32_t)d->capacity || n_head == 0 || n_head % d->n_head_kv ||
        n_head / d->n_head_kv > 8 || n_tokens == 0 || n_tokens > 65535 ||
        (uint32_t)d->n_head_kv > 65535)
        return fail(XQ_ERR_INVALID,
                    "attend_range_kvarn4: shape (active <= capacity, 1..8 q heads per kv head)");
    if (((reinterpret_cast<uintptr_t>(k_plane) | reinterpret_cast<uintptr_t>(v_plane)) & 15) != 0)
        return fail(XQ_ERR_INVALID, "attend_range_kvarn4: planes must be 16-byte aligned");
    const Kvarn4Plan pl =
        kvarn4_plan(active, (uint32_t)d->precision_tail, (uint32_t)d->n_head_kv, n_tokens);
    const int64_t s = pl.n_splits;
    const size_t q_off = kvarn4_q_offset(pl, n_head, n_tokens);
    const size_t need = q_off + (size_t)n_tokens * n_head * 256 * sizeof(float);
    if (!ws || ws_bytes < need)
        return fail(XQ_ERR_WORKSPACE, "attend_range_kvarn4: workspace %zu < %zu bytes", ws_bytes,
                    need);
    // q, out and lse may be in pinned host memory: q is staged into the
    // workspace by a kernel, out / lse are written through their device view
    HostView hq, ho, hl;
    const int kq = host_view(q, &hq), ko = host_view(out, &ho), kl = host_view(lse, &hl);
    if (kq < 0 || ko < 0 || kl < 0)
        return fail(XQ_ERR_INVALID,
                    "attend_range_kvarn4: q / out / lse in pageable host memory (pin them or use "
                    "the device)");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (kq == 1) {
        float *staged = reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + q_off);
        xq_tensor qt = {};
        qt.type = XQ_TYPE_F32;
        qt.ne[0] = 256, qt.ne[1] = n_head, qt.ne[2] = n_tokens, qt.ne[3] = 1;
        qt.nb[0] = 4, qt.nb[1] = 1024, qt.nb[2] = 1024 * (int64_t)n_head;
        qt.nb[3] = qt.nb[2] * n_tokens;
        const int rc = stage_q(qt, hq.dev, staged, st);
        if (rc)
            return rc;
        q = staged;
    }
    if (ko == 1)
        out = static_cast<float *>(ho.dev);
    if (kl == 1)
        lse = static_cast<float *>(hl.dev);
    xq::Kvarn4Launch l;
    l.k = static_cast<const uint8_t *>(k_plane);
    l.v = static_cast<const uint8_t *>(v_plane);
    l.q = q;
    l.positions = positions;
    l.partials = static_cast<float *>(ws);
    l.records_bytes = (int64_t)((d->capacity + 127) / 128) * 2 * d->n_head_kv * 8960;
    l.origin = d->origin;
    l.active = (int)active;
    l.tail = d->precision_tail;
    l.n_head = (int)n_head;
    l.n_head_kv = d->n_head_kv;
    l.n_tokens = (int)n_tokens;
    l.rows_per_split = (int)pl.rows;
    l.n_body = pl.n_body;
    l.n_splits = pl.n_splits;
    l.scale = kq_scale;
    int rc = cuda_status(xq::launch_kvarn4(l, st), "attend_range_kvarn4 partials");
    if (rc)
        return rc;
    return cuda_status(xq::launch_merge(l.partials, s, (int64_t)n_tokens * n_head, 256, out, lse,
                                        nullptr, 1, st),
                       "attend_range_kvarn4 merge");
}

// ---------------------------------------------------------------------------
// GATED_DELTA_NET.

// Validates a GATED_DELTA_NET call and fills the kernel arguments.
// head_begin / n_head_total: the call covers value heads [head_begin,
// head_begin + v->ne[1]) of an op with n_head_total value heads (< 0: the
// whole op, head_begin 0).
static int gdn_args(const xq_tensor *q, const xq_tensor *k, const xq_tensor *v,
                    const xq_tensor *g, const xq_tensor *beta, const xq_tensor *state,
                    float *dst, int32_t slots, xq::GdnArgs *out, int64_t head_begin = 0,
                    int64_t n_head_total = -1) {
    if (!q || !k || !v || !g || !beta || !state || !dst)
        return fail(XQ_ERR_INVALID, "gated_delta_net: null argument");
    const xq_tensor *all[6] = {q, k, v, g, beta, state};
    for (int i = 0; i < 6; ++i) {
        if (all[i]->type != XQ_TYPE_F32 || !all[i]->data)
            return fail(XQ_ERR_UNSUPPORTED, "gated_delta_net: src %d must be F32", i);
        if (all[i]->nb[0] != 4 && all[i]->ne[0] != 1)
            return fail(XQ_ERR_UNSUPPORTED, "gated_delta_net: src %d rows not contiguous", i);
    }
    const int64_t S = v->ne[0], H = v->ne[1], T = v->ne[2], n_seq = v->ne[3];
    const int64_t H_k = q->ne[1];
    if (S != 128)
        return fail(XQ_ERR_UNSUPPORTED, "gated_delta_net: head size %lld (supported: 128)",
                    (long long)S);
    if (n_head_total < 0)
        n_head_total = H;
    if (head_begin < 0 || head_begin + H > n_head_total || H <= 0)
        return fail(XQ_ERR_INVALID, "gated_delta_net: value heads [%lld, %lld) outside [0, %lld)",
                    (long long)head_begin, (long long)(head_begin + H), (long long)n_head_total);
    if (q->ne[0] != S || k->ne[0] != S || k->ne[1] != H_k || H_k <= 0 || n_head_total % H_k ||
        q->ne[2] != T || k->ne[2] != T || q->ne[3] <= 0 || k->ne[3] <= 0 || n_seq % q->ne[3] ||
        n_seq % k->ne[3] || T <= 0)
        return fail(XQ_ERR_INVALID, "gated_delta_net: inconsistent q/k/v shapes");
    for (const xq_tensor *gt : {g, beta})
        if (gt->ne[0] != 1 || gt->ne[1] != H || gt->ne[2] != T || gt->ne[3] != n_seq)
            return fail(XQ_ERR_UNSUPPORTED,
                        "gated_delta_net: gates must be scalar per head [1, H, T, n_seq]");
    if (state->ne[0] != S || state->ne[1] != S || state->ne[2] != H || state->ne[3] != n_seq)
        return fail(XQ_ERR_INVALID, "gated_delta_net: state must be [S, S, H, n_seq]");
    if (slots < 1 || slots > 64)
        return fail(XQ_ERR_INVALID, "gated_delta_net: slots %d outside [1, 64]", slots);
    if (H * n_seq > 65535 * 64)
        return fail(XQ_ERR_UNSUPPORTED, "gated_delta_net: too many heads x sequences");
    xq::GdnArgs a;
    a.q = static_cast<const float *>(q->data);
    a.k = static_cast<const float *>(k->data);
    a.v = static_cast<const float *>(v->data);
    a.g = static_cast<const float *>(g->data);
    a.beta = static_cast<const float *>(beta->data);
    a.state = static_cast<const float *>(state->data);
    a.q_nb1 = (int64_t)q->nb[1]; a.q_nb2 = (int64_t)q->nb[2]; a.q_nb3 = (int64_t)q->nb[3];
    a.k_nb1 = (int64_t)k->nb[1]; a.k_nb2 = (int64_t)k->nb[2]; a.k_nb3 = (int64_t)k->nb[3];
    a.v_nb1 = (int64_t)v->nb[1]; a.v_nb2 = (int64_t)v->nb[2]; a.v_nb3 = (int64_t)v->nb[3];
    a.g_nb1 = (int64_t)g->nb[1]; a.g_nb2 = (int64_t)g->nb[2]; a.g_nb3 = (int64_t)g->nb[3];
    a.b_nb1 = (int64_t)beta->nb[1]; a.b_nb2 = (int64_t)beta->nb[2]; a.b_nb3 = (int64_t)beta->nb[3];
    a.s_nb1 = (int64_t)state->nb[1]; a.s_nb2 = (int64_t)state->nb[2];
    a.s_nb3 = (int64_t)state->nb[3];
    a.dst = dst;
    a.H = (int)H;
    a.H_k = (int)H_k;
    a.T = (int)T;
    a.n_seq = (int)n_seq;
    a.rq3 = (int)(n_seq / q->ne[3]);
    a.rk3 = (int)(n_seq / k->ne[3]);
    a.slots = slots;
    a.scale = 1.0f / sqrtf((float)S);
    a.h_off = (int)(head_begin % H_k);
    *out = a;
    return XQ_OK;
}

int xq_gated_delta_net(const xq_tensor *q, const xq_tensor *k, const xq_tensor *v,
                       const xq_tensor *g, const xq_tensor *beta, const xq_tensor *state,
                       float *dst, int32_t slots, xq_stream_t stream) {
    xq::GdnArgs a;
    const int rc = gdn_args(q, k, v, g, beta, state, dst, slots, &a);
    if (rc != XQ_OK)
        return rc;
    return cuda_status(xq::launch_gdn(a, reinterpret_cast<cudaStream_t>(stream)),
                       "gated_delta_net");
}

size_t xq_gated_delta_net_workspace(const xq_tensor *v, int32_t slots) {
    if (!v || v->ne[0] != 128 || v->ne[1] <= 0 || v->ne[2] <= 0 || v->ne[3] <= 0 ||
        v->ne[1] > 65535 || v->ne[2] > INT32_MAX || v->ne[3] > 65535 || slots < 1 || slots > 64)
        return 0;
    return xq::gdn_chunk_workspace((int)v->ne[2], (int)v->ne[1], (int)v->ne[3], slots);
}

int xq_gated_delta_net_ws(const xq_tensor *q, const xq_tensor *k, const xq_tensor *v,
                          const xq_tensor *g, const xq_tensor *beta, const xq_tensor *state,
                          float *dst, int32_t slots, void *workspace, size_t workspace_bytes,
                          xq_stream_t stream) {
    xq::GdnArgs a;
    const int rc = gdn_args(q, k, v, g, beta, state, dst, slots, &a);
    if (rc != XQ_OK)
        return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (!xq::gdn_chunk_eligible(a))
        return cuda_status(xq::launch_gdn(a, st), "gated_delta_net");
    const size_t need = xq::gdn_chunk_workspace(a.T, a.H, a.n_seq, a.slots);
    if (!workspace || workspace_bytes < need)
        return fail(XQ_ERR_WORKSPACE, "gated_delta_net: workspace %zu bytes, %zu needed",
                    workspace_bytes, need);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return fail(XQ_ERR_WORKSPACE, "gated_delta_net: workspace must be 256-byte aligned");
    return cuda_status(xq::launch_gdn_chunked(a, workspace, workspace_bytes, st),
                       "gated_delta_net (chunked)");
}

int xq_gated_delta_net_heads(const xq_tensor *q, const xq_tensor *k, const xq_tensor *v,
                             const xq_tensor *g, const xq_tensor *beta, const xq_tensor *state,
                             float *dst, int32_t slots, int64_t head_begin, int64_t n_head_total,
                             void *workspace, size_t workspace_bytes, xq_stream_t stream) {
    if (n_head_total <= 0)
        return fail(XQ_ERR_INVALID, "gated_delta_net_heads: n_head_total must be positive");
    xq::GdnArgs a;
    const int rc = gdn_args(q, k, v, g, beta, state, dst, slots, &a, head_begin, n_head_total);
    if (rc != XQ_OK)
        return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (!xq::gdn_chunk_eligible(a))
        return cuda_status(xq::launch_gdn(a, st), "gated_delta_net_heads");
    const size_t need = xq::gdn_chunk_workspace(a.T, a.H, a.n_seq, a.slots);
    if (!workspace || workspace_bytes < need)
        return fail(XQ_ERR_WORKSPACE, "gated_delta_net_heads: workspace %zu bytes, %zu needed",
                    workspace_bytes, need);
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
        return fail(XQ_ERR_WORKSPACE, "gated_delta_net_heads: workspace must be 256-byte aligned");
    return cuda_status(xq::launch_gdn_chunked(a, workspace, workspace_bytes, st),
                       "gated_delta_net_heads (chunked)");
}

// ---------------------------------------------------------------------------
// Codecs.

int xq_set_rows(const xq_tensor *src, const xq_tensor *idx, const xq_tensor *dst,
                xq_stream_t stream) {
    if (!src || !idx || !dst)
        return fail(XQ_ERR_INVALID, "set_rows: null tensor");
    if (src->type != XQ_TYPE_F32 || src->nb[0] != 4)
        return fail(XQ_ERR_UNSUPPORTED, "set_rows: src must be F32 with contiguous rows");
    if (idx->type != XQ_TYPE_I32 && idx->type != XQ_TYPE_I64)
        return fail(XQ_ERR_UNSUPPORTED, "set_rows: indices must be I32 or I64");
    const int t = dst->type;
    if (t != XQ_TYPE_F32 && t != XQ_TYPE_F16 && t != XQ_TYPE_Q8_0 && t != XQ_TYPE_Q4_0)
        return fail(XQ_ERR_UNSUPPORTED, "set_rows: dst type %d (F32/F16/Q8_0/Q4_0)", t);
    const int64_t ne0 = src->ne[0], ne1 = src->ne[1], ne2 = src->ne[2], ne3 = src->ne[3];
    if (dst->ne[0] != ne0 || dst->ne[2] != ne2 || dst->ne[3] != ne3 || idx->ne[0] != ne1 ||
        idx->ne[1] <= 0 || idx->ne[2] <= 0 || ne2 % idx->ne[1] || ne3 % idx->ne[2] ||
        idx->ne[3] != 1 || ne0 <= 0)
        return fail(XQ_ERR_INVALID, "set_rows: shapes (ggml_set_rows rules)");
    if ((t == XQ_TYPE_Q8_0 || t == XQ_TYPE_Q4_0) && ne0 % 32)
        return fail(XQ_ERR_INVALID, "set_rows: row length %lld not a multiple of 32",
                    (long long)ne0);
    if (!src->data || !idx->data || !dst->data)
        return fail(XQ_ERR_INVALID, "set_rows: null data");
    xq::SetRowsArgs a;
    a.src = static_cast<const uint8_t *>(src->data);
    a.s_nb1 = src->nb[1];
    a.s_nb2 = src->nb[2];
    a.s_nb3 = src->nb[3];
    a.idx = static_cast<const uint8_t *>(idx->data);
    a.i_nb0 = idx->nb[0];
    a.i_nb1 = idx->nb[1];
    a.i_nb2 = idx->nb[2];
    a.i_ne1 = idx->ne[1];
    a.i_ne2 = idx->ne[2];
    a.idx_i64 = idx->type == XQ_TYPE_I64;
    a.dst = static_cast<uint8_t *>(const_cast<void *>(dst->data));
    a.d_nb1 = dst->nb[1];
    a.d_nb2 = dst->nb[2];
    a.d_nb3 = dst->nb[3];
    a.d_rows = dst->ne[1];
    a.ne0 = ne0;
    a.ne1 = ne1;
    a.ne2 = ne2;
    a.ne3 = ne3;
    a.n_units = ne1 * ne2 * ne3 * ((t == XQ_TYPE_F32 || t == XQ_TYPE_F16) ? ne0 : ne0 / 32);
    a.n_sm = sm_count();
    return cuda_status(xq::launch_set_rows(t, a, reinterpret_cast<cudaStream_t>(stream)),
                       "set_rows");
}

int xq_dequantize_rows(int32_t type, const void *src, uint64_t src_row_stride, float *dst,
                       uint64_t dst_row_stride, int64_t n_rows, int64_t n_per_row,
                       xq_stream_t stream) {
    if (!kv_type_ok(type))
        return fail(XQ_ERR_UNSUPPORTED, "dequantize_rows: type %d", type);
    if (!src || !dst || n_rows < 0 || n_per_row <= 0 || (type != XQ_TYPE_F16 && n_per_row % 32))
        return fail(XQ_ERR_INVALID, "dequantize_rows: bad arguments");
    return cuda_status(xq::launch_dequant(type, src, src_row_stride, dst, dst_row_stride, n_rows,
                                          n_per_row, reinterpret_cast<cudaStream_t>(stream)),
                       "dequantize_rows");
}

int xq_quantize_rows(int32_t type, const float *src, uint64_t src_row_stride, void *dst,
                     uint64_t dst_row_stride, int64_t n_rows, int64_t n_per_row,
                     xq_stream_t stream) {
    if (!kv_type_ok(type))
        return fail(XQ_ERR_UNSUPPORTED, "quantize_rows: type %d", type);
    if (!src || !dst || n_rows < 0 || n_per_row <= 0 || (type != XQ_TYPE_F16 && n_per_row % 32))
        return fail(XQ_ERR_INVALID, "quantize_rows: bad arguments");
    return cuda_status(xq::launch_quant(type, src, src_row_stride, dst, dst_row_stride, n_rows,
                                        n_per_row, reinterpret_cast<cudaStream_t>(stream)),
                       "quantize_rows");
}

} // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free FLASH_ATTN_EXT: split partials live in a file-scope device
// array instead of a caller workspace.  In host code the array's name is only
// a host-side stand-in, never a device address: the address each device uses
// comes from cudaGetSymbolAddress, looked up once per device with that device
// current, and is what the kernels receive.

static __device__ __align__(256) unsigned char g_noalloc_scratch[XQ_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kNoallocMaxDevices];
} // namespace

extern "C" int xq_flash_attn_ext_noalloc(const xq_fa_params *p, xq_stream_t stream) {
    if (!p)
        return fail(XQ_ERR_INVALID, "flash_attn_ext_noalloc: null params");
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return cuda_status(e, "flash_attn_ext_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kNoallocMaxDevices)
        return fail(XQ_ERR_UNSUPPORTED, "flash_attn_ext_noalloc: device %d beyond %d", dev,
                    kNoallocMaxDevices);
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void *ptr = nullptr;
            e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess)
                return cuda_status(e, "flash_attn_ext_noalloc: cudaGetSymbolAddress");
            g_noalloc_ptr[dev] = ptr;
        }
        scratch = g_noalloc_ptr[dev];
    }
    // q and dst: device memory, or pinned host memory (q staged into the
    // scratch by a kernel, dst written through its device view); pageable
    // host memory is rejected before anything is launched
    HostView hq, hd;
    const int kq = host_view(p->q.data, &hq), kd = host_view(p->dst, &hd);
    if (kq < 0 || kd < 0)
        return fail(XQ_ERR_INVALID,
                    "flash_attn_ext_noalloc: q / dst in pageable host memory (pin it or use the "
                    "device)");
    xq_fa_params p2 = *p;
    if (kd == 1)
        p2.dst = static_cast<float *>(hd.dev);
    FaPlan pl;
    int rc = fa_prepare(&p2, &pl);
    if (rc)
        return rc;
    plan_splits(&pl, p->n_splits);
    const size_t part = pl.n_splits > 1
                            ? (size_t)pl.n_splits * (size_t)pl.n_rows * (size_t)(pl.D + 2) * 4
                            : 0;
    const size_t q_off = (part + 255) / 256 * 256;
    const size_t need = kq == 1 ? q_off + q_stage_bytes(p->q) : part;
    if (need > (size_t)XQ_NOALLOC_SCRATCH_BYTES)
        return fail(XQ_ERR_WORKSPACE,
                    "flash_attn_ext_noalloc: %lld splits x %lld rows%s need %zu bytes of scratch, "
                    "the static scratch holds %u; pass a smaller n_splits",
                    (long long)pl.n_splits, (long long)pl.n_rows,
                    kq == 1 ? " and the staged q" : "", need, (unsigned)XQ_NOALLOC_SCRATCH_BYTES);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (kq == 1) {
        float *staged = reinterpret_cast<float *>(static_cast<uint8_t *>(scratch) + q_off);
        rc = stage_q(p->q, hq.dev, staged, st);
        if (rc)
            return rc;
        p2.q.data = staged;
        p2.q.nb[0] = 4;
        p2.q.nb[1] = 4 * p->q.ne[0];
        p2.q.nb[2] = p2.q.nb[1] * p->q.ne[1];
        p2.q.nb[3] = p2.q.nb[2] * p->q.ne[2];
        // same shapes, so the same split plan, now reading the staged q
        rc = fa_prepare(&p2, &pl);
        if (rc)
            return rc;
        plan_splits(&pl, p->n_splits);
    }
    dim3 grid((unsigned)pl.n_splits, (unsigned)(pl.a.n_head_kv * pl.n_qblocks),
              (unsigned)pl.a.n_seq);
    if (pl.n_splits == 1) {
        pl.a.direct = 1;
        return cuda_status(run_decode(pl, grid, st), "flash_attn_ext_noalloc decode");
    }
    pl.a.direct = 0;
    pl.a.partials = static_cast<float *>(scratch);
    rc = cuda_status(run_decode(pl, grid, st), "flash_attn_ext_noalloc decode");
    if (rc)
        return rc;
    return cuda_status(xq::launch_merge(pl.a.partials, pl.n_splits, pl.n_rows, pl.D, p2.dst,
                                        nullptr, p->sinks, pl.a.n_head, st, 1, false, pl.mma),
                       "flash_attn_ext_noalloc merge");
}
