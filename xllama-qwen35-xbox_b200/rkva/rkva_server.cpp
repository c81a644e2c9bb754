// The RKVA range server on a B200: a host keeps KV positions [0, P) and sends
// the rows at positions >= P to this server, which holds them in HBM and
// answers attention over them with (O, LSE) for the host to merge with its own
// partial -- the role of the reference's Xbox server (uwp/rkva/remote-attn.cpp,
// request dispatch :286-1240, connection loop :1370-1451) for row ranges.
//
// Served: HELLO, CREATE_SESSION, DESTROY_SESSION, RESET, TRIM / REWIND, PING,
// GET_STATS, RANGE_CONFIG, RANGE_UPLOAD, RANGE_ATTN, RANGE_UPLOAD_ATTN, with
// F16, Q8_0 and Q4_0 row storage (the rows stay in the layout they arrive in:
// [row][kv head][row bytes], the KV-cache layout the decode kernels read).
// Attention is one xq_attend_range call per request (split-KV partials and the
// LSE merge on the GPU).  The native KVarN4 plane operations, the legacy
// server-compressed attention ops, disk snapshots and profiling answer
// ERR_UNSUPPORTED_OP.
//
// One client at a time, strict request / response.  CUDA is touched only by
// requests that need the GPU (HELLO's memory report degrades to 0 without one).
//
//   xq_rkva_server [--port N] [--device D] [--once]
//     --port 0 picks a free port; the listening port is printed on stdout as
//     "listening <port>".  --once serves one connection and exits.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <signal.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "rkva_wire.h"
#include "xq_b200.h"

namespace {

using clk = std::chrono::steady_clock;
uint64_t us_since(clk::time_point t0) {
    return (uint64_t)std::chrono::duration_cast<std::chrono::microseconds>(clk::now() - t0).count();
}

constexpr uint32_t kMaxPayload = 1u << 30;
constexpr uint32_t kMaxQueries = 1024;

struct Layer {
    void *k = nullptr, *v = nullptr;
    uint32_t rows = 0; // live rows (positions origin .. origin + rows - 1)
};

struct Session {
    uint32_t capacity = 0;
    bool range = false, configured = false;
    uint32_t origin = 0, storage = 0;
    std::vector<Layer> layers;
};

// A device buffer that only grows.
struct DevBuf {
    void *p = nullptr;
    size_t n = 0;
    bool reserve(size_t bytes) {
        if (bytes <= n)
            return true;
        if (p)
            cudaFree(p);
        p = nullptr;
        n = 0;
        if (cudaMalloc(&p, bytes) != cudaSuccess)
            return false;
        n = bytes;
        return true;
    }
    void release() {
        if (p)
            cudaFree(p);
        p = nullptr;
        n = 0;
    }
};

class Server {
public:
    explicit Server(int device) : device_(device) {}
    ~Server() { reset_all(); }

    int32_t handle(const rkva::RkvaRequest &req, const std::vector<uint8_t> &in,
                   std::vector<uint8_t> &out, uint64_t &prepare_us, uint64_t &compute_us);
    void reset_all();

private:
    int32_t hello(const rkva::RkvaRequest &req, const std::vector<uint8_t> &in,
                  std::vector<uint8_t> &out);
    int32_t range_config(const rkva::RkvaRequest &req, const std::vector<uint8_t> &in);
    int32_t upload(Session &s, uint32_t layer, const rkva::RangeUpload &u, const uint8_t *k,
                   const uint8_t *v);
    int32_t attend(Session &s, uint32_t layer, uint32_t n_tokens, const int32_t *positions,
                   const float *q, std::vector<uint8_t> &out, uint64_t &compute_us);
    bool gpu();
    uint64_t row_bytes(const Session &s) const;
    int xq_type(const Session &s) const {
        return s.storage == rkva::kStorageQ8_0   ? XQ_TYPE_Q8_0
               : s.storage == rkva::kStorageQ4_0 ? XQ_TYPE_Q4_0
                                                 : XQ_TYPE_F16;
    }
    uint32_t wire_of(const Session &s) const {
        return s.storage == rkva::kStorageQ8_0   ? rkva::WIRE_Q8_0
               : s.storage == rkva::kStorageQ4_0 ? rkva::WIRE_Q4_0
                                                 : rkva::WIRE_F16;
    }
    void free_session(Session &s);

    int device_;
    bool cuda_ready_ = false;
    cudaStream_t st_ = nullptr;
    bool hello_done_ = false;
    rkva::Hello geo_{};
    std::map<uint32_t, Session> sessions_;
    DevBuf ws_, q_, pos_, o_, lse_;
    uint64_t served_ = 0, uploaded_rows_ = 0, attended_tokens_ = 0;
};

bool Server::gpu() {
    if (cuda_ready_)
        return true;
    if (cudaSetDevice(device_) != cudaSuccess ||
        cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking) != cudaSuccess)
        return false;
    cuda_ready_ = true;
    return true;
}

uint64_t Server::row_bytes(const Session &s) const {
    const uint64_t D = geo_.head_dim;
    const uint64_t rec = s.storage == rkva::kStorageQ8_0   ? D / 32 * 34
                         : s.storage == rkva::kStorageQ4_0 ? D / 32 * 18
                                                           : D * 2;
    return rec * geo_.n_head_kv;
}

void Server::free_session(Session &s) {
    for (Layer &l : s.layers) {
        if (l.k)
            cudaFree(l.k);
        if (l.v)
            cudaFree(l.v);
    }
    s.layers.clear();
    s.configured = false;
}

void Server::reset_all() {
    for (auto &kv : sessions_)
        free_session(kv.second);
    sessions_.clear();
    hello_done_ = false;
    if (cuda_ready_) {
        ws_.release();
        q_.release();
        pos_.release();
        o_.release();
        lse_.release();
    }
}

int32_t Server::hello(const rkva::RkvaRequest &req, const std::vector<uint8_t> &in,
                      std::vector<uint8_t> &out) {
    if (in.size() != sizeof(rkva::Hello))
        return rkva::ERR_BAD_PAYLOAD;
    rkva::Hello h;
    std::memcpy(&h, in.data(), sizeof(h));
    // the geometry the reference server validates, plus row storage only
    // (cache_bits 0 or >= 16: the host ships F16 / Q8_0 / Q4_0 rows)
    if (h.head_dim == 0 || h.n_head == 0 || h.n_head_kv == 0 || h.n_head % h.n_head_kv ||
        h.max_ctx == 0 || (h.head_dim != 128 && h.head_dim != 256) || !h.n_layer_remote ||
        h.n_layer_remote > 128 || h.n_head > 256 || h.n_head_kv > 256 ||
        h.max_ctx > (uint32_t)INT32_MAX || h.has_sinks || h.swa ||
        (h.cache_bits_k != 0 && h.cache_bits_k < 16) || h.domain != 0 ||
        !(h.kq_scale > 0.0f))
        return rkva::ERR_BAD_GEOMETRY;
    reset_all();
    geo_ = h;
    hello_done_ = true;
    rkva::HelloAck ack;
    std::memset(&ack, 0, sizeof(ack));
    const uint16_t ops[] = {rkva::OP_HELLO,        rkva::OP_CREATE_SESSION, rkva::OP_DESTROY_SESSION,
                            rkva::OP_RESET,        rkva::OP_TRIM,           rkva::OP_REWIND,
                            rkva::OP_PING,         rkva::OP_GET_STATS,      rkva::OP_RANGE_CONFIG,
                            rkva::OP_RANGE_UPLOAD, rkva::OP_RANGE_ATTN,     rkva::OP_RANGE_UPLOAD_ATTN};
    for (uint16_t op : ops)
        ack.supported_ops |= 1u << op;
    if (req.version != rkva::kVersion)
        ack.supported_ops &= ~((1u << rkva::OP_RANGE_CONFIG) | (1u << rkva::OP_RANGE_UPLOAD) |
                               (1u << rkva::OP_RANGE_ATTN) | (1u << rkva::OP_RANGE_UPLOAD_ATTN));
    else
        ack.reserved[0] = rkva::kCapRangeQ4_0 | rkva::kCapRangeQ8_0 | rkva::kCapRangeUploadAttn;
    ack.chosen_wire = (h.proto_flags & (1u << rkva::WIRE_F16)) ? rkva::WIRE_F16 : rkva::WIRE_F32;
    ack.max_sessions = 64;
    ack.server_version = 1;
    size_t free_b = 0, total_b = 0;
    if (gpu() && cudaMemGetInfo(&free_b, &total_b) == cudaSuccess)
        ack.mem_budget_bytes = free_b;
    else
        cudaGetLastError();
    out.resize(sizeof(ack));
    std::memcpy(out.data(), &ack, sizeof(ack));
    return rkva::OK;
}

int32_t Server::range_config(const rkva::RkvaRequest &req, const std::vector<uint8_t> &in) {
    if (in.size() != sizeof(rkva::RangeConfig))
        return rkva::ERR_BAD_PAYLOAD;
    auto it = sessions_.find(req.session_id);
    if (it == sessions_.end() || !it->second.range)
        return rkva::ERR_BAD_SESSION;
    Session &s = it->second;
    rkva::RangeConfig c;
    std::memcpy(&c, in.data(), sizeof(c));
    const uint32_t st = c.reserved[0];
    if ((st & ~(rkva::kStorageQ4_0 | rkva::kStorageQ8_0)) ||
        st == (rkva::kStorageQ4_0 | rkva::kStorageQ8_0) || c.reserved[1] ||
        c.capacity != s.capacity || c.origin > (uint32_t)INT32_MAX - c.capacity)
        return rkva::ERR_BAD_POSITION;
    if (!gpu())
        return rkva::ERR_GPU;
    // reissuing CONFIG clears every layer's rows of the session
    free_session(s);
    s.origin = c.origin;
    s.storage = st;
    const uint64_t plane = (uint64_t)s.capacity * row_bytes(s);
    s.layers.resize(geo_.n_layer_remote);
    for (Layer &l : s.layers) {
        if (cudaMalloc(&l.k, plane) != cudaSuccess || cudaMalloc(&l.v, plane) != cudaSuccess) {
            cudaGetLastError();
            free_session(s);
            return rkva::ERR_MEMORY;
        }
    }
    s.configured = true;
    return rkva::OK;
}

int32_t Server::upload(Session &s, uint32_t layer, const rkva::RangeUpload &u, const uint8_t *k,
                       const uint8_t *v) {
    Layer &l = s.layers[layer];
    // start_row 0 replaces the layer's rows; any other start appends exactly
    // at the current row count (uploads leave no gaps)
    if (u.start_row != 0 && u.start_row != l.rows)
        return rkva::ERR_BAD_POSITION;
    const uint64_t rb = row_bytes(s), off = (uint64_t)u.start_row * rb, n = (uint64_t)u.n_rows * rb;
    if (cudaMemcpyAsync(static_cast<uint8_t *>(l.k) + off, k, n, cudaMemcpyHostToDevice, st_) !=
            cudaSuccess ||
        cudaMemcpyAsync(static_cast<uint8_t *>(l.v) + off, v, n, cudaMemcpyHostToDevice, st_) !=
            cudaSuccess ||
        cudaStreamSynchronize(st_) != cudaSuccess) {
        cudaGetLastError();
        return rkva::ERR_GPU;
    }
    l.rows = u.start_row + u.n_rows;
    uploaded_rows_ += u.n_rows;
    return rkva::OK;
}

int32_t Server::attend(Session &s, uint32_t layer, uint32_t n_tokens, const int32_t *positions,
                       const float *q, std::vector<uint8_t> &out, uint64_t &compute_us) {
    Layer &l = s.layers[layer];
    const uint32_t H = geo_.n_head, Hkv = geo_.n_head_kv, D = geo_.head_dim;
    const size_t q_bytes = (size_t)n_tokens * H * D * 4, lse_bytes = (size_t)n_tokens * H * 4;
    const int ty = xq_type(s);
    const size_t ws = xq_attend_range_workspace(ty, n_tokens, l.rows, H, Hkv, D, 4);
    if (!q_.reserve(q_bytes) || !o_.reserve(q_bytes) || !pos_.reserve((size_t)n_tokens * 4) ||
        !lse_.reserve(lse_bytes) || !ws_.reserve(ws > 0 ? ws : 256)) {
        cudaGetLastError();
        return rkva::ERR_MEMORY;
    }
    const auto t0 = clk::now();
    xq_stream_t xs = reinterpret_cast<xq_stream_t>(st_);
    if (cudaMemcpyAsync(q_.p, q, q_bytes, cudaMemcpyHostToDevice, st_) != cudaSuccess ||
        cudaMemcpyAsync(pos_.p, positions, (size_t)n_tokens * 4, cudaMemcpyHostToDevice, st_) !=
            cudaSuccess) {
        cudaGetLastError();
        return rkva::ERR_GPU;
    }
    const int rc = xq_attend_range(ty, l.k, l.v, H, Hkv, D, s.origin, l.rows, n_tokens,
                                   static_cast<const int32_t *>(pos_.p),
                                   static_cast<const float *>(q_.p), geo_.kq_scale, 4,
                                   static_cast<float *>(o_.p), static_cast<float *>(lse_.p), ws_.p,
                                   ws_.n, xs);
    if (rc != XQ_OK) {
        std::fprintf(stderr, "[xq_rkva_server] attend_range: %s\n", xq_last_error());
        return rc == XQ_ERR_CUDA ? rkva::ERR_GPU : rkva::ERR_BAD_PAYLOAD;
    }
    out.resize(q_bytes + lse_bytes);
    if (cudaMemcpyAsync(out.data(), o_.p, q_bytes, cudaMemcpyDeviceToHost, st_) != cudaSuccess ||
        cudaMemcpyAsync(out.data() + q_bytes, lse_.p, lse_bytes, cudaMemcpyDeviceToHost, st_) !=
            cudaSuccess ||
        cudaStreamSynchronize(st_) != cudaSuccess) {
        cudaGetLastError();
        out.clear();
        return rkva::ERR_GPU;
    }
    compute_us = us_since(t0);
    attended_tokens_ += n_tokens;
    return rkva::OK;
}

int32_t Server::handle(const rkva::RkvaRequest &req, const std::vector<uint8_t> &in,
                       std::vector<uint8_t> &out, uint64_t &prepare_us, uint64_t &compute_us) {
    const auto t0 = clk::now();
    ++served_;
    if (req.op >= rkva::OP_RANGE_CONFIG && req.version != rkva::kVersion)
        return rkva::ERR_UNSUPPORTED_OP;
    switch (req.op) {
    case rkva::OP_HELLO:
        return hello(req, in, out);
    case rkva::OP_PING:
        return rkva::OK;
    case rkva::OP_CREATE_SESSION: {
        if (in.size() != sizeof(rkva::SessionReq))
            return rkva::ERR_BAD_PAYLOAD;
        if (!hello_done_)
            return rkva::ERR_STATE;
        rkva::SessionReq r;
        std::memcpy(&r, in.data(), sizeof(r));
        if (req.version == rkva::kVersion && (r.flags & ~rkva::kSessionRange))
            return rkva::ERR_BAD_PAYLOAD;
        auto old = sessions_.find(r.session_id);
        if (old != sessions_.end()) {
            free_session(old->second);
            sessions_.erase(old);
        }
        Session s;
        s.capacity = r.capacity ? r.capacity : geo_.max_ctx;
        s.range = (r.flags & rkva::kSessionRange) != 0;
        sessions_[r.session_id] = s;
        return rkva::OK;
    }
    case rkva::OP_DESTROY_SESSION: {
        auto it = sessions_.find(req.session_id);
        if (it != sessions_.end()) {
            free_session(it->second);
            sessions_.erase(it);
        }
        return rkva::OK;
    }
    case rkva::OP_RESET: {
        auto it = sessions_.find(req.session_id);
        if (it == sessions_.end())
            return rkva::ERR_BAD_SESSION;
        for (Layer &l : it->second.layers)
            l.rows = 0;
        return rkva::OK;
    }
    case rkva::OP_TRIM:
    case rkva::OP_REWIND: {
        if (in.size() != sizeof(rkva::TrimReq))
            return rkva::ERR_BAD_PAYLOAD;
        rkva::TrimReq t;
        std::memcpy(&t, in.data(), sizeof(t));
        auto it = sessions_.find(req.session_id);
        if (it == sessions_.end())
            return rkva::ERR_BAD_SESSION;
        if (t.pos0 < 0)
            return rkva::ERR_BAD_POSITION;
        // every stored position >= pos0 goes: rows keep positions < pos0
        Session &s = it->second;
        const int64_t keep = (int64_t)t.pos0 - (int64_t)s.origin;
        for (Layer &l : s.layers)
            l.rows = keep <= 0 ? 0u : (uint32_t)(keep < (int64_t)l.rows ? keep : (int64_t)l.rows);
        return rkva::OK;
    }
    case rkva::OP_GET_STATS: {
        char buf[512];
        size_t live = 0;
        for (auto &kv : sessions_)
            live += kv.second.configured;
        std::snprintf(buf, sizeof(buf),
                      "{\"service\":\"rkva-range-b200\",\"hello\":%s,\"sessions\":%zu,"
                      "\"configured\":%zu,\"requests\":%llu,\"uploaded_rows\":%llu,"
                      "\"attended_tokens\":%llu}",
                      hello_done_ ? "true" : "false", sessions_.size(), live,
                      (unsigned long long)served_, (unsigned long long)uploaded_rows_,
                      (unsigned long long)attended_tokens_);
        out.assign(buf, buf + std::strlen(buf));
        return rkva::OK;
    }
    case rkva::OP_RANGE_CONFIG:
        return range_config(req, in);
    case rkva::OP_RANGE_UPLOAD: {
        if (in.size() < sizeof(rkva::RangeUpload))
            return rkva::ERR_BAD_PAYLOAD;
        auto it = sessions_.find(req.session_id);
        if (it == sessions_.end() || !it->second.configured)
            return rkva::ERR_BAD_SESSION;
        Session &s = it->second;
        rkva::RangeUpload u;
        std::memcpy(&u, in.data(), sizeof(u));
        if (u.wire != wire_of(s) || u.reserved || !u.n_rows || u.start_row > s.capacity ||
            u.n_rows > s.capacity - u.start_row || req.layer_id >= geo_.n_layer_remote)
            return rkva::ERR_BAD_POSITION;
        const uint64_t plane = (uint64_t)u.n_rows * row_bytes(s);
        if (in.size() != sizeof(u) + 2 * plane)
            return rkva::ERR_BAD_PAYLOAD;
        const uint8_t *k = in.data() + sizeof(u);
        prepare_us = us_since(t0);
        const auto c0 = clk::now();
        const int32_t rc = upload(s, req.layer_id, u, k, k + plane);
        compute_us = us_since(c0);
        return rc;
    }
    case rkva::OP_RANGE_ATTN: {
        if (in.size() < sizeof(rkva::RangeAttn))
            return rkva::ERR_BAD_PAYLOAD;
        auto it = sessions_.find(req.session_id);
        if (it == sessions_.end() || !it->second.configured)
            return rkva::ERR_BAD_SESSION;
        rkva::RangeAttn a;
        std::memcpy(&a, in.data(), sizeof(a));
        if (a.wire != rkva::WIRE_F32 || a.flags || a.reserved[0] || a.reserved[1] ||
            !req.n_tokens || req.n_tokens > kMaxQueries || req.layer_id >= geo_.n_layer_remote)
            return rkva::ERR_BAD_PAYLOAD;
        const uint64_t q_bytes = (uint64_t)req.n_tokens * geo_.n_head * geo_.head_dim * 4;
        if (in.size() != sizeof(a) + (uint64_t)req.n_tokens * 4 + q_bytes)
            return rkva::ERR_BAD_PAYLOAD;
        const int32_t *pos = reinterpret_cast<const int32_t *>(in.data() + sizeof(a));
        for (uint32_t t = 0; t < req.n_tokens; ++t)
            if (pos[t] < 0)
                return rkva::ERR_BAD_POSITION;
        const float *q = reinterpret_cast<const float *>(in.data() + sizeof(a) + req.n_tokens * 4);
        prepare_us = us_since(t0);
        return attend(it->second, req.layer_id, req.n_tokens, pos, q, out, compute_us);
    }
    case rkva::OP_RANGE_UPLOAD_ATTN: {
        if (in.size() < sizeof(rkva::RangeUploadAttn))
            return rkva::ERR_BAD_PAYLOAD;
        auto it = sessions_.find(req.session_id);
        if (it == sessions_.end() || !it->second.configured)
            return rkva::ERR_BAD_SESSION;
        Session &s = it->second;
        rkva::RangeUploadAttn ua;
        std::memcpy(&ua, in.data(), sizeof(ua));
        const rkva::RangeUpload &u = ua.upload;
        const rkva::RangeAttn &a = ua.attention;
        if (u.wire != wire_of(s) || u.reserved || !u.n_rows || u.start_row > s.capacity ||
            u.n_rows > s.capacity - u.start_row || a.wire != rkva::WIRE_F32 || a.flags ||
            a.reserved[0] || a.reserved[1] || !req.n_tokens || req.n_tokens > kMaxQueries ||
            req.layer_id >= geo_.n_layer_remote)
            return rkva::ERR_BAD_PAYLOAD;
        const uint64_t plane = (uint64_t)u.n_rows * row_bytes(s);
        const uint64_t q_bytes = (uint64_t)req.n_tokens * geo_.n_head * geo_.head_dim * 4;
        const uint64_t pos_bytes = (uint64_t)req.n_tokens * 4;
        if (in.size() != sizeof(ua) + 2 * plane + pos_bytes + q_bytes)
            return rkva::ERR_BAD_PAYLOAD;
        const uint8_t *k = in.data() + sizeof(ua), *v = k + plane;
        const int32_t *pos = reinterpret_cast<const int32_t *>(v + plane);
        const float *q = reinterpret_cast<const float *>(v + plane + pos_bytes);
        // the queries are the uploaded chunk's last positions, consecutive,
        // ending at the new last row
        const uint64_t end = (uint64_t)s.origin + u.start_row + u.n_rows;
        for (uint32_t t = 0; t < req.n_tokens; ++t)
            if (pos[t] < (int64_t)s.origin || (uint64_t)pos[t] >= end ||
                (t && pos[t] != pos[t - 1] + 1))
                return rkva::ERR_BAD_POSITION;
        if ((uint64_t)pos[req.n_tokens - 1] + 1 != end)
            return rkva::ERR_BAD_POSITION;
        prepare_us = us_since(t0);
        int32_t rc = upload(s, req.layer_id, u, k, v);
        if (rc != rkva::OK)
            return rc;
        return attend(s, req.layer_id, req.n_tokens, pos, q, out, compute_us);
    }
    default:
        return rkva::ERR_UNSUPPORTED_OP;
    }
}

bool read_all(int fd, void *buf, size_t n) {
    uint8_t *p = static_cast<uint8_t *>(buf);
    while (n) {
        const ssize_t r = recv(fd, p, n, 0);
        if (r <= 0)
            return false;
        p += r;
        n -= (size_t)r;
    }
    return true;
}

bool write_all(int fd, const void *buf, size_t n) {
    const uint8_t *p = static_cast<const uint8_t *>(buf);
    while (n) {
        const ssize_t r = send(fd, p, n, MSG_NOSIGNAL);
        if (r <= 0)
            return false;
        p += r;
        n -= (size_t)r;
    }
    return true;
}

void client_loop(int fd, Server &server) {
    std::vector<uint8_t> in, out;
    uint64_t last_response_us = 0;
    for (;;) {
        rkva::RkvaRequest req;
        if (!read_all(fd, &req, sizeof(req)))
            return;
        rkva::RkvaResponse rsp;
        std::memset(&rsp, 0, sizeof(rsp));
        rsp.magic = rkva::kMagic;
        rsp.version = rkva::kVersion;
        rsp.op = req.op;
        rsp.cycle_id = req.cycle_id;
        if (req.magic != rkva::kMagic ||
            (req.version != rkva::kVersion && req.version != rkva::kVersionLegacy) ||
            req.payload_bytes > kMaxPayload) {
            // a frame this server cannot parse: report it and drop the connection
            rsp.status = rkva::ERR_PROTOCOL;
            write_all(fd, &rsp, sizeof(rsp));
            return;
        }
        const auto r0 = clk::now();
        in.resize(req.payload_bytes);
        if (req.payload_bytes && !read_all(fd, in.data(), req.payload_bytes))
            return;
        rsp.receive_us = us_since(r0);
        out.clear();
        uint64_t prepare_us = 0, compute_us = 0;
        rsp.status = server.handle(req, in, out, prepare_us, compute_us);
        if (rsp.status != rkva::OK)
            out.clear();
        rsp.payload_bytes = (uint32_t)out.size();
        rsp.prepare_us = prepare_us;
        rsp.compute_us = compute_us;
        rsp.response_us = last_response_us;
        const auto s0 = clk::now();
        if (!write_all(fd, &rsp, sizeof(rsp)) || (!out.empty() && !write_all(fd, out.data(), out.size())))
            return;
        last_response_us = us_since(s0);
    }
}

} // namespace

int main(int argc, char **argv) {
    int port = 50054, device = 0;
    bool once = false;
    for (int i = 1; i < argc; ++i) {
        if (!std::strcmp(argv[i], "--port") && i + 1 < argc)
            port = std::atoi(argv[++i]);
        else if (!std::strcmp(argv[i], "--device") && i + 1 < argc)
            device = std::atoi(argv[++i]);
        else if (!std::strcmp(argv[i], "--once"))
            once = true;
        else {
            std::fprintf(stderr, "usage: %s [--port N] [--device D] [--once]\n", argv[0]);
            return 2;
        }
    }
    signal(SIGPIPE, SIG_IGN);
    const int ls = socket(AF_INET, SOCK_STREAM, 0);
    if (ls < 0) {
        std::perror("socket");
        return 1;
    }
    const int one = 1;
    setsockopt(ls, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in addr;
    std::memset(&addr, 0, sizeof(addr));
    addr.sin_family = AF_INET;
    addr.sin_addr.s_addr = htonl(INADDR_ANY);
    addr.sin_port = htons((uint16_t)port);
    if (bind(ls, reinterpret_cast<sockaddr *>(&addr), sizeof(addr)) < 0 || listen(ls, 1) < 0) {
        std::perror("bind/listen");
        close(ls);
        return 1;
    }
    socklen_t len = sizeof(addr);
    getsockname(ls, reinterpret_cast<sockaddr *>(&addr), &len);
    std::printf("listening %d\n", (int)ntohs(addr.sin_port));
    std::fflush(stdout);
    Server server(device);
    for (;;) {
        const int fd = accept(ls, nullptr, nullptr);
        if (fd < 0)
            break;
        setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
        server.reset_all(); // a new connection starts from HELLO, as the reference's does
        client_loop(fd, server);
        close(fd);
        server.reset_all();
        if (once)
            break;
    }
    close(ls);
    return 0;
}
