// Wire format of the RKVA remote-attention protocol, v2 range subset, as the
// reference's host sends it (uwp/rkva/remote-attn-protocol.h:14-236).  The
// byte layouts are an interface the host already speaks, so every struct here
// reproduces the reference's field order and size exactly (checked by the
// static_asserts); names and comments are this project's own.
//
// Framing: one TCP connection, strictly alternating request / response.  A
// request is RkvaRequest (32 bytes) + payload_bytes of payload; a response is
// RkvaResponse (56 bytes) + payload_bytes of payload.  Little endian.
#pragma once

#include <cstdint>

namespace rkva {

constexpr uint32_t kMagic = 0x41564B52u; // "RKVA" little endian
constexpr uint16_t kVersion = 2;         // range operations need it
constexpr uint16_t kVersionLegacy = 1;

// Operation codes (the request's `op`).
enum Op : uint16_t {
    OP_HELLO = 1,
    OP_CREATE_SESSION = 2,
    OP_DESTROY_SESSION = 3,
    OP_ATTN_DECODE = 4,
    OP_ATTN_PREFILL = 5,
    OP_RESET = 6,
    OP_TRIM = 7,
    OP_REWIND = 8,
    OP_PING = 9,
    OP_GET_STATS = 10,
    OP_PROBE = 11,
    OP_RANGE_CONFIG = 12,
    OP_RANGE_UPLOAD = 13,
    OP_RANGE_ATTN = 14,
    OP_KVARN_RANGE_CONFIG = 15,
    OP_KVARN_RANGE_UPLOAD = 16,
    OP_SNAPSHOT_SAVE = 17,
    OP_SNAPSHOT_RESTORE = 18,
    OP_RANGE_UPLOAD_ATTN = 19,
    OP_RANGE_PROFILE = 20,
    OP_KVARN_RANGE_REWIND = 21,
    OP_KVARN_RANGE_BULK_ATTN = 22,
};

// Element encodings of payload planes.
enum Wire : uint32_t {
    WIRE_F16 = 0,
    WIRE_F32 = 1,
    WIRE_Q4_0 = 2, // ggml block_q4_0: f16 scale + 16 nibble bytes per 32 values
    WIRE_Q8_0 = 3, // ggml block_q8_0: f16 scale + 32 int8 per 32 values
};

// Response status.
enum Status : int32_t {
    OK = 0,
    ERR_PROTOCOL = -1,
    ERR_UNSUPPORTED_OP = -2,
    ERR_BAD_SESSION = -3,
    ERR_BAD_GEOMETRY = -4,
    ERR_MEMORY = -5,
    ERR_GPU = -6,
    ERR_BAD_POSITION = -7,
    ERR_BAD_PAYLOAD = -8,
    ERR_STATE = -9,
};

// Capability bits of HelloAck::reserved[0], range-storage bits of
// RangeConfig::reserved[0], session flag of SessionReq::flags.
constexpr uint64_t kCapRangeQ4_0 = 1ull << 0;
constexpr uint64_t kCapRangeQ8_0 = 1ull << 1;
constexpr uint64_t kCapRangeUploadAttn = 1ull << 4;
constexpr uint32_t kStorageQ4_0 = 1u << 0;
constexpr uint32_t kStorageQ8_0 = 1u << 1;
constexpr uint32_t kSessionRange = 1u << 0;
constexpr uint32_t kSessionNone = 0xFFFFFFFFu;

#pragma pack(push, 1)

struct RkvaRequest {
    uint32_t magic;
    uint16_t version;
    uint16_t op;
    uint64_t cycle_id;
    uint32_t session_id;
    uint32_t layer_id; // 0 .. n_layer_remote - 1
    uint32_t n_tokens;
    uint32_t payload_bytes;
};

struct RkvaResponse {
    uint32_t magic;
    uint16_t version;
    uint16_t op;
    uint64_t cycle_id;
    int32_t status;
    uint32_t payload_bytes;
    uint64_t receive_us; // payload receive time
    uint64_t prepare_us; // validation + staging
    uint64_t compute_us; // GPU work
    uint64_t response_us; // previous response's send time
};

struct Hello {
    uint32_t proto_flags;
    uint32_t n_layer_remote;
    uint32_t n_head;
    uint32_t n_head_kv;
    uint32_t head_dim;
    uint32_t max_ctx;
    uint32_t cache_bits_k; // 0 or >= 16: row (F16 / Q8_0 / Q4_0) storage
    uint32_t cache_bits_v;
    uint32_t group_tokens;
    uint32_t sinkhorn_iters;
    uint32_t tail_tokens;
    uint32_t tail_groups;
    uint32_t tail_type;
    uint32_t domain; // 0: automatic (the only domain range sessions take)
    uint32_t has_sinks;
    uint32_t swa;
    float kq_scale;
    uint64_t reserved[2];
};

struct HelloAck {
    uint32_t supported_ops; // bit op set for every op served
    uint32_t chosen_wire;
    uint32_t max_sessions;
    uint32_t server_version;
    uint64_t mem_budget_bytes;
    uint64_t reserved[2]; // [0]: capability bits
};

struct SessionReq {
    uint32_t session_id;
    uint32_t seq_id;
    uint32_t capacity; // rows; 0: the HELLO's max_ctx
    uint32_t flags;    // kSessionRange
};

struct TrimReq {
    int32_t pos0; // remove every position >= pos0
};

struct RangeConfig {
    uint32_t origin;   // absolute position of compact row 0
    uint32_t capacity; // compact rows (must equal the session's)
    uint32_t reserved[2]; // [0]: storage bits (0 = F16), [1] = 0
};

struct RangeUpload {
    uint32_t start_row; // 0 replaces the layer's rows; else appends at the row count
    uint32_t n_rows;
    uint32_t wire;      // the session's storage encoding
    uint32_t reserved;
};

struct RangeAttn {
    uint32_t wire;  // WIRE_F32
    uint32_t flags; // 0
    uint32_t reserved[2];
};

struct RangeUploadAttn {
    RangeUpload upload;
    RangeAttn attention;
};

#pragma pack(pop)

static_assert(sizeof(RkvaRequest) == 32, "request header");
static_assert(sizeof(RkvaResponse) == 56, "response header");
static_assert(sizeof(Hello) == 84, "hello");
static_assert(sizeof(HelloAck) == 40, "hello ack");
static_assert(sizeof(SessionReq) == 16, "session request");
static_assert(sizeof(TrimReq) == 4, "trim request");
static_assert(sizeof(RangeConfig) == 16, "range config");
static_assert(sizeof(RangeUpload) == 16, "range upload");
static_assert(sizeof(RangeAttn) == 16, "range attention");
static_assert(sizeof(RangeUploadAttn) == 32, "range upload + attention");

} // namespace rkva
