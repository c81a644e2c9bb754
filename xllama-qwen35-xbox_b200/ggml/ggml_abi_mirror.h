// Local stand-in for the ggml declarations the XQ_B200 backend uses, for
// builds outside the llama.cpp fork (this repository's self-tests).
//
// A real integration compiles ggml_xq_backend.cpp with -DXQ_GGML_REAL and the
// fork's ggml/include + ggml/src on the include path, so every struct layout,
// enum value and function below comes from the fork's own ggml.h,
// ggml-backend.h and ggml-backend-impl.h.  The layouts here follow upstream
// ggml with the fork's two extra 2-D tensor slots in the buffer and backend
// interfaces (the reference's vtables, src/bridge/ggml_d3d12.cpp:1371-1383 and
// :2268-2285, list them).  The op and type enum VALUES of this mirror are
// placeholders for the self-test harness only; the type ids match ggml.
#pragma once

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_MAX_DIMS 4
#define GGML_MAX_OP_PARAMS 64
#define GGML_MAX_SRC 10
#define GGML_MAX_NAME 64
#define GGML_BACKEND_API_VERSION 2

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_I32 = 26,
    GGML_TYPE_I64 = 27,
};

enum ggml_op {
    GGML_OP_NONE = 0,
    GGML_OP_RESHAPE = 36,
    GGML_OP_VIEW = 37,
    GGML_OP_PERMUTE = 38,
    GGML_OP_TRANSPOSE = 39,
    GGML_OP_SET_ROWS = 41,
    GGML_OP_FLASH_ATTN_EXT = 72,
    GGML_OP_GATED_DELTA_NET = 84,
};

enum ggml_status {
    GGML_STATUS_ALLOC_FAILED = -2,
    GGML_STATUS_FAILED = -1,
    GGML_STATUS_SUCCESS = 0,
    GGML_STATUS_ABORTED = 1,
};

enum ggml_tensor_flag {
    GGML_TENSOR_FLAG_INPUT = 1,
    GGML_TENSOR_FLAG_OUTPUT = 2,
    GGML_TENSOR_FLAG_PARAM = 4,
    GGML_TENSOR_FLAG_LOSS = 8,
    GGML_TENSOR_FLAG_COMPUTE = 16,
};

struct ggml_backend_buffer;

struct ggml_tensor {
    enum ggml_type type;
    struct ggml_backend_buffer *buffer;
    int64_t ne[GGML_MAX_DIMS];
    size_t nb[GGML_MAX_DIMS];
    enum ggml_op op;
    int32_t op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)];
    int32_t flags;
    struct ggml_tensor *src[GGML_MAX_SRC];
    struct ggml_tensor *view_src;
    size_t view_offs;
    void *data;
    char name[GGML_MAX_NAME];
    void *extra;
    char padding[8];
};

struct ggml_cgraph;
typedef uint8_t ggml_guid[16];
typedef ggml_guid *ggml_guid_t;

typedef struct ggml_backend_buffer_type *ggml_backend_buffer_type_t;
typedef struct ggml_backend_buffer *ggml_backend_buffer_t;
typedef struct ggml_backend *ggml_backend_t;
typedef struct ggml_backend_event *ggml_backend_event_t;
typedef struct ggml_backend_device *ggml_backend_dev_t;
typedef struct ggml_backend_reg *ggml_backend_reg_t;
typedef void *ggml_backend_graph_plan_t;

enum ggml_backend_buffer_usage {
    GGML_BACKEND_BUFFER_USAGE_ANY = 0,
    GGML_BACKEND_BUFFER_USAGE_WEIGHTS = 1,
    GGML_BACKEND_BUFFER_USAGE_COMPUTE = 2,
};

enum ggml_backend_dev_type {
    GGML_BACKEND_DEVICE_TYPE_CPU,
    GGML_BACKEND_DEVICE_TYPE_GPU,
    GGML_BACKEND_DEVICE_TYPE_IGPU,
    GGML_BACKEND_DEVICE_TYPE_ACCEL,
};

struct ggml_backend_dev_caps {
    bool async;
    bool host_buffer;
    bool buffer_from_host_ptr;
    bool events;
};

struct ggml_backend_dev_props {
    const char *name;
    const char *description;
    size_t memory_free;
    size_t memory_total;
    enum ggml_backend_dev_type type;
    const char *device_id;
    struct ggml_backend_dev_caps caps;
};

struct ggml_backend_buffer_type_i {
    const char *(*get_name)(ggml_backend_buffer_type_t buft);
    ggml_backend_buffer_t (*alloc_buffer)(ggml_backend_buffer_type_t buft, size_t size);
    size_t (*get_alignment)(ggml_backend_buffer_type_t buft);
    size_t (*get_max_size)(ggml_backend_buffer_type_t buft);
    size_t (*get_alloc_size)(ggml_backend_buffer_type_t buft, const struct ggml_tensor *tensor);
    bool (*is_host)(ggml_backend_buffer_type_t buft);
};

struct ggml_backend_buffer_type {
    struct ggml_backend_buffer_type_i iface;
    ggml_backend_dev_t device;
    void *context;
};

struct ggml_backend_buffer_i {
    void (*free_buffer)(ggml_backend_buffer_t buffer);
    void *(*get_base)(ggml_backend_buffer_t buffer);
    enum ggml_status (*init_tensor)(ggml_backend_buffer_t buffer, struct ggml_tensor *tensor);
    void (*memset_tensor)(ggml_backend_buffer_t buffer, struct ggml_tensor *tensor, uint8_t value,
                          size_t offset, size_t size);
    void (*set_tensor)(ggml_backend_buffer_t buffer, struct ggml_tensor *tensor, const void *data,
                       size_t offset, size_t size);
    void (*get_tensor)(ggml_backend_buffer_t buffer, const struct ggml_tensor *tensor, void *data,
                       size_t offset, size_t size);
    // fork slots: n_copies rows of `size` bytes, row i at tensor offset
    // offset + i * stride_tensor and at data + i * stride_data
    void (*set_tensor_2d)(ggml_backend_buffer_t buffer, struct ggml_tensor *tensor,
                          const void *data, size_t offset, size_t size, size_t n_copies,
                          size_t stride_tensor, size_t stride_data);
    void (*get_tensor_2d)(ggml_backend_buffer_t buffer, const struct ggml_tensor *tensor,
                          void *data, size_t offset, size_t size, size_t n_copies,
                          size_t stride_tensor, size_t stride_data);
    bool (*cpy_tensor)(ggml_backend_buffer_t buffer, const struct ggml_tensor *src,
                       struct ggml_tensor *dst);
    void (*clear)(ggml_backend_buffer_t buffer, uint8_t value);
    void (*reset)(ggml_backend_buffer_t buffer);
};

struct ggml_backend_buffer {
    struct ggml_backend_buffer_i iface;
    ggml_backend_buffer_type_t buft;
    void *context;
    size_t size;
    enum ggml_backend_buffer_usage usage;
};

struct ggml_backend_i {
    const char *(*get_name)(ggml_backend_t backend);
    void (*free)(ggml_backend_t backend);
    void (*set_tensor_async)(ggml_backend_t backend, struct ggml_tensor *tensor, const void *data,
                             size_t offset, size_t size);
    void (*get_tensor_async)(ggml_backend_t backend, const struct ggml_tensor *tensor, void *data,
                             size_t offset, size_t size);
    void (*set_tensor_2d_async)(ggml_backend_t backend, struct ggml_tensor *tensor,
                                const void *data, size_t offset, size_t size, size_t n_copies,
                                size_t stride_tensor, size_t stride_data);
    void (*get_tensor_2d_async)(ggml_backend_t backend, const struct ggml_tensor *tensor,
                                void *data, size_t offset, size_t size, size_t n_copies,
                                size_t stride_tensor, size_t stride_data);
    bool (*cpy_tensor_async)(ggml_backend_t backend_src, ggml_backend_t backend_dst,
                             const struct ggml_tensor *src, struct ggml_tensor *dst);
    void (*synchronize)(ggml_backend_t backend);
    ggml_backend_graph_plan_t (*graph_plan_create)(ggml_backend_t backend,
                                                   const struct ggml_cgraph *cgraph);
    void (*graph_plan_free)(ggml_backend_t backend, ggml_backend_graph_plan_t plan);
    void (*graph_plan_update)(ggml_backend_t backend, ggml_backend_graph_plan_t plan,
                              const struct ggml_cgraph *cgraph);
    enum ggml_status (*graph_plan_compute)(ggml_backend_t backend, ggml_backend_graph_plan_t plan);
    enum ggml_status (*graph_compute)(ggml_backend_t backend, struct ggml_cgraph *cgraph);
    void (*event_record)(ggml_backend_t backend, ggml_backend_event_t event);
    void (*event_wait)(ggml_backend_t backend, ggml_backend_event_t event);
    void (*graph_optimize)(ggml_backend_t backend, struct ggml_cgraph *cgraph);
};

struct ggml_backend {
    ggml_guid_t guid;
    struct ggml_backend_i iface;
    ggml_backend_dev_t device;
    void *context;
};

struct ggml_backend_device_i {
    const char *(*get_name)(ggml_backend_dev_t dev);
    const char *(*get_description)(ggml_backend_dev_t dev);
    void (*get_memory)(ggml_backend_dev_t dev, size_t *free, size_t *total);
    enum ggml_backend_dev_type (*get_type)(ggml_backend_dev_t dev);
    void (*get_props)(ggml_backend_dev_t dev, struct ggml_backend_dev_props *props);
    ggml_backend_t (*init_backend)(ggml_backend_dev_t dev, const char *params);
    ggml_backend_buffer_type_t (*get_buffer_type)(ggml_backend_dev_t dev);
    ggml_backend_buffer_type_t (*get_host_buffer_type)(ggml_backend_dev_t dev);
    ggml_backend_buffer_t (*buffer_from_host_ptr)(ggml_backend_dev_t dev, void *ptr, size_t size,
                                                  size_t max_tensor_size);
    bool (*supports_op)(ggml_backend_dev_t dev, const struct ggml_tensor *op);
    bool (*supports_buft)(ggml_backend_dev_t dev, ggml_backend_buffer_type_t buft);
    bool (*offload_op)(ggml_backend_dev_t dev, const struct ggml_tensor *op);
    ggml_backend_event_t (*event_new)(ggml_backend_dev_t dev);
    void (*event_free)(ggml_backend_dev_t dev, ggml_backend_event_t event);
    void (*event_synchronize)(ggml_backend_dev_t dev, ggml_backend_event_t event);
};

struct ggml_backend_device {
    struct ggml_backend_device_i iface;
    ggml_backend_reg_t reg;
    void *context;
};

struct ggml_backend_event {
    struct ggml_backend_device *device;
    void *context;
};

struct ggml_backend_reg_i {
    const char *(*get_name)(ggml_backend_reg_t reg);
    size_t (*get_device_count)(ggml_backend_reg_t reg);
    ggml_backend_dev_t (*get_device)(ggml_backend_reg_t reg, size_t index);
    void *(*get_proc_address)(ggml_backend_reg_t reg, const char *name);
};

struct ggml_backend_reg {
    int api_version;
    struct ggml_backend_reg_i iface;
    void *context;
};

// ggml functions the backend calls (provided by libggml-base in the fork).
ggml_backend_buffer_t ggml_backend_buffer_init(ggml_backend_buffer_type_t buft,
                                               struct ggml_backend_buffer_i iface, void *context,
                                               size_t size);
void ggml_backend_register(ggml_backend_reg_t reg);
int ggml_graph_n_nodes(struct ggml_cgraph *cgraph);
size_t ggml_nbytes(const struct ggml_tensor *tensor);
struct ggml_tensor *ggml_graph_node(struct ggml_cgraph *cgraph, int i);

#ifdef __cplusplus
}
#endif
