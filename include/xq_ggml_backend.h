/*
 * xq_ggml_backend.h -- the B200 attention path as a ggml backend
 * (libxq_ggml_b200.so).
 *
 * A ggml backend named "XQ_B200" whose devices are the process's CUDA GPUs.
 * Its supports_op claims exactly GGML_OP_FLASH_ATTN_EXT and
 * GGML_OP_GATED_DELTA_NET (plus the no-op view ops), so llama.cpp's graph
 * scheduler routes those two ops here and keeps everything else where it was.
 * graph_compute calls the C ABI of include/xq_b200.h on one CUDA stream per
 * backend; synchronize waits for it.
 *
 * Replaces the reference's ggml backend registration
 * ggml_d3d12_register() (src/bridge/ggml_d3d12.cpp:2498-2513), built from the
 * same ggml vtables (reg :2473-2478, device :2427-2446, backend :2268-2285,
 * buffer :1371-1383, buffer type :1516-1527).
 */
#ifndef XQ_GGML_BACKEND_H
#define XQ_GGML_BACKEND_H

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct ggml_backend;
struct ggml_backend_reg;
struct ggml_tensor;

/* The backend registry ("XQ_B200"); one device per visible CUDA GPU. */
struct ggml_backend_reg *ggml_backend_xq_b200_reg(void);

/* ggml_backend_register() of the registry, once per process.  False when no
 * CUDA device is visible (nothing is registered then). */
bool ggml_xq_b200_register(void);

/* The predicate behind the device's supports_op (pure host logic). */
bool ggml_xq_b200_supports_op(const struct ggml_tensor *op);

/* GPU time per op of one XQ_B200 backend created with XQ_GGML_TIMING=1 in the
 * environment: CUDA events around every node on the backend's stream, read
 * back as they complete (all of them at synchronize); op 0 FLASH_ATTN_EXT,
 * 1 GATED_DELTA_NET, 2 SET_ROWS.  nodes = timed nodes, ms = their summed GPU
 * time, untimed = nodes whose events failed.  The totals are also printed to
 * stderr when the backend is freed.  Every node also gets an NVTX range named
 * after its op.  Replaces the reference backend's GPU timestamp accounting
 * (src/bridge/ggml_d3d12.cpp:1897-1903, 2148-2151, 2202-2221).  False for
 * another backend, an op index outside 0..2 or a backend without timing. */
bool ggml_xq_b200_backend_op_time(struct ggml_backend *backend, int op, uint64_t *nodes,
                                  double *ms, uint64_t *untimed);

#ifdef __cplusplus
}
#endif
#endif /* XQ_GGML_BACKEND_H */
