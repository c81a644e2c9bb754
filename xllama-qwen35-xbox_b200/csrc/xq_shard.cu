// KV-sharded decode across GPUs: the exchange of per-group (O, lse) records
// over NVLink with plain peer stores, one process per GPU.
//
// The reference splits one sequence's KV cache by position between two
// devices and merges their (O, LSE) partials on the host
// (uwp/rkva/remote-attn-engine.cpp:2928-2978, the RANGE_ATTN reply of
// uwp/rkva/remote-attn-protocol.h:205-236).  Here every GPU holds a block of
// fixed global split groups; each step a rank merges each of its groups into
// one record, stores the records into every rank's exchange buffer (NVLink
// peer stores into IPC-mapped memory, no TMA, no multicast), and merges all
// groups' records in group order once they have all arrived.
//
// Exchange buffer of one rank (library-allocated, zeroed once):
//   [2][n_groups][n_rows][D + 2] f32 records   (half = step parity)
//   [2] u32 arrival counters, u32 error word    (256-byte aligned)
// A pushing CTA stores one chunk of its records into one receiver, fences at
// system scope and adds one arrival to that receiver's counter of the step's
// half.  The receiver's wait kernel spins (bounded by %globaltimer) until the
// count of every rank's chunks is there, then resets the counter.  A rank
// writes half b again only at step t + 2, after every peer's step t + 1
// records reached it -- which each peer pushes after its own step-t merge --
// so a half is never overwritten while it is being merged.
#include <float.h>
#include <stdint.h>

#include "xq_common.cuh"
#include "xq_internal.h"

namespace xq {

namespace sh {
constexpr int NT = 256;
constexpr int64_t CHUNK8 = 2048; // 8-byte units per pushing CTA (16 KB)
constexpr unsigned long long WAIT_NS = 2000000000ull; // 2 s
} // namespace sh

size_t shard_records_bytes(int64_t n_groups, int64_t n_rows, int D) {
    return (size_t)n_groups * n_rows * (D + 2) * sizeof(float);
}

size_t shard_exchange_bytes(int64_t n_groups, int64_t n_rows, int D) {
    return (2 * shard_records_bytes(n_groups, n_rows, D) + 255) / 256 * 256 + 256;
}

static size_t ctl_off(int64_t n_groups, int64_t n_rows, int D) {
    return (2 * shard_records_bytes(n_groups, n_rows, D) + 255) / 256 * 256;
}

int64_t shard_chunks(size_t bytes) {
    const int64_t n8 = (int64_t)(bytes / 8);
    return (n8 + sh::CHUNK8 - 1) / sh::CHUNK8;
}

// Grid (chunks, world): CTA (c, p) copies 8-byte units [c CHUNK8, ...) of this
// rank's records into receiver p's half at unit offset dst_off8, then adds one
// arrival to p's counter of that half.  Launched as a programmatic dependent
// of the record merge: the records are read after griddepcontrol.wait.
__global__ void __launch_bounds__(sh::NT) shard_push_kernel(ShardPushArgs a) {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    const int64_t c = blockIdx.x;
    const int p = (int)blockIdx.y;
    uint8_t *peer = a.peers[p];
    float2 *dst = reinterpret_cast<float2 *>(peer + a.half_off) + a.dst_off8;
    const int64_t lo = c * sh::CHUNK8, hi = min(a.n8, lo + sh::CHUNK8);
    for (int64_t i = lo + threadIdx.x; i < hi; i += sh::NT)
        dst[i] = __ldcg(a.src + i);
    __threadfence_system(); // this thread's stores reach the receiver ...
    __syncthreads();        // ... before the CTA's arrival
    if (threadIdx.x == 0)
        atomicAdd_system(reinterpret_cast<unsigned *>(peer + a.ctl_off) + a.parity, 1u);
}

// One CTA: wait until `expected` arrivals are counted in this rank's counter
// of the half (bounded), reset it; on timeout record the error and poison the
// half's records with NaN so that the merge after this kernel yields NaN.
__global__ void __launch_bounds__(sh::NT) shard_wait_kernel(uint8_t *ex, size_t ctl, int parity,
                                                            unsigned expected, float *half,
                                                            int64_t half_floats) {
    __shared__ int ok_s;
    volatile unsigned *cnt = reinterpret_cast<volatile unsigned *>(ex + ctl) + parity;
    if (threadIdx.x == 0) {
        uint64_t t0, t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
        int ok = 1;
        while (*cnt < expected) {
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > sh::WAIT_NS) {
                ok = 0;
                break;
            }
            __nanosleep(256);
        }
        __threadfence_system();
        ok_s = ok;
    }
    __syncthreads();
    if (!ok_s) {
        for (int64_t i = threadIdx.x; i < half_floats; i += sh::NT)
            half[i] = NAN;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0)
            atomicExch(reinterpret_cast<unsigned *>(ex + ctl) + 2, 1u);
    }
    if (threadIdx.x == 0)
        *cnt = 0u;
}

cudaError_t launch_shard_push(const ShardPushArgs &a, int world, cudaStream_t st) {
    const int64_t chunks = (a.n8 + sh::CHUNK8 - 1) / sh::CHUNK8;
    if (chunks <= 0)
        return cudaSuccess;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)chunks, (unsigned)world, 1);
    cfg.blockDim = dim3(sh::NT, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, shard_push_kernel, a);
}

cudaError_t launch_shard_wait(void *exchange, int64_t n_groups, int64_t n_rows, int D,
                              int parity, unsigned expected, cudaStream_t st) {
    uint8_t *ex = static_cast<uint8_t *>(exchange);
    const size_t ctl = ctl_off(n_groups, n_rows, D);
    const int64_t half_floats = n_groups * n_rows * (D + 2);
    float *half = reinterpret_cast<float *>(ex) + (int64_t)parity * half_floats;
    shard_wait_kernel<<<1, sh::NT, 0, st>>>(ex, ctl, parity, expected, half, half_floats);
    return cudaGetLastError();
}

size_t shard_ctl_off(int64_t n_groups, int64_t n_rows, int D) {
    return ctl_off(n_groups, n_rows, D);
}

} // namespace xq
