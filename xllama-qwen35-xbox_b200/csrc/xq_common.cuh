// Shared device helpers for the B200 attention kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "xq_b200.h"

namespace xq {

constexpr int kF32 = XQ_TYPE_F32;
constexpr int kF16 = XQ_TYPE_F16;
constexpr int kQ8 = XQ_TYPE_Q8_0;
constexpr int kQ4 = XQ_TYPE_Q4_0;

// Bytes of one row of D elements in a ggml type.
__host__ __device__ constexpr int rec_bytes(int type, int D) {
    return type == kF16 ? 2 * D : type == kQ8 ? D / 32 * 34 : type == kQ4 ? D / 32 * 18 : 4 * D;
}

// Shared-memory row stride: a multiple of 16 bytes with an odd count of
// 16-byte units, so rows read by neighbouring lanes start in different banks.
__host__ __device__ constexpr int smem_stride(int rec) {
    return ((rec + 15) / 16) % 2 == 0 ? (rec + 15) / 16 * 16 + 16 : (rec + 15) / 16 * 16;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Asynchronous global -> shared copy of VW bytes (LDGSTS).  16-byte copies
// bypass L1 (.cg): the KV stream is read once.
template <int VW>
__device__ __forceinline__ void cp_async(uint32_t dst, const void *src) {
    if constexpr (VW == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
    else if constexpr (VW == 8)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src));
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ float h2f_bits(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// Dequantise dims 4c..4c+3 of one row held in shared memory, exactly as
// ggml's to_float does (F16 -> F32; Q8_0: int8 * f32(d); Q4_0: (nibble - 8) *
// f32(d), low nibbles are elements 0..15 of a block, high nibbles 16..31).
// Each product of an integer of <= 8 bits and an fp16 scale is exact in fp32.
template <int T>
__device__ __forceinline__ void load4(const uint8_t *row, int c, float (&x)[4]);

template <>
__device__ __forceinline__ void load4<kF16>(const uint8_t *row, int c, float (&x)[4]) {
    const uint2 w = *reinterpret_cast<const uint2 *>(row + 8 * c);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
    x[0] = a.x;
    x[1] = a.y;
    x[2] = b.x;
    x[3] = b.y;
}

template <>
__device__ __forceinline__ void load4<kQ8>(const uint8_t *row, int c, float (&x)[4]) {
    const uint8_t *blk = row + 34 * (c >> 3);
    const float d = h2f_bits(*reinterpret_cast<const uint16_t *>(blk));
    const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2 + 4 * (c & 7));
    const uint32_t w = (uint32_t)p[0] | ((uint32_t)p[1] << 16);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        x[i] = (float)(int)(int8_t)(w >> (8 * i)) * d;
}

template <>
__device__ __forceinline__ void load4<kQ4>(const uint8_t *row, int c, float (&x)[4]) {
    const uint8_t *blk = row + 18 * (c >> 3);
    const float d = h2f_bits(*reinterpret_cast<const uint16_t *>(blk));
    const int o = 4 * (c & 7);
    const uint16_t *p = reinterpret_cast<const uint16_t *>(blk + 2 + (o & 15));
    const uint32_t w = ((uint32_t)p[0] | ((uint32_t)p[1] << 16)) >> ((o & 16) ? 4 : 0);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        x[i] = (float)((int)((w >> (8 * i)) & 15u) - 8) * d;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

} // namespace xq
