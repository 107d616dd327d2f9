// common.cuh -- shared definitions of the B200 routed-expert library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace moeb200 {

// ggml type ids (reference cpp/dequant_k.cpp:37-41).
enum : int { Q8_0 = 8, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14 };

// Status codes.  -1..-5 keep the reference's meaning
// (cpp/moe_quant_dot.cpp:181-212); -6.. are device-side conditions the
// reference cannot have.
enum : int {
    ST_OK = 0,
    ST_ARG = -1,        // null pointer, bad size or flag
    ST_TYPE = -2,       // unsupported type or columns not a block multiple
    ST_BYTES = -3,      // tensor byte count does not match its shape
    ST_NONFINITE = -4,  // an output is NaN or infinite
    ST_INTERNAL = -5,   // allocation or other host-side failure
    ST_CUDA = -6,       // a CUDA call failed (see moe_b200_last_cuda_error)
    ST_ALIGN = -7,      // a device pointer is not 16-byte aligned
    ST_WORKSPACE = -8,  // workspace too small
    ST_TIMEOUT = -9,    // a bounded device-side wait gave up
    ST_RANGE = -10,     // a prefill activation outside the fp16 range
};

__host__ __device__ constexpr int block_size(int t) {
    return t == Q8_0 ? 32 : (t == Q3_K || t == Q4_K || t == Q5_K || t == Q6_K) ? 256 : 0;
}

__host__ __device__ constexpr int block_bytes(int t) {
    return t == Q8_0 ? 34 : t == Q3_K ? 110 : t == Q4_K ? 144 : t == Q5_K ? 176
         : t == Q6_K ? 210 : 0;
}

inline bool supported(int t) { return block_size(t) != 0; }

inline size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

__host__ __device__ inline int64_t row_bytes(int t, int cols) {
    return (int64_t)(cols / block_size(t)) * block_bytes(t);
}

// A packed quantised matrix family: `count` consecutive [rows x cols]
// tensors of one ggml type starting at `base`, `stride` bytes apart.
struct QMat {
    const uint8_t* base;
    int64_t stride;     // bytes per tensor (one expert)
    int64_t row_bytes;  // bytes per row
    int type;
    int rows;
    int cols;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// binary16 round trip with round-to-nearest-even (the F16C conversion with
// rounding control 0 used by the reference, cpp/moe_quant_dot.cpp:8-10).
__device__ __forceinline__ float round16(float v) {
    return __half2float(__float2half_rn(v));
}

__device__ __forceinline__ float ld_f16(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// Copy `bytes` bytes from global to shared memory with all threads of the
// block.  Uses 16-byte vectors when both ends allow it, bytes otherwise.
__device__ __forceinline__ void stage_bytes(uint8_t* dst, const uint8_t* src, int64_t bytes) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if ((((uintptr_t)src | (uintptr_t)dst) & 15u) == 0) {
        const int64_t nv = bytes >> 4;
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(dst);
        for (int64_t i = tid; i < nv; i += nt) d4[i] = __ldg(s4 + i);
        for (int64_t i = (nv << 4) + tid; i < bytes; i += nt) dst[i] = src[i];
    } else {
        for (int64_t i = tid; i < bytes; i += nt) dst[i] = src[i];
    }
}

}  // namespace moeb200
