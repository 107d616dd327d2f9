// fused.cuh -- pieces shared by the cooperative decode kernels (decode.cu,
// decode_multi.cu): CTA size, workspace counters, bounded-wait budget and the
// fixed-order reductions.
#pragma once

#include "common.cuh"
#include "sm100.cuh"

namespace moeb200 {

constexpr int kFusedThreads = 512;
constexpr uint32_t kWaitPolls = 1u << 21;
constexpr int kTraceSlots = 32;

// Counters in the first 256 bytes of the workspace (uint32 words); the error
// word sits at byte 32, where moe_b200_workspace_error reads it.  C_SEQ is
// the fused single-token kernel's step sequence number: it only grows (each
// launch adds its step count), so the tag seq + s + 1 of step s never
// repeats on a workspace and a stale exchange word never matches.
enum { C_ROUTER = 0, C_SHARED = 1, C_GATEUP = 2, C_EXIT = 3, C_DONE = 4, C_SEQ = 5, C_ERROR = 8 };

__device__ __forceinline__ int part(int n, int c, int G) { return (int)(((int64_t)n * c) / G); }

__device__ __forceinline__ void set_error(uint32_t* ctr, int code) {
    atomicExch(reinterpret_cast<int*>(ctr + C_ERROR), code);
}

// fp32 row dot with x in shared memory, one warp.
__device__ __forceinline__ float dot_f32_warp(const float* row, const float* x, int n, int lane) {
    float acc = 0.f;
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int i = lane; i < (n >> 2); i += 32) {
        const float4 a = r4[i], b = x4[i];
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
        acc = fmaf(a.z, b.z, acc);
        acc = fmaf(a.w, b.w, acc);
    }
    return warp_sum(acc);
}

// The same dot for a row with no alignment guarantee (scalar loads).
__device__ __forceinline__ float dot_f32_warp_any(const float* row, const float* x, int n, int lane) {
    if ((((uintptr_t)row) & 15u) == 0) return dot_f32_warp(row, x, n, lane);
    float acc = 0.f;
    for (int i = lane; i < n; i += 32) acc = fmaf(row[i], x[i], acc);
    return warp_sum(acc);
}

// Sum of v over the CTA in a fixed order (warp trees, then warps in order);
// every thread gets the result.  `part` holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float* part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) part[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < kFusedThreads / 32; ++i) t += part[i];
    return t;
}

}  // namespace moeb200
