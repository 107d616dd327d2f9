// dequant.cu -- GGUF K-quant blocks -> fp32 / binary16 on the device.
//
// Device form of the reference's dequant_k (cpp/dequant_k.cpp:350-394).
// The work unit is a chunk of 2048 output values (8 K-quant blocks or 64
// Q8_0 blocks, a whole multiple of 16 bytes for every format).  A CTA stages
// one chunk's packed bytes into shared memory with 16-byte loads, then each of
// its 256 threads decodes 8 consecutive values and writes them with one or
// two 16-byte stores, so both the read and the write streams are coalesced.
// The kernel is bound by HBM writes (4 or 2 output bytes per value against
// 0.43-1.06 input bytes).
#include "common.cuh"
#include "kquant.cuh"
#include "launch.h"

namespace moeb200 {

__device__ __forceinline__ void store8(float* dst, const float* w, bool vec) {
    if (vec) {
        reinterpret_cast<float4*>(dst)[0] = make_float4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(w[4], w[5], w[6], w[7]);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) dst[k] = w[k];
    }
}

__device__ __forceinline__ void store8(__half* dst, const float* w, bool vec) {
    __half h[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) h[k] = __float2half_rn(w[k]);
    if (vec) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) dst[k] = h[k];
    }
}

template <int T, typename OutT>
__global__ void __launch_bounds__(256) k_dequant(const uint8_t* __restrict__ src,
                                                 OutT* __restrict__ dst, int64_t nblocks) {
    constexpr int BS = block_size(T), PB = block_bytes(T);
    constexpr int BPC = 2048 / BS;
    __shared__ __align__(16) uint8_t sm[BPC * PB];
    const bool vec = ((uintptr_t)dst & 15u) == 0;
    const int64_t nchunks = (nblocks + BPC - 1) / BPC;
    for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
        const int64_t b0 = c * BPC;
        const int nb = (int)min((int64_t)BPC, nblocks - b0);
        __syncthreads();
        stage_bytes(sm, src + b0 * PB, (int64_t)nb * PB);
        __syncthreads();
        const int v0 = threadIdx.x * 8;
        const int blk = v0 / BS;
        if (blk < nb) {
            float w[8];
            decode8<T>(sm + blk * PB, (v0 % BS) / 8, w);
            store8(dst + b0 * BS + v0, w, vec);
        }
    }
}

template <typename OutT>
static cudaError_t launch_dequant_t(int type, const uint8_t* src, OutT* dst, int64_t nblocks,
                                    cudaStream_t stream) {
    const int bpc = 2048 / block_size(type);
    const int64_t nchunks = (nblocks + bpc - 1) / bpc;
    const int grid = (int)(nchunks < (int64_t)sm_count() * 8 ? nchunks : (int64_t)sm_count() * 8);
    switch (type) {
        case Q8_0: k_dequant<Q8_0, OutT><<<grid, 256, 0, stream>>>(src, dst, nblocks); break;
        case Q3_K: k_dequant<Q3_K, OutT><<<grid, 256, 0, stream>>>(src, dst, nblocks); break;
        case Q4_K: k_dequant<Q4_K, OutT><<<grid, 256, 0, stream>>>(src, dst, nblocks); break;
        case Q5_K: k_dequant<Q5_K, OutT><<<grid, 256, 0, stream>>>(src, dst, nblocks); break;
        case Q6_K: k_dequant<Q6_K, OutT><<<grid, 256, 0, stream>>>(src, dst, nblocks); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant(int type, const void* src, void* dst, int64_t n, bool f16,
                           cudaStream_t stream) {
    const int64_t nblocks = n / block_size(type);
    if (nblocks <= 0) return cudaSuccess;
    const uint8_t* s = static_cast<const uint8_t*>(src);
    return f16 ? launch_dequant_t(type, s, static_cast<__half*>(dst), nblocks, stream)
               : launch_dequant_t(type, s, static_cast<float*>(dst), nblocks, stream);
}

}  // namespace moeb200
