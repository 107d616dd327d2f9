// block.cu -- the transformer-block steps around a many-token MoE call in
// the identity-mixer stack (reference TransformerBlock.forward with the
// DeltaNet/attention mixer replaced by identity,
// src/flash_moe/transformer.py:229-247; RMSNorm, src/flash_moe/norm.py:21-30,
// weight 1):
//   prepare: h = x + f16(x / rms(x)),  n = f16(h / rms(h))     per token
//   finish:  y = h + f16(m)                                    m = MoE(n)
// with rms(v) = sqrt(mean(v^2) + eps), fp32 reduction, binary16 outputs
// widened back to fp32.  One CTA per token; the reduction order is fixed.
#include "launch.h"

namespace moeb200 {

constexpr int kBlockThreads = 256;

__device__ __forceinline__ float cta_sum(float v, float* part) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) part[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < kBlockThreads / 32; ++i) t += part[i];
    return t;
}

__global__ void __launch_bounds__(kBlockThreads) k_block_prepare(const float* x, float* h, float* n,
                                                                 int H, float eps) {
    __shared__ float part[kBlockThreads / 32];
    const size_t base = (size_t)blockIdx.x * H;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += kBlockThreads) ss = fmaf(x[base + i], x[base + i], ss);
    ss = cta_sum(ss, part);
    const float rms = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)H), eps));
    float ss2 = 0.f;
    for (int i = threadIdx.x; i < H; i += kBlockThreads) {
        const float v = x[base + i];
        const float hv = __fadd_rn(v, round16(__fdiv_rn(v, rms)));
        h[base + i] = hv;
        ss2 = fmaf(hv, hv, ss2);
    }
    ss2 = cta_sum(ss2, part);
    const float rms2 = sqrtf(__fadd_rn(__fdiv_rn(ss2, (float)H), eps));
    for (int i = threadIdx.x; i < H; i += kBlockThreads) n[base + i] = round16(__fdiv_rn(h[base + i], rms2));
}

__global__ void __launch_bounds__(kBlockThreads) k_block_finish(const float* h, const float* m, float* y,
                                                                int H) {
    const size_t base = (size_t)blockIdx.x * H;
    for (int i = threadIdx.x; i < H; i += kBlockThreads)
        y[base + i] = __fadd_rn(h[base + i], round16(m[base + i]));
}

cudaError_t launch_block_prepare(const float* x, float* h, float* n, int T, int H, float eps,
                                 cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    k_block_prepare<<<T, kBlockThreads, 0, s>>>(x, h, n, H, eps);
    return cudaGetLastError();
}

cudaError_t launch_block_finish(const float* h, const float* m, float* y, int T, int H,
                                cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    k_block_finish<<<T, kBlockThreads, 0, s>>>(h, m, y, H);
    return cudaGetLastError();
}

}  // namespace moeb200
