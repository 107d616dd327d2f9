// route.cu -- router scores, top-k selection and routing weights.
//
// Device form of ExpertRouter.scores/route (reference
// src/flash_moe/router.py:140-170) for a batch of tokens, plus the
// shared-expert gate sigmoid(x . w_inp) (src/flash_moe/shared_expert.py:242).
//
//  k_scores: one warp per (token, expert) fp32 dot product over H, 16-byte
//            loads of the [E x H] router rows; + the optional bias.
//  k_topk:   one warp per token.  K rounds of a warp arg-max over the E
//            scores (ties go to the lower expert id), then the softmax over
//            the K selected scores in float64 with numpy's summation order
//            for the denominator, rounded to fp32 as numpy rounds the Python
//            float when it multiplies an fp32 array.
#include <math.h>

#include "launch.h"
#include "topk.cuh"

namespace moeb200 {

__global__ void __launch_bounds__(256) k_scores(RoutePlan p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * 8 + warp, t = blockIdx.y;
    if (e >= p.E) return;
    const float* xr = p.x + (size_t)t * p.H;
    const float* wr = p.router + (size_t)e * p.H;
    float acc = 0.f;
    if ((((uintptr_t)xr | (uintptr_t)wr) & 15u) == 0 && (p.H & 3) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        const float4* w4 = reinterpret_cast<const float4*>(wr);
        for (int i = lane; i < (p.H >> 2); i += 32) {
            const float4 a = __ldg(x4 + i), b = __ldg(w4 + i);
            acc = fmaf(a.x, b.x, acc);
            acc = fmaf(a.y, b.y, acc);
            acc = fmaf(a.z, b.z, acc);
            acc = fmaf(a.w, b.w, acc);
        }
    } else {
        for (int i = lane; i < p.H; i += 32) acc = fmaf(__ldg(xr + i), __ldg(wr + i), acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) {
        if (p.bias) acc = __fadd_rn(acc, p.bias[e]);
        p.scores[(size_t)t * p.E + e] = acc;
    }
}

__global__ void __launch_bounds__(32) k_topk(RoutePlan p) {
    extern __shared__ float s_scores[];
    unsigned char* taken = reinterpret_cast<unsigned char*>(s_scores + p.E);
    const int t = blockIdx.x, lane = threadIdx.x;
    if (p.K > 0 && p.E <= 256) {
        // the same selection and weights from registers (topk.cuh)
        topk_softmax_warp_fast(p.scores + (size_t)t * p.E, p.E, p.K, p.ids + (size_t)t * p.K,
                               p.w + (size_t)t * p.K);
    } else if (p.K > 0) {
        for (int e = lane; e < p.E; e += 32) s_scores[e] = p.scores[(size_t)t * p.E + e];
        __syncwarp();
        topk_softmax_warp(s_scores, taken, p.E, p.K, p.ids + (size_t)t * p.K,
                          p.w + (size_t)t * p.K);
    }
    if (p.gate_inp) {
        // lane-strided, each lane in order (unrolled so the loads overlap)
        const float* xr = p.x + (size_t)t * p.H;
        float acc = 0.f;
#pragma unroll 8
        for (int i = lane; i < p.H; i += 32) acc = fmaf(__ldg(xr + i), __ldg(p.gate_inp + i), acc);
        acc = warp_sum(acc);
        if (lane == 0) p.sg[t] = shared_sigmoid(acc);
    }
}

cudaError_t launch_route(const RoutePlan& p, cudaStream_t stream) {
    if (p.T <= 0) return cudaSuccess;
    if (p.K > 0) {
        dim3 g1((p.E + 7) / 8, p.T);
        k_scores<<<g1, 256, 0, stream>>>(p);
    }
    const size_t sm = (size_t)p.E * sizeof(float) + (size_t)p.E;
    k_topk<<<p.T, 32, sm, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace moeb200
