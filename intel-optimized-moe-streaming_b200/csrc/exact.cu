// exact.cu -- the exact expert engine.
//
// Every weight is dequantised bit-identically to the reference decoder and
// folded into an fp32 fused multiply-add, the arithmetic of the reference's
// quant_dot (cpp/moe_quant_dot.cpp:143-169) with a different (warp tree)
// summation order.  It implements moe_quant_expert in both fp16_graph modes
// and any hidden/intermediate size up to 65536, so it reads weights and
// activations straight from global memory (L1-cached) instead of staging
// them in shared memory.  It is the compatibility and cross-check engine;
// the fast decode engine is in decode.cu.
//
//  k_gateup: one CTA per (token, slot, 16-row tile); one warp per row pair
//            computes g and u, then the SwiGLU activation (reference
//            moe_quant_dot.cpp:196-206, shared expert shared_expert.py:247-249).
//  k_down:   one CTA per (token, 8-row tile); one warp per output row sums
//            weight_k * down_k(a_k) over the slots in top-k order, then adds
//            sigmoid-gate * shared_down(a_s) (moe_layer.py:70-105).
#include <math.h>

#include "kquant.cuh"
#include "launch.h"

namespace moeb200 {

constexpr int kGateUpRows = 16;

template <bool ROUND>
__device__ __forceinline__ float row_dot(int type, const uint8_t* __restrict__ row,
                                         const float* __restrict__ x, int cols, int lane) {
    const int bs = block_size(type), pb = block_bytes(type), spb = bs >> 3;
    const int nsub = cols >> 3;
    float acc = 0.f;
    for (int s = lane; s < nsub; s += 32) {
        const int blk = s / spb, sub = s - blk * spb;
        float w[8];
        decode8_any(type, row + (int64_t)blk * pb, sub, w);
        const float4 xa = __ldg(reinterpret_cast<const float4*>(x + 8 * s));
        const float4 xb = __ldg(reinterpret_cast<const float4*>(x + 8 * s + 4));
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float wk = ROUND ? round16(w[k]) : w[k];
            const float xk = ROUND ? round16(xv[k]) : xv[k];
            acc = fmaf(wk, xk, acc);
        }
    }
    return warp_sum(acc);
}

__device__ __forceinline__ int slot_expert(const ExactPlan& p, int t, int k) {
    return p.ids ? p.ids[(size_t)t * p.K + k] : 0;
}

__device__ __forceinline__ bool held(const ExactPlan& p, int e) {
    return e >= p.expert_begin && e < p.expert_begin + p.expert_count;
}

template <bool ROUND>
__global__ void __launch_bounds__(256) k_gateup(ExactPlan p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x, t = item / (p.K + 1), slot = item % (p.K + 1);
    const bool shared = slot == p.K;
    if (shared && p.sgate.base == nullptr) return;
    const int rows = shared ? p.Is : p.I;
    const int r0 = blockIdx.y * kGateUpRows;
    if (r0 >= rows) return;
    const QMat& G = shared ? p.sgate : p.gate;
    const QMat& U = shared ? p.sup : p.up;
    int64_t e = 0;
    if (!shared) {
        const int ge = slot_expert(p, t, slot);
        if (!held(p, ge)) return;
        e = ge - p.expert_begin;
    }
    const float* x = p.x + (size_t)t * p.H;
    const uint8_t* gbase = G.base + e * G.stride;
    const uint8_t* ubase = U.base + e * U.stride;
    for (int rr = warp; rr < kGateUpRows && r0 + rr < rows; rr += 8) {
        const int r = r0 + rr;
        const bool rnd = ROUND && !shared;
        float g, u;
        if (rnd) {
            g = round16(row_dot<true>(G.type, gbase + (int64_t)r * G.row_bytes, x, p.H, lane));
            u = round16(row_dot<true>(U.type, ubase + (int64_t)r * U.row_bytes, x, p.H, lane));
        } else {
            g = row_dot<false>(G.type, gbase + (int64_t)r * G.row_bytes, x, p.H, lane);
            u = row_dot<false>(U.type, ubase + (int64_t)r * U.row_bytes, x, p.H, lane);
        }
        if (lane == 0) {
            float a;
            if (shared) {
                // _sigmoid of the reference shared expert (shared_expert.py:55-62)
                float sgm;
                if (g >= 0.f) {
                    sgm = 1.0f / (1.0f + expf(-g));
                } else {
                    const float ee = expf(g);
                    sgm = ee / (1.0f + ee);
                }
                a = (g * sgm) * u;
            } else if (rnd) {
                const float sgm = round16(1.0f / (1.0f + expf(-g)));
                const float silu = round16(g * sgm);
                a = round16(silu * u);
            } else {
                const float sgm = 1.0f / (1.0f + expf(-g));
                a = (g * sgm) * u;
            }
            p.act[(size_t)item * p.Imax + r] = a;
        }
    }
}

template <bool ROUND>
__global__ void __launch_bounds__(256) k_down(ExactPlan p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x, h = blockIdx.y * 8 + warp;
    if (h >= p.H) return;
    float combined = 0.f;
    for (int k = 0; k < p.K; ++k) {
        const int ge = slot_expert(p, t, k);
        if (!held(p, ge)) continue;
        const int64_t e = ge - p.expert_begin;
        const float* a = p.act + ((size_t)t * (p.K + 1) + k) * p.Imax;
        float v = row_dot<ROUND>(p.down.type,
                                 p.down.base + e * p.down.stride + (int64_t)h * p.down.row_bytes,
                                 a, p.I, lane);
        if (ROUND) v = round16(v);
        const float wk = p.w ? p.w[(size_t)t * p.K + k] : 1.0f;
        combined = __fadd_rn(combined, __fmul_rn(wk, v));
    }
    if (p.sdown.base != nullptr) {
        const float* a = p.act + ((size_t)t * (p.K + 1) + p.K) * p.Imax;
        const float v = row_dot<false>(p.sdown.type, p.sdown.base + (int64_t)h * p.sdown.row_bytes,
                                       a, p.Is, lane);
        combined = __fadd_rn(combined, __fmul_rn(p.sg[t], v));
    }
    if (lane == 0) p.y[(size_t)t * p.H + h] = combined;
}

cudaError_t launch_exact(const ExactPlan& p, cudaStream_t stream) {
    if (p.T <= 0) return cudaSuccess;
    dim3 g1(p.T * (p.K + 1), (p.Imax + kGateUpRows - 1) / kGateUpRows);
    dim3 g2(p.T, (p.H + 7) / 8);
    if (p.round16) {
        k_gateup<true><<<g1, 256, 0, stream>>>(p);
        k_down<true><<<g2, 256, 0, stream>>>(p);
    } else {
        k_gateup<false><<<g1, 256, 0, stream>>>(p);
        k_down<false><<<g2, 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace moeb200
