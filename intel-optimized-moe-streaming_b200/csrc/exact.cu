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
//  k_gateup: one CTA per (token, slot, 8-row tile); one warp per row pair
//            computes g and u (one loop over both rows when they share a
//            format, the quant bytes read as 8-byte runs), then the SwiGLU
//            activation (reference
//            moe_quant_dot.cpp:196-206, shared expert shared_expert.py:247-249).
//  k_down:   one CTA per (token, 8-row tile); one warp per output row sums
//            weight_k * down_k(a_k) over the slots in top-k order, then adds
//            sigmoid-gate * shared_down(a_s) (moe_layer.py:70-105).
#include <math.h>

#include "kquant.cuh"
#include "launch.h"

namespace moeb200 {

constexpr int kGateUpRows = 8;  // one row pair per warp

// 8 bytes at a 2-byte aligned address as two little-endian words, by aligned
// loads of exactly those bytes (read-only data: the non-coherent path).
__device__ __forceinline__ uint2 ld8_a2(const uint8_t* p) {
    if (((uintptr_t)p & 3u) == 0) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(p);
        return make_uint2(__ldg(w), __ldg(w + 1));
    }
    const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
    const uint32_t m = __ldg(reinterpret_cast<const uint32_t*>(p + 2));
    return make_uint2((uint32_t)__ldg(h) | (m << 16), (m >> 16) | ((uint32_t)__ldg(h + 3) << 16));
}

__device__ __forceinline__ int byte_of(const uint2 v, int k) {
    return (int)(((k < 4 ? v.x : v.y) >> (8 * (k & 3))) & 0xFFu);
}

// Values 8*sub .. 8*sub+7 of one block: decode8<T>'s arithmetic (the same
// roundings in the same order, so the same bits), with the eight quant
// bytes (and Q5_K/Q6_K/Q3_K's high-bit bytes) read as two words.  Every
// such run starts at an even offset of a 2-byte aligned block.
template <int T>
__device__ __forceinline__ void lane8(const uint8_t* b, int sub, float* w);

template <>
__device__ __forceinline__ void lane8<Q8_0>(const uint8_t* b, int sub, float* w) {
    const float d = ld_f16(b);
    const uint2 q = ld8_a2(b + 2 + 8 * sub);
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = __fmul_rn((float)(int8_t)byte_of(q, j), d);
}

template <>
__device__ __forceinline__ void lane8<Q4_K>(const uint8_t* b, int sub, float* w) {
    const int i0 = 8 * sub, j = i0 >> 5;
    int sc, mn;
    k4_scale_min(b + 4, j, sc, mn);
    const float d1 = __fmul_rn(ld_f16(b), (float)sc);
    const float m1 = __fmul_rn(ld_f16(b + 2), (float)mn);
    const uint2 q = ld8_a2(b + 16 + 32 * (i0 >> 6) + (i0 & 31));
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = __fsub_rn(__fmul_rn(d1, (float)((byte_of(q, k) >> sh) & 15)), m1);
}

template <>
__device__ __forceinline__ void lane8<Q5_K>(const uint8_t* b, int sub, float* w) {
    const int i0 = 8 * sub, j = i0 >> 5;
    int sc, mn;
    k4_scale_min(b + 4, j, sc, mn);
    const float dsc = __fmul_rn(ld_f16(b), (float)sc);
    const float m1 = __fmul_rn(ld_f16(b + 2), (float)mn);
    const uint2 q = ld8_a2(b + 48 + 32 * (i0 >> 6) + (i0 & 31));
    const uint2 qh = ld8_a2(b + 16 + (i0 & 31));
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int v = ((byte_of(q, k) >> sh) & 15) | (((byte_of(qh, k) >> j) & 1) << 4);
        w[k] = __fsub_rn(__fmul_rn(dsc, (float)v), m1);
    }
}

template <>
__device__ __forceinline__ void lane8<Q6_K>(const uint8_t* b, int sub, float* w) {
    const int i0 = 8 * sub;
    const float ds = __fmul_rn(ld_f16(b + 208), (float)(int8_t)b[192 + (i0 >> 4)]);
    const uint2 ql = ld8_a2(b + 64 * (i0 >> 7) + (i0 & 63));
    const uint2 qh = ld8_a2(b + 128 + 32 * (i0 >> 7) + (i0 & 31));
    const int sl = ((i0 >> 6) & 1) * 4, shh = ((i0 >> 5) & 3) * 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int v = (((byte_of(ql, k) >> sl) & 15) | (((byte_of(qh, k) >> shh) & 3) << 4)) - 32;
        w[k] = __fmul_rn(ds, (float)v);
    }
}

template <>
__device__ __forceinline__ void lane8<Q3_K>(const uint8_t* b, int sub, float* w) {
    const int i0 = 8 * sub, g = i0 >> 5;
    const float ds = __fmul_rn(ld_f16(b + 108), (float)q3_scale(b + 96, i0 >> 4));
    const uint2 ql = ld8_a2(b + 32 + 32 * (i0 >> 7) + (i0 & 31));
    const uint2 hm = ld8_a2(b + (i0 & 31));
    const int sl = 2 * (g & 3);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int v = ((byte_of(ql, k) >> sl) & 3) - ((((byte_of(hm, k) >> g) & 1) ^ 1) << 2);
        w[k] = __fmul_rn(ds, (float)v);
    }
}

// Dots of NR rows of format T with x (fp32 FMA, each lane summing its
// 8-value runs s = lane, lane + 32, ... in order, then a warp tree).  The
// rows share the loop so their loads overlap.
template <int T, bool ROUND, int NR>
__device__ __forceinline__ void rows_dot_t(const uint8_t* const (&rows)[NR],
                                           const float* __restrict__ x, int cols, int lane,
                                           float (&out)[NR]) {
    constexpr int spb = block_size(T) >> 3, pb = block_bytes(T);
    const int nsub = cols >> 3;
    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.f;
#pragma unroll 4
    for (int s = lane; s < nsub; s += 32) {
        const int blk = s / spb, sub = s - blk * spb;
        const float4 xa = __ldg(reinterpret_cast<const float4*>(x + 8 * s));
        const float4 xb = __ldg(reinterpret_cast<const float4*>(x + 8 * s + 4));
        float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        if (ROUND) {
#pragma unroll
            for (int k = 0; k < 8; ++k) xv[k] = round16(xv[k]);
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            float w[8];
            lane8<T>(rows[r] + (int64_t)blk * pb, sub, w);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[r] = fmaf(ROUND ? round16(w[k]) : w[k], xv[k], acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < NR; ++r) out[r] = warp_sum(acc[r]);
}

template <bool ROUND, int NR>
__device__ __forceinline__ void rows_dot(int type, const uint8_t* const (&rows)[NR],
                                         const float* __restrict__ x, int cols, int lane,
                                         float (&out)[NR]) {
    switch (type) {
        case Q8_0: rows_dot_t<Q8_0, ROUND, NR>(rows, x, cols, lane, out); break;
        case Q3_K: rows_dot_t<Q3_K, ROUND, NR>(rows, x, cols, lane, out); break;
        case Q4_K: rows_dot_t<Q4_K, ROUND, NR>(rows, x, cols, lane, out); break;
        case Q5_K: rows_dot_t<Q5_K, ROUND, NR>(rows, x, cols, lane, out); break;
        default:   rows_dot_t<Q6_K, ROUND, NR>(rows, x, cols, lane, out); break;
    }
}

// Two rows of format T, row r with its own vector x_r: the same per-row
// arithmetic and order as rows_dot_t, the two rows' loads in one loop.
template <int T, bool ROUND>
__device__ __forceinline__ float2 dot2x_t(const uint8_t* r0, const float* __restrict__ x0,
                                          const uint8_t* r1, const float* __restrict__ x1,
                                          int cols, int lane) {
    constexpr int spb = block_size(T) >> 3, pb = block_bytes(T);
    const int nsub = cols >> 3;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 2
    for (int s = lane; s < nsub; s += 32) {
        const int blk = s / spb, sub = s - blk * spb;
        const float4 p0 = __ldg(reinterpret_cast<const float4*>(x0 + 8 * s));
        const float4 q0 = __ldg(reinterpret_cast<const float4*>(x0 + 8 * s + 4));
        const float4 p1 = __ldg(reinterpret_cast<const float4*>(x1 + 8 * s));
        const float4 q1 = __ldg(reinterpret_cast<const float4*>(x1 + 8 * s + 4));
        const float v0[8] = {p0.x, p0.y, p0.z, p0.w, q0.x, q0.y, q0.z, q0.w};
        const float v1[8] = {p1.x, p1.y, p1.z, p1.w, q1.x, q1.y, q1.z, q1.w};
        float w0[8], w1[8];
        lane8<T>(r0 + (int64_t)blk * pb, sub, w0);
        lane8<T>(r1 + (int64_t)blk * pb, sub, w1);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            a0 = fmaf(ROUND ? round16(w0[k]) : w0[k], ROUND ? round16(v0[k]) : v0[k], a0);
            a1 = fmaf(ROUND ? round16(w1[k]) : w1[k], ROUND ? round16(v1[k]) : v1[k], a1);
        }
    }
    return make_float2(warp_sum(a0), warp_sum(a1));
}

template <bool ROUND>
__device__ __forceinline__ float2 dot2x(int type, const uint8_t* r0, const float* x0,
                                        const uint8_t* r1, const float* x1, int cols, int lane) {
    switch (type) {
        case Q8_0: return dot2x_t<Q8_0, ROUND>(r0, x0, r1, x1, cols, lane);
        case Q3_K: return dot2x_t<Q3_K, ROUND>(r0, x0, r1, x1, cols, lane);
        case Q4_K: return dot2x_t<Q4_K, ROUND>(r0, x0, r1, x1, cols, lane);
        case Q5_K: return dot2x_t<Q5_K, ROUND>(r0, x0, r1, x1, cols, lane);
        default:   return dot2x_t<Q6_K, ROUND>(r0, x0, r1, x1, cols, lane);
    }
}

template <bool ROUND>
__device__ __forceinline__ float row_dot(int type, const uint8_t* __restrict__ row,
                                         const float* __restrict__ x, int cols, int lane) {
    const uint8_t* const rows[1] = {row};
    float out[1];
    rows_dot<ROUND, 1>(type, rows, x, cols, lane, out);
    return out[0];
}

// The gate and the up row of one intermediate row: one loop when they share
// a format.
template <bool ROUND>
__device__ __forceinline__ void gate_up_dot(int gt, const uint8_t* g, int ut, const uint8_t* u,
                                            const float* __restrict__ x, int cols, int lane,
                                            float& gv, float& uv) {
    if (gt == ut) {
        const uint8_t* const rows[2] = {g, u};
        float out[2];
        rows_dot<ROUND, 2>(gt, rows, x, cols, lane, out);
        gv = out[0];
        uv = out[1];
    } else {
        gv = row_dot<ROUND>(gt, g, x, cols, lane);
        uv = row_dot<ROUND>(ut, u, x, cols, lane);
    }
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
            gate_up_dot<true>(G.type, gbase + (int64_t)r * G.row_bytes, U.type,
                              ubase + (int64_t)r * U.row_bytes, x, p.H, lane, g, u);
            g = round16(g);
            u = round16(u);
        } else {
            gate_up_dot<false>(G.type, gbase + (int64_t)r * G.row_bytes, U.type,
                               ubase + (int64_t)r * U.row_bytes, x, p.H, lane, g, u);
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

// PAIR: two held slots' rows per loop (their loads overlap, at twice the
// registers; for few tokens, where the GPU is latency-bound).
template <bool ROUND, bool PAIR>
__global__ void __launch_bounds__(256) k_down(ExactPlan p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x, h = blockIdx.y * 8 + warp;
    if (h >= p.H) return;
    float combined = 0.f;
    if constexpr (!PAIR) {
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
    } else {
        // the held slots two at a time, combined in top-k order
        int k = 0;
        while (k < p.K) {
            int ks[2];
            int n = 0;
            for (; k < p.K && n < 2; ++k)
                if (held(p, slot_expert(p, t, k))) ks[n++] = k;
            if (n == 0) break;
            const int k1 = n == 2 ? ks[1] : ks[0];
            const int64_t e0 = slot_expert(p, t, ks[0]) - p.expert_begin;
            const int64_t e1 = slot_expert(p, t, k1) - p.expert_begin;
            const float2 d = dot2x<ROUND>(
                p.down.type, p.down.base + e0 * p.down.stride + (int64_t)h * p.down.row_bytes,
                p.act + ((size_t)t * (p.K + 1) + ks[0]) * p.Imax,
                p.down.base + e1 * p.down.stride + (int64_t)h * p.down.row_bytes,
                p.act + ((size_t)t * (p.K + 1) + k1) * p.Imax, p.I, lane);
            const float out[2] = {d.x, d.y};
            for (int i = 0; i < n; ++i) {
                const float v = ROUND ? round16(out[i]) : out[i];
                const float wk = p.w ? p.w[(size_t)t * p.K + ks[i]] : 1.0f;
                combined = __fadd_rn(combined, __fmul_rn(wk, v));
            }
        }
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
    // a few tokens with several slots: paired down rows (B200: the 1-token
    // layer 56 -> 48 us); otherwise one row at a time (more warps resident)
    const bool pair = p.T <= 4 && p.K >= 2;
    if (p.round16) {
        k_gateup<true><<<g1, 256, 0, stream>>>(p);
        if (pair) k_down<true, true><<<g2, 256, 0, stream>>>(p);
        else k_down<true, false><<<g2, 256, 0, stream>>>(p);
    } else {
        k_gateup<false><<<g1, 256, 0, stream>>>(p);
        if (pair) k_down<false, true><<<g2, 256, 0, stream>>>(p);
        else k_down<false, false><<<g2, 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

}  // namespace moeb200
