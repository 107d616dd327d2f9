// qdot.cuh -- integer dot products of packed GGUF rows with a quantised
// activation vector (the fast decode engine).
//
// Activation vectors are quantised per 256-value block b to 16-bit fixed
// point, s_b = amax_b / 32512, q = rint(v / s_b), and split into two signed
// bytes q = 256*hi + lo (lo in [-128, 127], hi in [-127, 127]).  Weights are
// unpacked to their small integer codes u (Q3_K: 0..7, Q4_K: 0..15, Q5_K:
// 0..31, Q6_K: 0..63, Q8_0: the int8 itself) four per 32-bit word, and
// dp4a accumulates sum(u*hi) and sum(u*lo) exactly in int32.  Each format's
// block scales are applied to those exact integer sums:
//   Q3_K: d * s_b * sum_j sc_j * (S_j - 4 * X_j)        (u = q + 4)
//   Q4_K: s_b * (d * sum_j sc_j S_j - dmin * sum_j m_j X_j)
//   Q5_K: as Q4_K
//   Q6_K: d * s_b * sum_j sc_j * (S_j - 32 * X_j)       (u = q + 32)
//   Q8_0: s_b * sum_G d_G * S_G
// with S = 256*sum(u*hi) + sum(u*lo) and X the matching sums of the
// activation codes (precomputed per 8 values).  The only rounding beyond
// fp32 arithmetic is the activation quantisation (~2^-16 of the block
// maximum per value).
//
// Lane mapping (shared by every format): a lane owns "pair" p = (b, o) of a
// row -- block b (256 values; for Q8_0 eight consecutive 34-byte blocks) and
// octet o in 0..3 -- i.e. the 64 values 256*b + 32*G + 8*o + e,
// G = 0..7, e = 0..7.  For Q3_K/Q4_K/Q5_K/Q6_K those are exactly the values
// whose quant bits share bytes in the block layout (see kquant.cuh), so one
// lane reads each packed byte once.
#pragma once

#include "common.cuh"
#include "kquant.cuh"

namespace moeb200 {

struct QVec {
    int8_t* hi;
    int8_t* lo;
    float* s;     // [n/256] block scales
    int16_t* oh;  // [n/8] octet sums of hi
    int16_t* ol;  // [n/8] octet sums of lo
};

// Bytes of shared memory a QVec of n values uses (16-byte multiple).
__host__ __device__ constexpr uint32_t qvec_bytes(int n) {
    return (uint32_t)(2 * n + 4 * (n / 256) + 4 * (n / 8) + 15) & ~15u;
}

__device__ __forceinline__ QVec qvec_at(uint8_t* base, int n) {
    QVec q;
    q.hi = reinterpret_cast<int8_t*>(base);
    q.lo = reinterpret_cast<int8_t*>(base + n);
    q.s = reinterpret_cast<float*>(base + 2 * n);
    q.oh = reinterpret_cast<int16_t*>(base + 2 * n + 4 * (n / 256));
    q.ol = q.oh + n / 8;
    return q;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Quantise 256-value block b of an fp32 vector in shared memory with one
// warp: lane l takes values 8l..8l+7 (octet l).  No block-wide barrier; the
// caller synchronises before the codes are read.
__device__ __forceinline__ void quantize_block_warp(const float* v, QVec q, int b) {
    const int lane = threadIdx.x & 31;
    const float4 a0 = *reinterpret_cast<const float4*>(v + 256 * b + 8 * lane);
    const float4 a1 = *reinterpret_cast<const float4*>(v + 256 * b + 8 * lane + 4);
    const float vals[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(vals[e]));
    m = warp_max(m);
    float iv;
    if (!(m <= 3.0e38f)) {  // inf / nan in the block: propagate as nan
        iv = 0.f;
        if (lane == 0) q.s[b] = __int_as_float(0x7fc00000);
    } else {
        iv = m > 0.f ? 32512.f / m : 0.f;
        if (lane == 0) q.s[b] = m / 32512.f;
    }
    int sh = 0, sl = 0;
    uint32_t ph[2] = {0, 0}, pl[2] = {0, 0};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        int qv = __float2int_rn(vals[e] * iv);
        qv = max(-32512, min(32512, qv));
        const int lo = ((qv + 128) & 255) - 128;
        const int hi = (qv - lo) >> 8;
        sh += hi;
        sl += lo;
        ph[e >> 2] |= (uint32_t)(hi & 255) << (8 * (e & 3));
        pl[e >> 2] |= (uint32_t)(lo & 255) << (8 * (e & 3));
    }
    const int oc = 32 * b + lane;
    *reinterpret_cast<uint2*>(q.hi + 8 * oc) = make_uint2(ph[0], ph[1]);
    *reinterpret_cast<uint2*>(q.lo + 8 * oc) = make_uint2(pl[0], pl[1]);
    q.oh[oc] = (int16_t)sh;
    q.ol[oc] = (int16_t)sl;
}

// One lane's 64 activation codes of pair (b, o), in registers.
struct XLane {
    uint32_t h[8][2];
    uint32_t l[8][2];
    int32_t sh8[8];
    int32_t sl8[8];
    float s;
    __device__ __forceinline__ uint2 h2(int G) const { return make_uint2(h[G][0], h[G][1]); }
    __device__ __forceinline__ uint2 l2(int G) const { return make_uint2(l[G][0], l[G][1]); }
    __device__ __forceinline__ int sh(int G) const { return sh8[G]; }
    __device__ __forceinline__ int sl(int G) const { return sl8[G]; }
};

__device__ __forceinline__ void load_xlane(XLane& x, const QVec& v, int b, int o) {
#pragma unroll
    for (int G = 0; G < 8; ++G) {
        const int base = 256 * b + 32 * G + 8 * o;
        const uint2 hh = *reinterpret_cast<const uint2*>(v.hi + base);
        const uint2 ll = *reinterpret_cast<const uint2*>(v.lo + base);
        x.h[G][0] = hh.x;
        x.h[G][1] = hh.y;
        x.l[G][0] = ll.x;
        x.l[G][1] = ll.y;
        x.sh8[G] = v.oh[base >> 3];
        x.sl8[G] = v.ol[base >> 3];
    }
    x.s = v.s[b];
}

__device__ __forceinline__ uint32_t ld32(const uint8_t* p) {
    return *reinterpret_cast<const uint32_t*>(p);
}

// 32-bit load from a 2-byte aligned shared address.
__device__ __forceinline__ uint32_t ld32a2(const uint8_t* p) {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
    return (uint32_t)q[0] | ((uint32_t)q[1] << 16);
}

__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) {
    return __dp4a((int)a, (int)b, c);
}

// ---- per-format partial dot of one lane's 64 values (block pointer bp) ----

__device__ __forceinline__ float qdot_q3k(const uint8_t* bp, int o, const XLane& x) {
    const uint32_t hm0 = ld32a2(bp + 8 * o), hm1 = ld32a2(bp + 8 * o + 4);
    const uint32_t qa0 = ld32a2(bp + 32 + 8 * o), qa1 = ld32a2(bp + 36 + 8 * o);
    const uint32_t qb0 = ld32a2(bp + 64 + 8 * o), qb1 = ld32a2(bp + 68 + 8 * o);
    const uint8_t* s = bp + 96;
    const int jo = o >> 1;
    int ah = 0, al = 0;
#pragma unroll
    for (int G = 0; G < 8; ++G) {
        const uint32_t q0 = G < 4 ? qa0 : qb0, q1 = G < 4 ? qa1 : qb1;
        const int sh = 2 * (G & 3);
        const uint32_t u0 = ((q0 >> sh) & 0x03030303u) | (((hm0 >> G) & 0x01010101u) << 2);
        const uint32_t u1 = ((q1 >> sh) & 0x03030303u) | (((hm1 >> G) & 0x01010101u) << 2);
        const uint2 xh = x.h2(G), xl = x.l2(G);
        const int h = dp4(u1, xh.y, dp4(u0, xh.x, 0));
        const int l = dp4(u1, xl.y, dp4(u0, xl.x, 0));
        const int sc = q3_scale(s, 2 * G + jo);
        ah += sc * (h - 4 * x.sh(G));
        al += sc * (l - 4 * x.sl(G));
    }
    return ld_f16(bp + 108) * x.s * fmaf(256.f, (float)ah, (float)al);
}

__device__ __forceinline__ float qdot_q4k(const uint8_t* bp, int o, const XLane& x) {
    int ah = 0, al = 0, mh = 0, ml = 0;
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
        const uint32_t w0 = ld32(bp + 16 + 32 * pp + 8 * o), w1 = ld32(bp + 20 + 32 * pp + 8 * o);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int G = 2 * pp + hf;
            const uint32_t u0 = (w0 >> (4 * hf)) & 0x0F0F0F0Fu, u1 = (w1 >> (4 * hf)) & 0x0F0F0F0Fu;
            const uint2 xh = x.h2(G), xl = x.l2(G);
            const int h = dp4(u1, xh.y, dp4(u0, xh.x, 0));
            const int l = dp4(u1, xl.y, dp4(u0, xl.x, 0));
            int sc, mn;
            k4_scale_min(bp + 4, G, sc, mn);
            ah += sc * h;
            al += sc * l;
            mh += mn * x.sh(G);
            ml += mn * x.sl(G);
        }
    }
    const float a = fmaf(256.f, (float)ah, (float)al);
    const float m = fmaf(256.f, (float)mh, (float)ml);
    return x.s * (ld_f16(bp) * a - ld_f16(bp + 2) * m);
}

__device__ __forceinline__ float qdot_q5k(const uint8_t* bp, int o, const XLane& x) {
    const uint32_t qh0 = ld32(bp + 16 + 8 * o), qh1 = ld32(bp + 20 + 8 * o);
    int ah = 0, al = 0, mh = 0, ml = 0;
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
        const uint32_t w0 = ld32(bp + 48 + 32 * pp + 8 * o), w1 = ld32(bp + 52 + 32 * pp + 8 * o);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int G = 2 * pp + hf;
            const uint32_t u0 = ((w0 >> (4 * hf)) & 0x0F0F0F0Fu) | (((qh0 >> G) & 0x01010101u) << 4);
            const uint32_t u1 = ((w1 >> (4 * hf)) & 0x0F0F0F0Fu) | (((qh1 >> G) & 0x01010101u) << 4);
            const uint2 xh = x.h2(G), xl = x.l2(G);
            const int h = dp4(u1, xh.y, dp4(u0, xh.x, 0));
            const int l = dp4(u1, xl.y, dp4(u0, xl.x, 0));
            int sc, mn;
            k4_scale_min(bp + 4, G, sc, mn);
            ah += sc * h;
            al += sc * l;
            mh += mn * x.sh(G);
            ml += mn * x.sl(G);
        }
    }
    const float a = fmaf(256.f, (float)ah, (float)al);
    const float m = fmaf(256.f, (float)mh, (float)ml);
    return x.s * (ld_f16(bp) * a - ld_f16(bp + 2) * m);
}

__device__ __forceinline__ float qdot_q6k(const uint8_t* bp, int o, const XLane& x) {
    const uint32_t ha0 = ld32a2(bp + 128 + 8 * o), ha1 = ld32a2(bp + 132 + 8 * o);
    const uint32_t hb0 = ld32a2(bp + 160 + 8 * o), hb1 = ld32a2(bp + 164 + 8 * o);
    const int8_t* sc = reinterpret_cast<const int8_t*>(bp + 192);
    const int jo = o >> 1;
    int ah = 0, al = 0;
#pragma unroll
    for (int G = 0; G < 8; ++G) {
        const uint8_t* lp = bp + 64 * (G >> 2) + 32 * (G & 1) + 8 * o;
        const uint32_t w0 = ld32a2(lp), w1 = ld32a2(lp + 4);
        const int ns = 4 * ((G >> 1) & 1), hs = 2 * (G & 3);
        const uint32_t h0 = G < 4 ? ha0 : hb0, h1 = G < 4 ? ha1 : hb1;
        const uint32_t u0 = ((w0 >> ns) & 0x0F0F0F0Fu) | (((h0 >> hs) & 0x03030303u) << 4);
        const uint32_t u1 = ((w1 >> ns) & 0x0F0F0F0Fu) | (((h1 >> hs) & 0x03030303u) << 4);
        const uint2 xh = x.h2(G), xl = x.l2(G);
        const int h = dp4(u1, xh.y, dp4(u0, xh.x, 0));
        const int l = dp4(u1, xl.y, dp4(u0, xl.x, 0));
        const int s8 = sc[2 * G + jo];
        ah += s8 * (h - 32 * x.sh(G));
        al += s8 * (l - 32 * x.sl(G));
    }
    return ld_f16(bp + 208) * x.s * fmaf(256.f, (float)ah, (float)al);
}

// Q8_0: bp points at 8 consecutive 34-byte blocks (256 values).
__device__ __forceinline__ float qdot_q8_0(const uint8_t* bp, int o, const XLane& x) {
    float acc = 0.f;
#pragma unroll
    for (int G = 0; G < 8; ++G) {
        const uint8_t* qb = bp + 34 * G;
        const uint32_t q0 = ld32a2(qb + 2 + 8 * o), q1 = ld32a2(qb + 6 + 8 * o);
        const uint2 xh = x.h2(G), xl = x.l2(G);
        const int h = dp4(q1, xh.y, dp4(q0, xh.x, 0));
        const int l = dp4(q1, xl.y, dp4(q0, xl.x, 0));
        acc = fmaf(ld_f16(qb), fmaf(256.f, (float)h, (float)l), acc);
    }
    return x.s * acc;
}

// Bytes of one 256-value column block of a row of `type`.
__host__ __device__ constexpr int block256_bytes(int type) {
    return type == Q8_0 ? 8 * 34 : block_bytes(type);
}

// Lane partial of pair (b, o) of a packed row in shared memory.
__device__ __forceinline__ float qdot_pair(int type, const uint8_t* row, int b, int o,
                                           const XLane& x) {
    const uint8_t* bp = row + b * block256_bytes(type);
    switch (type) {
        case Q3_K: return qdot_q3k(bp, o, x);
        case Q4_K: return qdot_q4k(bp, o, x);
        case Q5_K: return qdot_q5k(bp, o, x);
        case Q6_K: return qdot_q6k(bp, o, x);
        default:   return qdot_q8_0(bp, o, x);
    }
}

// Compile-time format when T >= 0 (one decoder inlined), runtime switch on
// `rt` when T < 0.
template <int T>
__device__ __forceinline__ float qdot_t(int rt, const uint8_t* row, int b, int o, const XLane& x) {
    if constexpr (T < 0) {
        return qdot_pair(rt, row, b, o, x);
    } else {
        const uint8_t* bp = row + b * block256_bytes(T);
        if constexpr (T == Q3_K) return qdot_q3k(bp, o, x);
        else if constexpr (T == Q4_K) return qdot_q4k(bp, o, x);
        else if constexpr (T == Q5_K) return qdot_q5k(bp, o, x);
        else if constexpr (T == Q6_K) return qdot_q6k(bp, o, x);
        else return qdot_q8_0(bp, o, x);
    }
}

// Sum over the `lpr` consecutive lanes of a row group (lpr a power of two).
__device__ __forceinline__ float group_sum(float v, int lpr) {
    for (int off = lpr >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

}  // namespace moeb200
