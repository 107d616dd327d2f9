// kquant.cuh -- exact device decoders for the GGUF K-quant block formats.
//
// decode8<T>(blk, sub, w) writes values 8*sub .. 8*sub+7 of one block.  The
// values are bit-identical to the reference's scalar decoders
// (cpp/dequant_k.cpp:146-298) and to gguf.quants: every product and
// difference is rounded on its own (__fmul_rn / __fsub_rn, never contracted
// into a fused multiply-add) and in the reference's association order,
// (d*scale)*q [- dmin*min].
//
// Block layouts (byte offsets inside one block):
//   Q8_0 34 B : d f16 @0, int8 q[32] @2                      y = q*d
//   Q4_K 144 B: d @0, dmin @2, 12 scale bytes @4, q4[128] @16
//               value i: byte 16 + 32*(i/64) + i%32, high nibble iff (i/32) odd
//               y = (d*sc)*q - dmin*mn, (sc, mn) = six-bit pair i/32
//   Q5_K 176 B: as Q4_K with q4 @48 and bit 4 = bit i/32 of qh[i%32] @16
//   Q6_K 210 B: ql[128] @0, qh[64] @128, int8 scales[16] @192, d @208
//               low4 = ql[64*(i/128) + i%64] >> 4*((i/64)%2)
//               high2 = qh[32*(i/128) + i%32] >> 2*((i/32)%4)
//               y = (d*scale[i/16]) * ((low4 | high2<<4) - 32)
//   Q3_K 110 B: hmask[32] @0, qs[64] @32, 12 scale bytes @96, d @108
//               low2 = qs[32*(i/128) + i%32] >> 2*((i/32)%4)
//               hbit = hmask[i%32] >> (i/32)
//               y = (d*scale[i/16]) * (low2 - 4*(1-hbit))
#pragma once

#include "common.cuh"

namespace moeb200 {

// Six-bit (scale, min) pair j of Q4_K/Q5_K (reference unpack_scale_min_k4,
// cpp/dequant_k.cpp:166-175).
__device__ __forceinline__ void k4_scale_min(const uint8_t* s, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Signed six-bit scale j of Q3_K (reference dequant_q3_k, :284-289).
__device__ __forceinline__ int q3_scale(const uint8_t* s, int j) {
    const int low4 = (j < 8) ? (s[j] & 15) : (s[j - 8] >> 4);
    const int high2 = (s[8 + (j & 3)] >> (2 * (j >> 2))) & 3;
    return (low4 | (high2 << 4)) - 32;
}

template <int T>
__device__ __forceinline__ void decode8(const uint8_t* b, int sub, float* w);

template <>
__device__ __forceinline__ void decode8<Q8_0>(const uint8_t* b, int sub, float* w) {
    const float d = ld_f16(b);
    const int8_t* q = reinterpret_cast<const int8_t*>(b + 2 + 8 * sub);
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = __fmul_rn((float)q[j], d);
}

template <>
__device__ __forceinline__ void decode8<Q4_K>(const uint8_t* b, int sub, float* w) {
    const int i0 = 8 * sub, j = i0 >> 5;
    int sc, mn;
    k4_scale_min(b + 4, j, sc, mn);
    const float d1 = __fmul_rn(ld_f16(b), (float)sc);
    const float m1 = __fmul_rn(ld_f16(b + 2), (float)mn);
    const uint8_t* q = b + 16 + 32 * (i0 >> 6) + (i0 & 31);
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = __fsub_rn(__fmul_rn(d1, (float)((q[k] >> sh) & 15)), m1);
}

template <>
__device__ __forceinline__ void decode8<Q5_K>(const uint8_t* b, int sub, float* w) {
    const int i0 = 8 * sub, j = i0 >> 5;
    int sc, mn;
    k4_scale_min(b + 4, j, sc, mn);
    const float dsc = __fmul_rn(ld_f16(b), (float)sc);
    const float m1 = __fmul_rn(ld_f16(b + 2), (float)mn);
    const uint8_t* q = b + 48 + 32 * (i0 >> 6) + (i0 & 31);
    const uint8_t* qh = b + 16 + (i0 & 31);
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int v = ((q[k] >> sh) & 15) | (((qh[k] >> j) & 1) << 4);
        w[k] = __fsub_rn(__fmul_rn(dsc, (float)v), m1);
    }
}

template <>
__device__ __forceinline__ void decode8<Q6_K>(const uint8_t* b, int sub, float* w) {
    const int i0 = 8 * sub;
    const float ds = __fmul_rn(ld_f16(b + 208), (float)(int8_t)b[192 + (i0 >> 4)]);
    const uint8_t* ql = b + 64 * (i0 >> 7) + (i0 & 63);
    const uint8_t* qh = b + 128 + 32 * (i0 >> 7) + (i0 & 31);
    const int sl = ((i0 >> 6) & 1) * 4, shh = ((i0 >> 5) & 3) * 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int v = (((ql[k] >> sl) & 15) | (((qh[k] >> shh) & 3) << 4)) - 32;
        w[k] = __fmul_rn(ds, (float)v);
    }
}

template <>
__device__ __forceinline__ void decode8<Q3_K>(const uint8_t* b, int sub, float* w) {
    const int i0 = 8 * sub, g = i0 >> 5;
    const float ds = __fmul_rn(ld_f16(b + 108), (float)q3_scale(b + 96, i0 >> 4));
    const uint8_t* ql = b + 32 + 32 * (i0 >> 7) + (i0 & 31);
    const uint8_t* hm = b + (i0 & 31);
    const int sl = 2 * (g & 3);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int v = ((ql[k] >> sl) & 3) - ((((hm[k] >> g) & 1) ^ 1) << 2);
        w[k] = __fmul_rn(ds, (float)v);
    }
}

// Runtime-dispatched form (warp-uniform type).
__device__ __forceinline__ void decode8_any(int t, const uint8_t* b, int sub, float* w) {
    switch (t) {
        case Q8_0: decode8<Q8_0>(b, sub, w); break;
        case Q3_K: decode8<Q3_K>(b, sub, w); break;
        case Q4_K: decode8<Q4_K>(b, sub, w); break;
        case Q5_K: decode8<Q5_K>(b, sub, w); break;
        default:   decode8<Q6_K>(b, sub, w); break;
    }
}

}  // namespace moeb200
